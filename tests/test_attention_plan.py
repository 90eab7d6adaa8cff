"""The tcgen05 attention template's launch plans on the CPU: shared memory, TMEM columns,
the warpgroups' register split and the persistent grid, for the BASELINE configuration,
its per-GPU batch splits and the fixture shapes' families (causal, masked keys, GQA,
smaller head dims)."""

import pytest

from conftest import ROOT  # noqa: F401  (puts the package on sys.path)

SMEM_MAX = 232448


def _cases():
    base = dict(Sq=4096, Sk=4096, D=128)
    out = [dict(BH=256, **base), dict(BH=128, **base), dict(BH=64, **base), dict(BH=32, **base),
           dict(BH=8, Sq=1024, Sk=1024, D=64), dict(BH=4, Sq=512, Sk=640, D=128),
           dict(BH=16, Sq=2048, Sk=2048, D=128, causal=True),
           dict(BH=8, Sq=256, Sk=200, D=96),
           dict(BH=32, Sq=1024, Sk=1024, D=128, heads=8, kv_group=4),
           dict(BH=4, Sq=128, Sk=512, D=128)]
    return out


@pytest.mark.parametrize("case", _cases(), ids=lambda c: "-".join(f"{k}{v}" for k, v in c.items()))
def test_attention_plan_fits(case):
    import math
    from compiler import parse_launch
    from compiler.kernels.attention import AttnConfig, emit_attention_module, register_split
    cfg = AttnConfig(scale=case["D"] ** -0.5, name="k_plan", buffers=("q", "k", "v", "o"), **case)
    text = emit_attention_module(cfg)
    launch = parse_launch(text)
    nq = cfg.NQ
    nthreads = launch["block"][0]
    assert nthreads == 128 * (nq + 1)
    assert launch["smem"] <= SMEM_MAX - 512
    # TMEM: S (128 columns) and O (DP columns) per query tile, allocated as a power of two
    assert nq * (128 + cfg.DP) <= 512
    cap, ctl, soft = register_split(nq)
    assert cap * nthreads <= 65536
    if nq == 2:
        assert 128 * ctl + 128 * nq * soft <= nthreads * cap
        assert ctl % 8 == 0 and soft % 8 == 0 and 24 <= ctl <= soft <= 256
    # persistent grid: one CTA per SM at most, every unit of nq tiles taken
    units = math.ceil(cfg.Sq / (128 * nq)) * cfg.BH
    assert launch["grid"][0] == min(148, units)
    visible = (sum(min(r + 1, cfg.Sk) for r in range(cfg.Sq)) if cfg.causal else cfg.Sq * cfg.Sk)
    assert launch["flops"] == 4 * cfg.BH * visible * cfg.D
