"""The persistent split-key attention schedule (``AttnConfig.schedule = "split_keys"``).

On the CPU: the template assembles for sm_100a without spills and refuses the problems
it does not serve.  On the B200: parity with the f64 oracle (``‖out - ref‖ / ‖ref‖``
within 1e-2 and every element within 4 bf16 ulps of the output's largest magnitude)
on problems that exercise one tile per CTA, several tiles per CTA (a reduced CTA
count), grouped-query heads, ragged tile counts and large scores (rescaling).
"""

import math

import numpy as np
import pytest

from parity import assert_parity


def _cfg(bh, sq, sk, **kw):
    from compiler.kernels.attention import AttnConfig
    return AttnConfig(BH=bh, Sq=sq, Sk=sk, D=128, dtype="bf16", scale=1 / math.sqrt(128),
                      name=f"k_attn_split_{bh}_{sq}_{sk}", buffers=("q", "k", "v", "o"),
                      schedule="split_keys", **kw)


def test_split_schedule_assembles_without_spills():
    import emmyrt
    from compiler.kernels.attention import emit_attention_module
    log = emmyrt.assemble(emit_attention_module(_cfg(256, 4096, 4096)))[1]
    assert "0 bytes spill stores" in log and "0 bytes spill loads" in log, log


@pytest.mark.parametrize("kw", [{"causal": True}, {"mask_param": "m"}, {"kt_layout": True}])
def test_split_schedule_refuses_other_problems(kw):
    from compiler.kernels.attention import emit_attention_module
    with pytest.raises(NotImplementedError):
        emit_attention_module(_cfg(2, 256, 256, **kw))
    with pytest.raises(NotImplementedError):
        emit_attention_module(_cfg(2, 256, 200))        # ragged key blocks


def _run(bh, sq, sk, sms, seed, q_scale=1.0, kv_group=1, heads=0):
    import emmyrt
    from compiler.kernels.attention_split import emit_attention_split_module
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel
    from hostfmt import bf16_bits_to_f32, f32_to_bf16_bits
    cfg = _cfg(bh, sq, sk, kv_group=kv_group, heads=heads)
    ck = CompiledKernel.from_module(emit_attention_split_module(cfg, sms=sms), cfg.name, ["q", "k", "v", "o"])
    rng = np.random.default_rng(seed)
    host = {"q": f32_to_bf16_bits(rng.standard_normal((bh, sq, 128), dtype=np.float32) * np.float32(q_scale)),
            "k": f32_to_bf16_bits(rng.standard_normal((bh // kv_group, sk, 128), dtype=np.float32)),
            "v": f32_to_bf16_bits(rng.standard_normal((bh // kv_group, sk, 128), dtype=np.float32))}
    bufs = {n: DeviceBuffer(a.nbytes) for n, a in host.items()}
    for n, a in host.items():
        bufs[n].upload(a)
    bufs["o"] = DeviceBuffer(bh * sq * 128 * 2)
    bufs["o"].zero()
    ck({n: b.ptr for n, b in bufs.items()})
    emmyrt.stream_wait(0, 60)
    assert ck.status() == 0, f"kernel status {ck.status()}"
    out = np.zeros((bh, sq, 128), np.uint16)
    bufs["o"].download(out)
    for b in bufs.values():
        b.free()
    return bf16_bits_to_f32(out), {n: bf16_bits_to_f32(a) for n, a in host.items()}, cfg


@pytest.mark.gpu
@pytest.mark.parametrize("bh,sq,sk,sms,seed,q_scale,kv_group,heads", [
    (2, 256, 256, 148, 1, 1.0, 1, 0),      # one tile per CTA, two key blocks
    (3, 384, 640, 148, 2, 1.0, 1, 0),      # odd tile and block counts
    (40, 512, 512, 148, 3, 1.0, 1, 0),     # 160 tiles over 148 CTAs: some CTAs take two
    (8, 512, 1024, 5, 4, 1.0, 1, 0),       # 32 tiles over 5 CTAs: 6 or 7 tiles each
    (6, 256, 384, 4, 5, 1.0, 1, 0),        # 12 tiles over 4 CTAs, three key blocks
    (4, 512, 512, 148, 6, 8.0, 1, 0),      # large scores: the running maxima move
    (8, 256, 512, 3, 7, 1.0, 4, 4),        # grouped-query heads, persistent
])
def test_split_schedule_matches_the_oracle(runtime, bh, sq, sk, sms, seed, q_scale, kv_group, heads):
    from oracle.refs import attn_bf16
    got, f, cfg = _run(bh, sq, sk, sms, seed, q_scale, kv_group, heads)
    assert np.isfinite(got).all()
    outs, refs = [], []
    for b in range(bh):
        rows = np.random.default_rng(b).choice(sq, size=min(sq, 24), replace=False)
        kvh = b if kv_group == 1 else (b // heads) * (heads // kv_group) + (b % heads) // kv_group
        outs.append(got[b, rows])
        refs.append(attn_bf16(f["q"][b, rows], f["k"][kvh], f["v"][kvh], cfg.scale))
        assert_parity(outs[-1], refs[-1], rel=1e-2, what=f"batch x head {b}")
    assert_parity(np.concatenate(outs), np.concatenate(refs), rel=1e-2, what="all heads")


def test_schedule_override_applies_only_where_the_split_schedule_serves(monkeypatch):
    """``EMMY_ATTENTION_SCHEDULE=split_keys`` moves the whole compile path (bench.py
    included) onto the split-key schedule for unmasked, non-causal problems and leaves
    every other attention problem on the two-tile template."""
    from compiler.kernels.attention import AttnConfig, emit_attention_module
    from compiler.ptx import parse_launch

    def sched(**kw):
        cfg = AttnConfig(BH=4, Sq=512, Sk=512, D=128, scale=0.1, buffers=("q", "k", "v", "o"), **kw)
        return parse_launch(emit_attention_module(cfg)).get("schedule", "tiles")

    assert sched() == "tiles"
    monkeypatch.setenv("EMMY_ATTENTION_SCHEDULE", "split_keys")
    assert sched() == "split_keys"
    assert sched(causal=True) == "tiles"
