"""The f32 attention template (warp per query row, key chunks in shared memory) launched
directly at shapes the reference's fixtures do not reach: ragged key counts (scalar
staging), head dims that are not whole float4s, several output columns per lane, more
than one query row per warp, key-major k, grouped-query heads, single partial chunks.
Checked against a float64 numpy evaluation of softmax(q k^T c) v with the fixtures'
f32 attention tolerance (rtol 1e-3, atol 1e-4)."""

import numpy as np
import pytest

# B, Sq, Sk, D, Dv, kt layout, query entries per k / v entry, scale = 1 / param
CASES = [
    (1, 64, 70, 32, 24, True, 1, True),        # Sk % 4 != 0: scalar staging; Dv < 32
    (2, 100, 200, 30, 48, False, 1, False),    # key-major k, D % 4 != 0 (padded q rows); Dv 48
    (8, 512, 300, 64, 64, True, 1, True),      # 4 rows per warp, ragged last chunk
    (4, 96, 1000, 128, 100, False, 2, False),  # grouped heads, 16 chunks, D 128, Dv 100
    (3, 33, 20, 16, 8, True, 1, True),         # one partial 32-key chunk
]


def _reference(q, k, v, c, kt, group):
    out = np.empty(q.shape[:-1] + (v.shape[-1],))
    for b in range(q.shape[0]):
        kb = b // group
        km = k[kb].astype(np.float64)
        s = q[b].astype(np.float64) @ (km if kt else km.T) * c
        s -= s.max(-1, keepdims=True)
        e = np.exp(s)
        out[b] = (e / e.sum(-1, keepdims=True)) @ v[kb].astype(np.float64)
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("B,Sq,Sk,D,Dv,kt,group,recip", CASES)
def test_attention_f32_direct(runtime, B, Sq, Sk, D, Dv, kt, group, recip):
    import emmyrt
    from compiler.kernels.attention_f32 import F32AttnConfig, WARPS, emit_module
    from compiler.loader import KernelSpec, Param
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel
    rng = np.random.default_rng(B * 1000 + Sk)
    Bk = B // group
    host = {"q": rng.standard_normal((B, Sq, D), dtype=np.float32),
            "k": rng.standard_normal((Bk, D, Sk) if kt else (Bk, Sk, D), dtype=np.float32),
            "v": rng.standard_normal((Bk, Sk, Dv), dtype=np.float32)}
    c = 1.0 / np.sqrt(D)
    host["c"] = np.array([1.0 / c if recip else c], np.float32)
    params = (Param("c", "f32", (1,)), Param("q", "f32", (B, Sq, D)), Param("k", "f32", host["k"].shape),
              Param("v", "f32", (Bk, Sk, Dv)), Param("o", "f32", (B, Sq, Dv)))
    spec = KernelSpec("k_attn_f32_direct", (), params, None, None, {})
    cfg = F32AttnConfig(spec.name, B, Sq, Sk, D, Dv, "q", "k", "v", "o", "c", recip, 1.0,
                        kt=kt, group=group)
    cfg.KC = 32 if Sk <= 32 else 64
    for R in (4, 2):
        if B * -(-Sq // (WARPS * R)) >= 148:
            cfg.R = R
            break
    ck = CompiledKernel.from_ptx(spec, emit_module(spec, cfg))
    bufs = {n: DeviceBuffer(a.nbytes) for n, a in host.items()}
    for n, a in host.items():
        bufs[n].upload(a)
    bufs["o"] = DeviceBuffer(B * Sq * Dv * 4)
    bufs["o"].zero()
    ck({n: b.ptr for n, b in bufs.items()})
    emmyrt.stream_wait(0, 60)
    got = np.zeros((B, Sq, Dv), np.float32)
    bufs["o"].download(got)
    ref = _reference(host["q"], host["k"], host["v"], float(c), kt, group)
    assert np.allclose(got, ref, rtol=1e-3, atol=1e-4), f"max abs err {np.max(np.abs(got - ref))}"
