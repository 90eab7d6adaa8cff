"""The BASELINE-size parity criterion tells a correct kernel from a slightly broken one.

Mistakes are planted in the oracle, on the CPU: a GEMM that skips one 64-deep K block
and an attention that skips one 128-key block must fail the criterion that
``test_gpu_baseline.py`` applies, while an independent correct evaluation (f32
accumulation in another order, P rounded to bf16 before the PV product as the
tensor-core kernel does) passes it.
"""

import math

import numpy as np

from parity import bf16_ulp, parity


def _bf16(x):
    from hostfmt import bf16_bits_to_f32, f32_to_bf16_bits
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, np.float32)))


def test_bf16_ulp():
    assert bf16_ulp(1.0) == 2.0 ** -7
    assert bf16_ulp(1.99) == 2.0 ** -7
    assert bf16_ulp(0.1) == 2.0 ** -11
    assert bf16_ulp(0.0) == 0.0


def test_gemm_criterion_catches_a_skipped_k_block():
    from oracle.refs import mm_bf16
    rng = np.random.default_rng(0)
    m, n, k = 64, 256, 2048
    a = _bf16(rng.standard_normal((m, k), dtype=np.float32) * np.float32(0.05))
    b = _bf16(rng.standard_normal((k, n), dtype=np.float32) * np.float32(0.05))
    ref = mm_bf16(a, b)
    # a correct kernel: f32 products summed in K blocks of 64, result rounded once to bf16
    acc = np.zeros((m, n), np.float32)
    for k0 in range(0, k, 64):
        acc += a[:, k0:k0 + 64] @ b[k0:k0 + 64]
    assert parity(_bf16(acc), ref, 1e-2)["ok"]
    # the same kernel losing one K block
    bad = acc - a[:, 1024:1088] @ b[1024:1088]
    s = parity(_bf16(bad), ref, 1e-2)
    assert not s["ok"], s


def _attention_f32_p_rounded(q, k, v, scale, drop=None):
    """Flash-style attention: f32 scores, running max, P rounded to bf16 before P V,
    O / l at the end; ``drop`` skips one 128-key block."""
    s = (q.astype(np.float32) @ k.astype(np.float32).T) * np.float32(scale)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    if drop is not None:
        p[:, drop * 128:(drop + 1) * 128] = 0.0
    l_ = p.sum(-1, keepdims=True)
    o = (_bf16(p) @ v.astype(np.float32)) / l_
    return _bf16(o)


def test_attention_criterion_catches_a_skipped_key_block():
    from oracle.refs import attn_bf16
    rng = np.random.default_rng(1)
    s_len, d = 4096, 128
    q, k, v = (_bf16(rng.standard_normal((s_len, d), dtype=np.float32)) for _ in range(3))
    rows = np.arange(0, s_len, 64)
    scale = 1.0 / math.sqrt(d)
    ref = attn_bf16(q[rows], k, v, scale)
    good = _attention_f32_p_rounded(q[rows], k, v, scale)
    assert parity(good, ref, 1e-2)["ok"], parity(good, ref, 1e-2)
    bad = _attention_f32_p_rounded(q[rows], k, v, scale, drop=17)
    s = parity(bad, ref, 1e-2)
    assert not s["ok"], s


def test_criterion_has_no_absolute_floor():
    ref = np.full(16, 0.02, np.float32)
    got = ref.copy()
    got[3] += 0.009          # under the old 1e-2 absolute floor, but ~73 bf16 ulps of 0.02
    assert not parity(got, ref, 1e-2)["ok"]
