"""CPU oracle for the hot path: numpy restatements of the reference harness's refs.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / ``--impl reference`` arm may import this module, and only as the
checker or the timed CPU baseline -- never as a path that produces a product result.

The reference computes every expected output with a numpy ``ref`` lambda over the
seeded inputs (``tools/generate.py:169-176``: input ``i`` of the graph is
``np.random.default_rng(i).standard_normal(shape)`` cast to its dtype).  The
functions below restate those lambdas; each cites the line it follows.  They are
pinned against the reference's own ``expected.npz`` golden vectors by
``tests/test_oracle.py`` (``max |diff| == 0`` for most problems: same formula, same
precision).
"""

from __future__ import annotations

import numpy as np

f64 = lambda a: np.asarray(a).astype(np.float64)   # noqa: E731
f32 = lambda a: np.asarray(a).astype(np.float32)   # noqa: E731
f16 = lambda a: np.asarray(a).astype(np.float16)   # noqa: E731


# ---------------------------------------------------------------------------
# inputs


def seeded(seed: int, shape, dtype="f32") -> np.ndarray:
    """``default_rng(seed).standard_normal(shape)`` cast to the buffer dtype
    (``tools/generate.py:169-176``; ``docs/API.md:46``)."""
    a = np.random.default_rng(seed).standard_normal(tuple(shape) or (1,))
    if dtype == "f16":
        return a.astype(np.float16)
    if dtype == "f64":
        return a
    if dtype in ("i32", "i64"):            # truncated toward zero, as numpy's astype
        return a.astype(np.int32 if dtype == "i32" else np.int64)
    return a.astype(np.float32)


# ---------------------------------------------------------------------------
# reductions (category 2) -- tools/expressions_open.py:45-59,
# tests/expressions_extra.py:186-205, 278-287


def total_sum(x):
    """``f32(f64(x).sum())`` (expressions_open.py:47-52; expressions_extra.py:187-190, 204-205)."""
    return f32(f64(x).sum())


def total_mean(x):
    """``f32(f64(x).mean())`` (expressions_open.py:53-55)."""
    return f32(f64(x).mean())


def total_max(x):
    """``x.max()`` (expressions_extra.py:191-192)."""
    return np.asarray(x).max()


def total_abs_max(x):
    """``f32(abs(x).max())`` (expressions_extra.py:282-283)."""
    return f32(np.abs(x).max())


def total_sumsq(x):
    """``f32((f64(x) ** 2).sum())`` (expressions_extra.py:193-194)."""
    return f32((f64(x) ** 2).sum())


def row_sum(x):
    """``f32(f64(x).sum(-1))`` (expressions_open.py:56-58; expressions_extra.py:197-198)."""
    return f32(f64(x).sum(-1))


def row_mean(x):
    """``f32(f64(x).mean(-1))`` (expressions_extra.py:195-196, 278-279)."""
    return f32(f64(x).mean(-1))


def row_max(x):
    """``x.max(-1)`` (expressions_extra.py:199-200)."""
    return np.asarray(x).max(-1)


def axis_sum(x, axis):
    """``f32(f64(x).sum(axis))`` (expressions_extra.py:201-202 x_r_colsum, 280-281
    x_r_sum_dim0, 284-285 x_r_unpinned_rows)."""
    return f32(f64(x).sum(axis))


def axis_mean(x, axis):
    """``f32(f64(x).mean(axis))`` (expressions_extra.py:286-287, x_r_mean_mid_3d)."""
    return f32(f64(x).mean(axis))


def f16_sum(x):
    """``f16(f64(x).sum())`` (expressions_extra.py:307-308, x_d_f16_sum)."""
    return f16(f64(x).sum())


def f16_row_mean(x):
    """``f16(f64(x).mean(-1))`` (expressions_extra.py:309-310, x_d_f16_mean)."""
    return f16(f64(x).mean(-1))


def f16_sq_mean(x):
    """The f16 product rounded before the mean: ``f16(f64(f16(f32(x) * f32(x))).mean(-1))``
    (expressions_extra.py:317-318, x_d_f16_sq_mean)."""
    return f16(f64(f16(f32(x) * f32(x))).mean(-1))


# ---------------------------------------------------------------------------
# fused row kernels (category 4)


def _softmax(x, axis=-1):
    """Max-subtracted softmax in the input's precision (expressions_open.py:27-30)."""
    m = x.max(axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=axis, keepdims=True)


def softmax(x, scale=None):
    """``f32(softmax(f64(x) [* scale]))`` (expressions_open.py:79-81;
    expressions_extra.py:208-209, 249-250, 255-256)."""
    xd = f64(x)
    if scale is not None:
        xd = xd * scale
    return f32(_softmax(xd))


def layernorm_ish(x):
    """``f32(f64(x) - f64(x).mean(-1, keepdims=True))`` (expressions_extra.py:210-211)."""
    return f32(f64(x) - f64(x).mean(-1, keepdims=True))


def max_sub(x):
    """``f32(f64(x) - f64(x).max(-1, keepdims=True))`` (expressions_extra.py:259-260)."""
    return f32(f64(x) - f64(x).max(-1, keepdims=True))


def layernorm(x, w, b, eps=1e-5):
    """``(x - mean) / sqrt(var + eps) * w + b`` in f64 (expressions_extra.py:238-243)."""
    xd = f64(x)
    return f32((xd - xd.mean(-1, keepdims=True)) / np.sqrt(xd.var(-1, keepdims=True) + eps)
               * f64(w) + f64(b))


def log_softmax(x):
    """``f32(log(softmax(f64(x))))`` (expressions_extra.py:245-250)."""
    return f32(np.log(_softmax(f64(x))))


def rmsnorm_silu(x, eps=1e-6):
    """``silu(x / sqrt(mean(x^2) + eps))`` in f64 (expressions_extra.py:251-254)."""
    y = f64(x) / np.sqrt((f64(x) ** 2).mean(-1, keepdims=True) + eps)
    return f32(y / (1 + np.exp(-y)))


def softmax_axis(x, axis):
    """``f32(softmax(f64(x), axis))`` (expressions_extra.py:257-258, x_f_softmax_dim0)."""
    return f32(_softmax(f64(x), axis=axis))


def f16_softmax(x):
    """``f16(softmax(f64(x)))`` (expressions_extra.py:305-306, x_d_f16_softmax)."""
    return f16(_softmax(f64(x)))


def rmsnorm_sqrt(x, w, eps):
    """``x / sqrt(mean(x^2) + eps) * w`` with the mean in f64
    (expressions_open.py:73-78, problem f01_rmsnorm)."""
    return f32(x / np.sqrt((f64(x) ** 2).mean(-1, keepdims=True) + eps) * w)


def rmsnorm(x, w, eps=1e-6):
    """``f32(f64(x) / sqrt(mean(f64(x)^2) + eps) * f64(w))`` -- the BASELINE formula
    ``x * rsqrt(mean(x^2) + eps) * w`` (expressions_llm.py:76-78, x_l_rmsnorm_w)."""
    return f32(f64(x) / np.sqrt((f64(x) ** 2).mean(-1, keepdims=True) + eps) * f64(w))


def l2norm(x):
    """``x / sqrt(sum(x^2))`` (expressions_open.py:82-84, problem f03_l2norm)."""
    return f32(x / np.sqrt((f64(x) ** 2).sum(-1, keepdims=True)))


# ---------------------------------------------------------------------------
# tensor-core GEMM / attention (expressions_extra.py:48-63, 366-431;
# expressions_quant.py:39-41)


def mm_f16(a, b):
    """torch's f16 matmul: exact products summed in f32, one rounding to f16
    (``_mmh``, expressions_extra.py:50-51, computed in f64)."""
    return f16(f64(a) @ f64(b))


def attn_f16(q, kt, v, scale, causal=False, mask=None):
    """torch's f16 attention with each op's result rounded to f16
    (``_attn_h``, expressions_extra.py:54-63)."""
    s = f16(f16(f64(q) @ f64(kt)) * scale)
    if mask is not None:
        s = f16(s + mask)
    s = f64(s)
    if causal:
        s = np.where(np.tril(np.ones(s.shape[-2:], dtype=bool)), s, -np.inf)
    return f16(f64(f16(_softmax(s))) @ f64(v))


def f16_dot(a, b, out):
    """Row dot products of f16 vectors whose elementwise products are rounded to f16
    first (their own torch op), summed in f64: ``out(f64(f16(f32(a) * f32(b))).sum(-1))``
    (expressions_extra.py:313-316, x_d_f16_dot / x_d_f16_dot_f32)."""
    return out(f64(f16(f32(a) * f32(b))).sum(-1))


def swiglu(x, w1, w3):
    """``silu(x @ w1) * (x @ w3)`` in f64, ``silu(y) = y / (1 + exp(-y))``
    (expressions_llm.py:66-68, x_l_swiglu)."""
    g = f64(x) @ f64(w1)
    return f32(g / (1 + np.exp(-g)) * (f64(x) @ f64(w3)))


def linattn(q, k, v):
    """Causal linear attention ``y_t = q_t . sum_{s<=t} k_s v_s^T`` in f64
    (expressions_llm.py:38-41)."""
    state = np.cumsum(f64(k)[:, :, None] * f64(v)[:, None, :], 0)
    return f32((f64(q)[:, :, None] * state).sum(1))


def gelu(x):
    """Exact (erf) GELU, ``0.5 x (1 + erf(x / sqrt 2))`` (expressions_extra.py:66-67)."""
    from math import erf, sqrt
    v = np.vectorize(lambda t: 0.5 * t * (1.0 + erf(t / sqrt(2.0))))
    return v(np.asarray(x, dtype=np.float64))


def bf16_round(a) -> np.ndarray:
    """Round f32 values to bf16 (nearest even) and return them as f32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    u = (u + (((u >> 16) & 1) + 0x7FFF)) & 0xFFFF0000
    return u.view(np.float32)


def bf16_math(a, b):
    """``(a.bf16() * b.bf16() + a.bf16()).float()``: each bf16 op computed in f32 and
    rounded to bf16 (expressions_quant.py:31-33, x_q_bf16_math)."""
    A, B = bf16_round(a), bf16_round(b)
    return bf16_round(bf16_round(A * B) + A)


def mm_bf16(a, b):
    """bf16 GEMM with f32 accumulation and a bf16 result, evaluated on the
    bf16-valued operands in f64 (the BASELINE GEMM; x_q_bf16_mm's
    ``a.bfloat16() @ b.bfloat16()``, expressions_quant.py:39-41)."""
    return bf16_round(f32(f64(a) @ f64(b)))


def attn_bf16(q, k, v, scale, causal=False, mask=None, q_offset=0):
    """Attention on bf16-valued inputs, softmax in f64, bf16 result:
    ``softmax(q k^T * scale [+ mask]) v`` with ``[..., S, D]`` operands (the BASELINE
    attention: F.scaled_dot_product_attention, as in x_h_sdpa).  ``causal`` drops keys
    after the query (top-left aligned, ``is_causal``); ``q_offset`` is the absolute
    index of the first query row when ``q`` holds a slice of the rows."""
    s = f64(q) @ np.swapaxes(f64(k), -1, -2) * scale
    if mask is not None:
        s = s + f64(mask)
    if causal:
        rows = np.arange(s.shape[-2])[:, None] + q_offset
        s = np.where(np.arange(s.shape[-1])[None, :] <= rows, s, -np.inf)
    return bf16_round(f32(_softmax(s) @ f64(v)))


def e4m3_round(a) -> np.ndarray:
    """Round to float8 e4m3fn with saturation to +-448 (torch's ``float8_e4m3fn``
    cast, the semantics of the reference's dtypes.py:181-227), returned as f32."""
    x = np.asarray(a, dtype=np.float64)
    sign = np.sign(x)
    m = np.minimum(np.abs(x), 448.0)
    out = np.zeros_like(m)
    nz = m > 0
    e = np.floor(np.log2(m[nz]))
    e = np.maximum(e, -6.0)                  # subnormals share the 2^-6 exponent
    q = 2.0 ** (e - 3)                       # 3 mantissa bits
    r = m[nz] / q
    rn = np.round(r)                         # numpy rounds half to even
    out[nz] = rn * q
    out = np.minimum(out, 448.0)
    return (sign * out).astype(np.float32)


def e5m2_round(a) -> np.ndarray:
    """Round to float8 e5m2 (nearest even; 2 mantissa bits, exponents down to 2^-14 and
    subnormals in steps of 2^-16), overflowing to +-inf past the largest finite 57344 as
    torch's ``float8_e5m2`` cast does (tests/expressions_quant.py:18-24), returned as f32."""
    x = np.asarray(a, dtype=np.float64)
    sign = np.where(np.signbit(x), -1.0, 1.0)
    m = np.abs(x)
    out = np.zeros_like(m)
    nz = (m > 0) & np.isfinite(m)
    e = np.maximum(np.floor(np.log2(m[nz])), -14.0)
    q = 2.0 ** (e - 2)
    out[nz] = np.round(m[nz] / q) * q
    out[~np.isfinite(m)] = m[~np.isfinite(m)]
    out[out > 57344.0] = np.inf
    return (sign * out).astype(np.float32)


def mm_f32(a, b):
    """f32 matmul: the product in f64, rounded once to f32 (the reference's refs for
    ``m01_matmul_512`` / ``m02_matmul_rect``, tools/expressions_open.py:66-73, and the
    ``x_m_*`` family, tests/expressions_extra.py:215-233)."""
    return f32(f64(a) @ f64(b))


def mm_fp8(aq, bq, sa, sb):
    """FP8 GEMM oracle: ``(A_q . B_q) * s_a * s_b`` in f64 from the e4m3-valued
    operands, rounded to bf16 (no reference kernel: the reference has no FP8 GEMM)."""
    return bf16_round(f32((f64(aq) @ f64(bq)) * sa * sb))


# ---------------------------------------------------------------------------
# per-problem table: which ref a golden fixture was generated with, with the
# graph inputs in the order of meta.json's graph_inputs

PROBLEM_REFS = {
    "m01_matmul_512": lambda a, b: [mm_f32(a, b)],
    "m02_matmul_rect": lambda a, b: [mm_f32(a, b)],
    "x_m_small": lambda a, b: [mm_f32(a, b)],
    "x_m_tall": lambda a, b: [mm_f32(a, b)],
    "x_m_wide": lambda a, b: [mm_f32(a, b)],
    "x_m_longk": lambda a, b: [mm_f32(a, b)],
    "x_m_256": lambda a, b: [mm_f32(a, b)],
    "x_m_batched": lambda a, b: [mm_f32(a, b)],
    "x_m_bias_relu": lambda a, b, c: [f32(np.maximum(f64(a) @ f64(b) + f64(c), 0))],
    "x_m_scaled": lambda a, b: [f32((f64(a) @ f64(b)) * 0.5)],
    "f01_rmsnorm": lambda x, w: [rmsnorm_sqrt(x, w, 1e-5)],
    "f02_row_softmax": lambda x: [softmax(x)],
    "f03_l2norm": lambda x: [l2norm(x)],
    "r01_array_sum": lambda x: [total_sum(x)],
    "r02_big_sum": lambda x: [total_sum(x)],
    "r03_mean": lambda x: [total_mean(x)],
    "r04_row_sum": lambda x: [row_sum(x)],
    "x_l_rmsnorm_w": lambda x, w: [rmsnorm(x, w, 1e-6)],
    "x_r_unpinned_sum": lambda x: [total_sum(x)],
    "x_r_rowmax": lambda x: [row_max(x)],
    "x_r_mean_rows": lambda x: [row_mean(x)],
    "x_r_rowsum_wide": lambda x: [row_sum(x)],
    "x_f_softmax_wide": lambda x: [softmax(x)],
    "x_f_softmax_scaled": lambda x: [softmax(x, 0.125)],
    "x_f_softmax_odd": lambda x: [softmax(x)],
    "x_r_sumsq": lambda x: [total_sumsq(x)],
    "x_r_max": lambda x: [total_max(x)],
    "x_r_abs_max": lambda x: [total_abs_max(x)],
    "x_r_sum100": lambda x: [total_sum(x)],
    "x_r_sum1000": lambda x: [total_sum(x)],
    "x_r_mean_3d": lambda x: [row_mean(x)],
    "x_r_colsum": lambda x: [axis_sum(x, 0)],
    "x_r_sum_dim0": lambda x: [axis_sum(x, 0)],
    "x_r_unpinned_rows": lambda x: [axis_sum(x, -1)],
    "x_r_mean_mid_3d": lambda x: [axis_mean(x, 1)],
    "x_f_layernorm_ish": lambda x: [layernorm_ish(x)],
    "x_f_max_sub": lambda x: [max_sub(x)],
    "x_f_layernorm": lambda x, w, b: [layernorm(x, w, b)],
    "x_f_log_softmax": lambda x: [log_softmax(x)],
    "x_f_rmsnorm_silu": lambda x: [rmsnorm_silu(x)],
    "x_f_softmax_dim0": lambda x: [softmax_axis(x, 0)],
    "x_d_f16_softmax": lambda x: [f16_softmax(x)],
    "x_d_f16_sum": lambda x: [f16_sum(x)],
    "x_d_f16_mean": lambda x: [f16_row_mean(x)],
    "x_d_f16_sq_mean": lambda x: [f16_sq_mean(x)],
    "x_h_mm_1024": lambda a, b: [mm_f16(a, b)],
    "x_h_mm_256": lambda a, b: [mm_f16(a, b)],
    "x_h_mm_relu": lambda a, b: [np.maximum(mm_f16(a, b), f16(0))],
    "x_h_mm_t_n8": lambda a, b: [mm_f16(a, b.T)],
    "x_h_mm_t_odd": lambda a, b: [mm_f16(a, b.T)],
    "x_h_linear": lambda x, w: [mm_f16(x, w.T)],
    "x_h_bmm_t": lambda q, k: [mm_f16(q, np.swapaxes(k, -1, -2))],
    "x_h_linear_bias_gelu": lambda x, w, b: [f16(gelu(f64(mm_f16(x, w.T) + b)))],
    "x_h_mm_residual": lambda a, b, r: [mm_f16(a, b) + r],
    "x_h_mm_rect": lambda a, b: [mm_f16(a, b)],
    "x_h_mm_16": lambda a, b: [mm_f16(a, b)],
    "x_h_mm_64": lambda a, b: [mm_f16(a, b)],
    "x_h_mm_128": lambda a, b: [mm_f16(a, b)],
    "x_h_mm_t": lambda a, b: [mm_f16(a, b.T)],
    "x_h_mm_vec": lambda a, b: [mm_f16(a, b)],
    "x_q_f16_mm_t": lambda a, b: [f32(mm_f16(f16(a), f16(b).T))],
    "x_q_bf16_mm": lambda a, b: [mm_bf16(bf16_round(a), bf16_round(b))],
    "x_q_bf16_mm_t": lambda a, b: [mm_bf16(bf16_round(a), bf16_round(b).T)],
    "x_q_bf16_mm_odd": lambda a, b: [mm_bf16(bf16_round(a), bf16_round(b))],
    "x_h_mm_odd": lambda a, b: [mm_f16(a, b)],
    "x_h_mm_odd2": lambda a, b: [mm_f16(a, b)],
    "x_h_mm_mixed": lambda a, b: [mm_f32(a, b)],
    "x_m_odd": lambda a, b: [mm_f32(a, b)],
    "x_d_f16_dot": lambda a, b: [f16_dot(a, b, f16)],
    "x_d_f16_dot_f32": lambda a, b: [f16_dot(a, b, f32)],
    "x_l_swiglu": lambda x, w1, w3: [swiglu(x, w1, w3)],
    "x_p_odd7": lambda a, b: [a + b],
    "x_q_fp8_e4m3": lambda x: [e4m3_round(x)],
    "x_q_fp8_e4m3_sat": lambda x: [e4m3_round(f32(x * f32(300.0)))],
    "x_q_fp8_scaled": lambda x: [e4m3_round(f32(x * f32(64.0))) / f32(64.0)],
    "x_q_bf16_cast": lambda x: [bf16_round(x)],
    "x_q_bf16_math": lambda a, b: [bf16_math(a, b)],
    # -- elementwise (tools/expressions_open.py:33-46, tests/expressions_extra.py:77-175, 295-322)
    "p00_scalar_add": lambda a, b: [a + b],
    "p01_vector_add": lambda a, b: [a + b],
    "p02_scale_shift": lambda x: [x * np.float32(2.0) + np.float32(1.0)],
    "p03_relu_mul": lambda x, y: [np.maximum(x, 0) * y],
    "x_p_short_launch": lambda a, b: [a + b],
    "x_p_sub1000": lambda a, b: [a - b],
    "x_p_big": lambda a, b: [a + b],
    "x_p_bcast_row": lambda a, b: [a + b],
    "x_p_bcast_col": lambda a, b: [a * b],
    "x_p_3d": lambda a, b: [a * b],
    "x_p_3d_bcast": lambda a, b: [a + b],
    "x_p_odd_2d": lambda a, b: [a + b],
    "x_p_div": lambda x, y: [x / y],
    "x_p_neg_abs": lambda x: [-np.abs(x)],
    "x_p_maxmin": lambda x, y: [np.maximum(x, y) - np.minimum(x, y)],
    "x_p_clamp": lambda x: [np.clip(x, np.float32(-0.5), np.float32(0.5))],
    "x_p_square": lambda x: [x * x],
    "x_p_sub_const": lambda x: [np.float32(3.0) - x],
    "x_p_sqrt": lambda x: [np.sqrt(np.abs(x))],
    "x_p_chain3": lambda x, y, z: [f32((f64(x) * 1.5 + f64(y)) * f64(z) - 0.25 * f64(x))],
    "x_p_exp": lambda x: [f32(np.exp(f64(x)))],
    "x_p_exp_wide": lambda x: [f32(np.exp(f64(np.float32(20.0) * x)))],
    "x_p_log": lambda x: [f32(np.log(f64(np.abs(x) + np.float32(0.5))))],
    "x_p_rsqrt": lambda x: [f32(1.0 / np.sqrt(f64(np.abs(x) + np.float32(0.1))))],
    "x_p_recip": lambda x: [f32(1.0 / f64(np.abs(x) + np.float32(1.0)))],
    "x_p_silu": lambda x: [f32(f64(x) / (1.0 + np.exp(-f64(x))))],
    "x_p_gelu": lambda x: [f32(gelu(x))],
    "x_p_pow_half": lambda x: [f32(np.sqrt(f64(np.abs(x))))],
    "x_p_softplus": lambda x: [f32(np.logaddexp(0.0, f64(x)))],
    "x_p_hardtanh_clamp": lambda x: [np.clip(x * np.float32(2), np.float32(-1), np.float32(1))],
    "x_p_softsign": lambda x: [f32(f64(x) / (1 + np.abs(f64(x))))],
    "x_p_mul_add_exact": lambda a, b, c: [a * b + c],
    "x_d_f16_add": lambda a, b: [a + b],
    "x_d_f16_bcast_mul": lambda a, b: [a * b],
    "x_d_f16_div_sqrt": lambda x: [x / np.sqrt(np.abs(x) + f16(1))],
    "x_d_f16_exp": lambda x: [f16(np.exp(f64(x)))],
    "x_d_f16_gelu": lambda x: [f16(gelu(x))],
    "x_d_f32_to_f16": lambda x: [f16(x) * f16(2)],
    "x_d_f16_to_f32": lambda x: [f32(x) * np.float32(3)],
    # -- f32 attention and causal linear attention (expressions_open.py:93-98,
    #    expressions_llm.py:38-41, 62-64)
    "a01_attention": lambda q, kt, v: [f32(_softmax(f64(q) @ f64(kt) / 8.0) @ f64(v))],
    "x_l_linattn": lambda q, k, v: [linattn(q, k, v)],
    "a02_attention_128": lambda q, kt, v: [f32(_softmax(f64(q) @ f64(kt) / 5.656854) @ f64(v))],
    "x_a_rect": lambda q, kt, v: [f32(_softmax((f64(q) @ f64(kt)) * 0.17677669) @ f64(v))],
    # integer and f64 element maps (expressions_extra.py:323-368; expressions_quant.py:25-26)
    "x_d_f64_add": lambda a, b: [a + b],
    "x_d_f64_mm": lambda a, b: [a @ b],
    "x_d_f64_sum": lambda x: [x.sum()],
    "x_d_f64_softmax": lambda x: [_softmax(x)],
    "x_d_i32_max": lambda x: [x.max(-1)],
    "x_d_i64_max": lambda x: [x.max(-1)],
    "x_d_i32_sum": lambda x: [x.astype(np.int64).sum()],
    "x_d_f64_div": lambda a, b: [a * b / (np.abs(b) + 1)],
    "x_d_f64_exp": lambda x: [np.exp(x)],
    "x_d_i32_add": lambda a, b: [a + b],
    "x_d_i64_mul_add": lambda a, b: [a * b + b],
    "x_d_i32_floordiv": lambda a, b: [a // (np.abs(b) + 1)],
    "x_d_i32_rem": lambda a, b: [a % (np.abs(b) + 1)],
    "x_d_i32_floordiv_c": lambda a: [a // 2],
    "x_d_i32_bitwise": lambda a, b: [(a & b) ^ (a | b)],
    "x_d_i32_rshift": lambda a: [a >> 1],
    "x_d_i32_cmp": lambda a, b: [f32(a > b)],
    "x_d_i32_where": lambda a: [np.where(a > 0, a, -a)],
    "x_d_i32_abs_sub": lambda a: [np.abs(a) - 1],
    "x_d_i32_mixed": lambda a, b: [f32(a) * np.float32(0.5) + b],
    "x_d_f32_to_i32": lambda x: [(x * np.float32(10)).astype(np.int32)],
    "x_d_i32_to_f32": lambda a: [f32(a) / np.float32(3)],
    "x_d_i64_cumsum": lambda x: [np.cumsum(x, -1)],
    "x_q_int4_unpack": lambda x: [(((x >> 4) & 15) - 8).astype(np.float32) * np.float32(0.1)],
    # pow and sin / cos (expressions_extra.py:136-172)
    "x_p_pow3": lambda x: [f32(f64(x) ** 3)],
    "x_p_pow_frac": lambda x: [f32(np.abs(f64(x)) ** 0.7)],
    "x_p_pow_tensor": lambda a, b: [f32(f64(np.abs(a) + np.float32(0.5)) ** f64(b))],
    "x_p_neg_pow": lambda x: [f32(f64(np.abs(x) + np.float32(0.5)) ** -2)],
    "x_p_sin_cos": lambda x: [f32(np.sin(f64(x)) + np.cos(f64(x)))],
    # e5m2 casts (expressions_quant.py:18-24)
    "x_q_fp8_e5m2": lambda x: [e5m2_round(x)],
    "x_q_fp8_e5m2_inf": lambda x: [np.clip(e5m2_round(x * np.float32(40000.0)), -1e5, 1e5).astype(np.float32)],
    # bool masks / where, tanh and sigmoid (expressions_extra.py:106-184; expressions_llm.py:79-80)
    "x_l_softcap": lambda x: [f32(_softmax(30 * np.tanh(f64(x) / 30)))],
    "x_p_where": lambda x, y: [np.where(x > 0, x, y)],
    "x_p_cmp_mask": lambda x, y: [np.where((x >= y) & (x < np.float32(0.5)), x, -y)],
    "x_p_elu_where": lambda x: [f32(np.where(f64(x) > 0, f64(x), np.exp(f64(x)) - 1.0))],
    "x_p_leaky_where": lambda x: [np.where(x > 0, x, x * np.float32(0.1))],
    "x_p_mask_and": lambda x: [np.where((x > -1) & (x < 1), x, np.float32(0))],
    "x_p_mask_float": lambda x: [(x > 0.5).astype(np.float32) + x],
    "x_p_mask_mul": lambda x: [x * (x > 0)],
    "x_p_mask_not": lambda x: [np.where(~(x > 0), x * np.float32(2), x)],
    "x_p_gelu_tanh": lambda x: [f32(0.5 * f64(x) * (1 + np.tanh(np.sqrt(2 / np.pi) * (f64(x) + 0.044715 * f64(x) ** 3))))],
    "x_p_mish": lambda x: [f32(f64(x) * np.tanh(np.logaddexp(0.0, f64(x))))],
    "x_p_sigmoid": lambda x: [f32(1.0 / (1.0 + np.exp(-f64(x))))],
    "x_p_tanh": lambda x: [f32(np.tanh(f64(x)))],
    "x_p_tanhshrink": lambda x: [f32(f64(x) - np.tanh(f64(x)))],
    # (expressions_extra.py:263-274)
    "x_a_32x16": lambda q, kt, v: [f32(_softmax((f64(q) @ f64(kt)) / 4.0) @ f64(v))],
    "x_a_256x64": lambda q, kt, v: [f32(_softmax((f64(q) @ f64(kt)) / 8.0) @ f64(v))],
    "x_a_batched": lambda q, kt, v: [f32(_softmax((f64(q) @ f64(kt)) / 5.656854) @ f64(v))],
    # scans (expressions_extra.py:288-291; expressions_llm.py:27-29, 56-58)
    "x_r_cumsum": lambda x: [f32(np.cumsum(f64(x)))],
    "x_r_cumsum_rows": lambda x: [f32(np.cumsum(f64(x), -1))],
    "x_l_ssm_decay": lambda a, x: [f32(np.exp(np.cumsum(-np.abs(f64(a)) * 0.1, -1)) * f64(x))],
    # Mamba-2 style scan in matrix form, rotary embedding (expressions_llm.py:27-46, 59-61, 73-75)
    "x_l_ssm_scan": lambda a, u: [f32(np.tril(np.exp(np.cumsum(-np.abs(f64(a)) * 0.1)[:, None]
                                                     - np.cumsum(-np.abs(f64(a)) * 0.1)[None, :])) @ f64(u))],
    "x_l_rope": lambda x, c, s: [f32(f64(x) * c + np.concatenate((-f64(x)[:, 32:], f64(x)[:, :32]), -1) * s)],
    # grouped-query sdpa: key / value heads repeated 4 times (expressions_llm.py:49-51, 81-84)
    "x_l_gqa": lambda q, k, v: [f32(_softmax(f64(q) @ np.swapaxes(np.repeat(f64(k), 4, 1), -1, -2)
                                             / np.sqrt(q.shape[-1])) @ np.repeat(f64(v), 4, 1))],
    # the scalar stays f32 (torch's opmath; the kernel folds the constant buffer's value)
    "x_q_f16_scalar": lambda x: [f32(f16(f32(f16(x)) * f32(0.1)))],
    "x_p_odd1001": lambda a, b: [a * b],
    "x_h_bmm": lambda a, b: [mm_f16(a, b)],
    "x_h_mm_bias": lambda a, b, c: [mm_f16(a, b) + c],
    "x_h_attn": lambda q, kt, v: [attn_f16(q, kt, v, 1 / 8)],
    "x_h_attn_128": lambda q, kt, v: [attn_f16(q, kt, v, 1 / 8)],
    "x_h_attn_b": lambda q, kt, v: [attn_f16(q, kt, v, 1 / 5.66)],
    "x_h_sdpa": lambda q, k, v: [attn_f16(q, np.swapaxes(k, -1, -2), v, 1 / np.sqrt(32))],
    "x_h_sdpa_causal": lambda q, k, v: [attn_f16(q, np.swapaxes(k, -1, -2), v, 1 / np.sqrt(32),
                                                 causal=True)],
    "x_h_sdpa_mask": lambda q, k, v, m: [attn_f16(q, np.swapaxes(k, -1, -2), v, 1 / np.sqrt(32),
                                                  mask=m)],
    # (expressions_extra.py:424-431)
    "x_h_attn_mask": lambda q, kt, m, v: [attn_f16(q, kt, v, 1 / 8, mask=m)],
    "x_h_attn_odd": lambda q, kt, v: [attn_f16(q, kt, v, 1 / 6)],
    # two contractions in one kernel (expressions_extra.py:396-400; expressions_llm.py:23-24, 69-72)
    "x_h_mlp": lambda x, w1, w2: [mm_f16(np.maximum(mm_f16(x, w1), f16(0)), w2)],
    "x_l_swiglu_h": lambda x, w1, w3: [f16((lambda h: h / (1 + np.exp(-h)))(f64(f16(f64(x) @ f64(w1))))
                                           * f64(f16(f64(x) @ f64(w3))))],
    # softmax of input scores @ V (expressions_extra.py:434-439)
    "x_h_softmax_mm": lambda s, v: [f16(f64(f16(_softmax(f64(s)))) @ f64(v))],
    "x_h_softmax_mm_odd": lambda s, v: [f16(f64(f16(_softmax(f64(s)))) @ f64(v))],
    "x_h_sdpa_mask_odd": lambda q, k, v, m: [attn_f16(q, np.swapaxes(k, -1, -2), v, 1 / np.sqrt(32),
                                                      mask=m)],
}


def problem_inputs(meta: dict) -> list:
    """The seeded graph inputs of a problem, in graph_inputs order."""
    args = {a["name"]: a for k in meta["kernels"] for a in k["args"]}
    out = []
    for i, name in enumerate(meta["graph_inputs"]):
        a = args[name]
        out.append(seeded(a.get("seed", i), a["shape"], a["dtype"]))
    return out


def problem_expected(meta: dict) -> dict:
    """Recompute a problem's expected outputs with the oracle."""
    ref = PROBLEM_REFS[meta["id"]]
    res = ref(*problem_inputs(meta))
    return {name: np.asarray(r) for name, r in zip(meta["graph_outputs"], res)}
