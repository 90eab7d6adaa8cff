#!/usr/bin/env python3
"""Copy the hot-path known-answer problems out of the reference checkout.

Each fixture is a problem folder of the reference (``problems/<id>`` or
``tests/problems/<id>``) reduced to what a run needs: the kernels' IR json
(``<entry>.ir.json``, the compiler input), ``meta.json`` (arg order, seeds,
constants, tolerances) and ``expected.npz`` (the reference harness's golden
outputs, computed by its numpy ``ref`` lambdas from the seeded inputs,
``tools/generate.py:169-176``).  Emmy's rendered CUDA (``*.ref.cu``) and the
pretty prints are not copied.

Run from the repository root with the reference checked out at REFERENCE
(default: a "reference" folder beside the repository):  python tests/golden/make_fixtures.py
"""

from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

REFERENCE = Path(os.environ.get("REFERENCE", Path(__file__).resolve().parents[3] / "reference"))
OUT = Path(__file__).resolve().parent / "problems"

# the hot-path families (RMSNorm / softmax / L2 norm / row + global reductions,
# tensor-core GEMM, tensor-core attention)
FIXTURES = [
    "problems/f01_rmsnorm", "problems/f02_row_softmax", "problems/f03_l2norm",
    "problems/r01_array_sum", "problems/r02_big_sum", "problems/r03_mean", "problems/r04_row_sum",
    "tests/problems/x_l_rmsnorm_w", "tests/problems/x_r_unpinned_sum", "tests/problems/x_r_rowmax",
    "tests/problems/x_r_mean_rows", "tests/problems/x_r_rowsum_wide", "tests/problems/x_f_softmax_wide",
    "tests/problems/x_f_softmax_scaled", "tests/problems/x_f_softmax_odd", "tests/problems/x_r_sumsq",
    "tests/problems/x_r_max", "tests/problems/x_r_abs_max", "tests/problems/x_r_sum100",
    "tests/problems/x_r_sum1000", "tests/problems/x_r_mean_3d",
    "tests/problems/x_h_mm_1024", "tests/problems/x_h_mm_256", "tests/problems/x_h_mm_relu",
    "tests/problems/x_h_mm_residual", "tests/problems/x_h_mm_t_n8", "tests/problems/x_h_mm_t_odd",
    "tests/problems/x_h_bmm_t", "tests/problems/x_h_linear", "tests/problems/x_h_linear_bias_gelu",
    "tests/problems/x_h_sdpa", "tests/problems/x_h_attn_128", "tests/problems/x_h_attn",
    "tests/problems/x_h_attn_b", "tests/problems/x_h_sdpa_causal", "tests/problems/x_h_sdpa_mask",
    # more reduction shapes: column / leading-axis sums, middle-axis mean, fused row ops
    "tests/problems/x_f_layernorm_ish", "tests/problems/x_f_max_sub", "tests/problems/x_f_rmsnorm_silu",
    "tests/problems/x_f_softmax_dim0", "tests/problems/x_r_colsum", "tests/problems/x_r_sum_dim0",
    "tests/problems/x_r_mean_mid_3d", "tests/problems/x_r_unpinned_rows", "tests/problems/x_f_layernorm",
    "tests/problems/x_f_log_softmax",
    # f16-input reductions (f32 math, f16 result)
    "tests/problems/x_d_f16_softmax", "tests/problems/x_d_f16_sum", "tests/problems/x_d_f16_mean",
    "tests/problems/x_d_f16_sq_mean",
    # emmy's split-K matmul pairs (partial products + a kernel summing them)
    "tests/problems/x_h_mm_rect", "tests/problems/x_h_bmm", "tests/problems/x_h_mm_bias",
    # more GEMM shapes (small, transposed B, vector x matrix), f16 dot rows, an f32 SwiGLU,
    # elementwise kernels of odd length
    "tests/problems/x_h_mm_16", "tests/problems/x_h_mm_64", "tests/problems/x_h_mm_128",
    "tests/problems/x_h_mm_t", "tests/problems/x_h_mm_vec", "tests/problems/x_q_f16_mm_t",
    "tests/problems/x_d_f16_dot", "tests/problems/x_d_f16_dot_f32", "tests/problems/x_l_swiglu",
    "tests/problems/x_p_odd7", "tests/problems/x_p_odd1001",
    # low-precision casts inside kernels: e4m3 (saturating), bf16, f16 with a constant
    "tests/problems/x_q_fp8_e4m3", "tests/problems/x_q_fp8_e4m3_sat", "tests/problems/x_q_fp8_scaled",
    "tests/problems/x_q_bf16_cast", "tests/problems/x_q_bf16_math", "tests/problems/x_q_f16_scalar",
    "tests/problems/x_l_gqa", "problems/a02_attention_128", "tests/problems/x_a_rect",
    # serial scans emmy writes as per-element loops (element maps)
    "tests/problems/x_r_cumsum", "tests/problems/x_r_cumsum_rows", "tests/problems/x_l_ssm_decay",
    # element maps of the reference's elementwise set (f32 / f16), its f32 attention and linear
    # attention problems (emmy lowers them as row reductions)
    "problems/a01_attention", "problems/p00_scalar_add", "problems/p01_vector_add",
    "problems/p02_scale_shift", "problems/p03_relu_mul", "tests/problems/x_d_f16_add",
    "tests/problems/x_d_f16_bcast_mul", "tests/problems/x_d_f16_div_sqrt",
    "tests/problems/x_d_f16_exp", "tests/problems/x_d_f16_gelu", "tests/problems/x_d_f16_to_f32",
    "tests/problems/x_d_f32_to_f16", "tests/problems/x_l_linattn", "tests/problems/x_p_3d",
    "tests/problems/x_p_3d_bcast", "tests/problems/x_p_bcast_col", "tests/problems/x_p_bcast_row",
    "tests/problems/x_p_big", "tests/problems/x_p_chain3", "tests/problems/x_p_clamp",
    "tests/problems/x_p_div", "tests/problems/x_p_exp", "tests/problems/x_p_exp_wide",
    "tests/problems/x_p_gelu", "tests/problems/x_p_hardtanh_clamp", "tests/problems/x_p_log",
    "tests/problems/x_p_maxmin", "tests/problems/x_p_mul_add_exact", "tests/problems/x_p_neg_abs",
    "tests/problems/x_p_odd_2d", "tests/problems/x_p_pow_half", "tests/problems/x_p_recip",
    "tests/problems/x_p_rsqrt", "tests/problems/x_p_short_launch", "tests/problems/x_p_silu",
    "tests/problems/x_p_softplus", "tests/problems/x_p_softsign", "tests/problems/x_p_sqrt",
    "tests/problems/x_p_square", "tests/problems/x_p_sub1000", "tests/problems/x_p_sub_const",
    # f32 matmuls (emmy's SIMT FMA schedule; split-K atomics in m02 / x_m_scaled)
    "problems/m01_matmul_512", "problems/m02_matmul_rect", "tests/problems/x_m_small",
    "tests/problems/x_m_tall", "tests/problems/x_m_wide", "tests/problems/x_m_longk",
    "tests/problems/x_m_256", "tests/problems/x_m_batched", "tests/problems/x_m_bias_relu",
    "tests/problems/x_m_scaled",
    # f32 operands cast to bf16 before the product (tensor-core and warp-shuffle forms)
    "tests/problems/x_q_bf16_mm", "tests/problems/x_q_bf16_mm_t",
    # rows TMA cannot address (not 16-byte aligned), 16-bit and mixed operands: the converter
    # warps load the tiles themselves
    "tests/problems/x_q_bf16_mm_odd", "tests/problems/x_h_mm_odd", "tests/problems/x_h_mm_odd2",
    "tests/problems/x_h_mm_mixed", "tests/problems/x_m_odd",
    # f64 buffers, products taken in f32 as the IR says (f32 rounding of each operand, 3xTF32)
    "tests/problems/x_d_f64_mm",
    # emmy's register-tiled f32 attention with bounds guards (element maps with Cond)
    "tests/problems/x_a_32x16", "tests/problems/x_a_256x64", "tests/problems/x_a_batched",
    # bool masks / where, tanh (this back end's own, from its series and exp), sigmoid; the
    # soft-capped softmax (Gemma-style logit capping) is a row reduction
    "tests/problems/x_l_softcap", "tests/problems/x_p_where", "tests/problems/x_p_cmp_mask",
    "tests/problems/x_p_elu_where", "tests/problems/x_p_leaky_where", "tests/problems/x_p_mask_and",
    "tests/problems/x_p_mask_float", "tests/problems/x_p_mask_mul", "tests/problems/x_p_mask_not",
    "tests/problems/x_p_gelu_tanh", "tests/problems/x_p_mish", "tests/problems/x_p_sigmoid",
    "tests/problems/x_p_tanh", "tests/problems/x_p_tanhshrink",
    # e5m2 casts, overflowing to inf like torch's
    "tests/problems/x_q_fp8_e5m2", "tests/problems/x_q_fp8_e5m2_inf",
    # masked attention in emmy's unrolled SIMT form (key steps replicated, one output
    # element per cooperative tile), on the tcgen05 attention template
    "tests/problems/x_h_attn_mask", "tests/problems/x_h_sdpa_mask_odd",
    # odd attention split in two kernels: Q K^T (split-K atomics into a zeroed buffer, one
    # pass here on the tf32 template) and emmy's serial online softmax @ V (element map)
    "tests/problems/x_h_attn_odd",
    # softmax of input scores @ V (no Q K^T): an element map of the same arithmetic
    "tests/problems/x_h_softmax_mm", "tests/problems/x_h_softmax_mm_odd",
    # two contractions in one kernel: relu(x W1) W2 and silu(x W1) * (x W3)
    "tests/problems/x_h_mlp", "tests/problems/x_l_swiglu_h",
    # element maps with Select (rotary embedding's rotate-half; the SSM scan's triangular mask)
    "tests/problems/x_l_rope", "tests/problems/x_l_ssm_scan",
    # pow (constant integer exponents as products) and sin / cos written here
    "tests/problems/x_p_pow3", "tests/problems/x_p_pow_frac", "tests/problems/x_p_pow_tensor",
    "tests/problems/x_p_neg_pow", "tests/problems/x_p_sin_cos",
    # integer / f64 reductions: emmy's cooperative form run one thread per output
    "tests/problems/x_d_f64_sum", "tests/problems/x_d_f64_softmax", "tests/problems/x_d_i32_max",
    "tests/problems/x_d_i64_max", "tests/problems/x_d_i32_sum",
    # integer (i32 / i64) and f64 element maps: torch's promotions, floor division, remainder,
    # shifts, bit operations, casts; f64 exp written here
    "tests/problems/x_d_f32_to_i32", "tests/problems/x_d_f64_add", "tests/problems/x_d_f64_div", "tests/problems/x_d_f64_exp",
    "tests/problems/x_d_i32_abs_sub", "tests/problems/x_d_i32_add", "tests/problems/x_d_i32_bitwise", "tests/problems/x_d_i32_cmp",
    "tests/problems/x_d_i32_floordiv", "tests/problems/x_d_i32_floordiv_c", "tests/problems/x_d_i32_mixed", "tests/problems/x_d_i32_rem",
    "tests/problems/x_d_i32_rshift", "tests/problems/x_d_i32_to_f32", "tests/problems/x_d_i32_where", "tests/problems/x_d_i64_cumsum",
    "tests/problems/x_d_i64_mul_add", "tests/problems/x_q_int4_unpack",
]


def main() -> int:
    if not REFERENCE.exists():
        print(f"reference checkout not found at {REFERENCE}", file=sys.stderr)
        return 1
    for rel in FIXTURES:
        src = REFERENCE / rel
        dst = OUT / src.name
        if dst.exists():
            shutil.rmtree(dst)
        dst.mkdir(parents=True)
        for f in sorted(src.iterdir()):
            if f.name == "meta.json" or f.name == "expected.npz" or f.name.endswith(".ir.json"):
                shutil.copy(f, dst / f.name)
        print(f"{rel} -> {dst.relative_to(OUT.parent.parent.parent)}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
