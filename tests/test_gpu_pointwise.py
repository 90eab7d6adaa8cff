"""Element-map kernels on the B200 against the golden vectors: f32 add / mul, e4m3 / bf16 / f16
casts inside a kernel (all exact: rtol = atol = 0 in the fixtures)."""

import json

import numpy as np
import pytest

from conftest import GOLDEN

MAP = ["x_p_odd7", "x_p_odd1001", "x_q_fp8_e4m3", "x_q_fp8_e4m3_sat", "x_q_fp8_scaled", "x_q_bf16_cast",
       "x_q_fp8_e5m2", "x_q_fp8_e5m2_inf",
       "x_q_bf16_math", "x_q_f16_scalar",
       "p00_scalar_add", "p01_vector_add", "p02_scale_shift", "p03_relu_mul", "x_p_short_launch",
       "x_p_sub1000", "x_p_big", "x_p_bcast_row", "x_p_bcast_col", "x_p_3d", "x_p_3d_bcast", "x_p_odd_2d",
       "x_p_div", "x_p_neg_abs", "x_p_maxmin", "x_p_clamp", "x_p_square", "x_p_sub_const", "x_p_sqrt",
       "x_p_chain3", "x_p_exp", "x_p_exp_wide", "x_p_log", "x_p_rsqrt", "x_p_recip", "x_p_silu",
       "x_p_gelu", "x_p_pow_half", "x_p_softplus", "x_p_hardtanh_clamp", "x_p_softsign",
       "x_p_mul_add_exact", "x_d_f16_add", "x_d_f16_bcast_mul", "x_d_f16_div_sqrt", "x_d_f16_exp",
       "x_d_f16_gelu", "x_d_f32_to_f16", "x_d_f16_to_f32",
       # f32 attention / causal linear attention lowered as row reductions and element maps
       "a01_attention", "x_l_linattn", "x_l_gqa", "a02_attention_128", "x_a_rect",
       "x_a_32x16", "x_a_256x64", "x_a_batched",
       # bool masks and where; tanh and sigmoid from this back end's own exp
       "x_p_where", "x_p_cmp_mask", "x_p_elu_where", "x_p_leaky_where", "x_p_mask_and", "x_p_mask_float",
       "x_p_mask_mul", "x_p_mask_not", "x_p_gelu_tanh", "x_p_mish", "x_p_sigmoid", "x_p_tanh",
       "x_p_tanhshrink",
       # scans written as per-element serial loops
       "x_r_cumsum", "x_r_cumsum_rows", "x_l_ssm_decay",
       # Select over index conditions: rotary embedding, the SSM scan in matrix form
       "x_l_rope", "x_l_ssm_scan",
       # pow and sin / cos
       "x_p_pow3", "x_p_pow_frac", "x_p_pow_tensor", "x_p_neg_pow", "x_p_sin_cos",
       # integer / f64 reductions, serialised per output
       "x_d_f64_sum", "x_d_f64_softmax", "x_d_i32_max", "x_d_i64_max", "x_d_i32_sum",
       # integer and f64 element maps
       "x_d_f32_to_i32", "x_d_f64_add", "x_d_f64_div", "x_d_f64_exp", "x_d_i32_abs_sub",
       "x_d_i32_add", "x_d_i32_bitwise", "x_d_i32_cmp", "x_d_i32_floordiv", "x_d_i32_floordiv_c",
       "x_d_i32_mixed", "x_d_i32_rem", "x_d_i32_rshift", "x_d_i32_to_f32", "x_d_i32_where",
       "x_d_i64_cumsum", "x_d_i64_mul_add", "x_q_int4_unpack",]


@pytest.mark.gpu
@pytest.mark.parametrize("pid", MAP)
def test_map_matches_golden(runtime, pid):
    from emmyrt.runner import run_problem
    from oracle.refs import problem_expected
    d = GOLDEN / pid
    meta = json.loads((d / "meta.json").read_text())
    out = run_problem(d)["outputs"]
    exp = dict(np.load(d / "expected.npz"))
    ora = problem_expected(meta)
    for name, ref in exp.items():
        got = out[name].reshape(ref.shape)
        assert np.allclose(got, ref, rtol=meta["rtol"], atol=meta["atol"]), \
            f"{pid}:{name} max abs err {np.max(np.abs(got - ref))}"
        o = np.asarray(ora[name]).reshape(ref.shape)
        if meta["rtol"] == 0 and meta["atol"] == 0:
            assert np.array_equal(got, o)
        else:
            assert np.allclose(got, o, rtol=meta["rtol"], atol=meta["atol"])
