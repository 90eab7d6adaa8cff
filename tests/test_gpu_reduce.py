"""Parity of the streaming reduction kernels on the B200 (through the C-ABI runtime)."""

import json

import numpy as np
import pytest

from conftest import GOLDEN

REDUCE = ["f01_rmsnorm", "f02_row_softmax", "f03_l2norm", "r01_array_sum", "r02_big_sum", "r03_mean",
          "r04_row_sum", "x_l_rmsnorm_w", "x_r_unpinned_sum", "x_r_rowmax", "x_r_mean_rows",
          "x_r_rowsum_wide", "x_f_softmax_wide", "x_f_softmax_scaled", "x_f_softmax_odd", "x_r_sumsq",
          "x_r_max", "x_r_abs_max", "x_r_sum100", "x_r_sum1000", "x_r_mean_3d",
          # leading / middle axes, split rows, fused row kernels
          "x_r_colsum", "x_r_sum_dim0", "x_r_mean_mid_3d", "x_r_unpinned_rows", "x_f_layernorm_ish",
          "x_f_max_sub", "x_f_rmsnorm_silu", "x_f_softmax_dim0", "x_f_layernorm", "x_f_log_softmax",
          # f16 inputs and results (f32 arithmetic with the IR's per-op f16 roundings)
          "x_d_f16_softmax", "x_d_f16_sum", "x_d_f16_mean", "x_d_f16_sq_mean", "x_d_f16_dot",
          "x_d_f16_dot_f32",
          # an f32 SwiGLU that emmy lowers as a row reduction over K
          "x_l_swiglu",
          # softmax of tanh-capped logits (30 tanh(x / 30))
          "x_l_softcap"]


# row reductions that are dot products over K (cancellation in f32 sums): no 1e-5 bar
MATMUL_LIKE = {"x_l_swiglu"}


@pytest.mark.gpu
@pytest.mark.parametrize("pid", REDUCE)
def test_reduction_matches_golden_and_oracle(runtime, pid):
    from emmyrt.runner import run_problem
    from oracle.refs import problem_expected
    d = GOLDEN / pid
    meta = json.loads((d / "meta.json").read_text())
    res = run_problem(d)
    exp = dict(np.load(d / "expected.npz"))
    ora = problem_expected(meta)
    for name, ref in exp.items():
        got = res["outputs"][name].reshape(ref.shape)
        assert np.allclose(got, ref, rtol=meta["rtol"], atol=meta["atol"]), \
            f"{pid}:{name} max abs err {np.max(np.abs(got - ref))}"
        if ref.dtype != np.float32 or pid in MATMUL_LIKE:
            continue      # 16-bit results (one f16 ulp ~ 1e-3) and dot products: the fixture's tolerance
        # the BASELINE reduction bar: within 1e-5 relative of the f64 oracle
        o = np.asarray(ora[name], dtype=np.float64).reshape(ref.shape)
        tol = 1e-5 * np.maximum(np.abs(o), 1.0) if "sum" in pid or "mean" in pid else 1e-5 * np.abs(o) + 1e-6
        assert np.all(np.abs(got - o) <= tol), f"{pid}:{name} oracle err {np.max(np.abs(got - o))}"


@pytest.mark.gpu
def test_rerun_is_deterministic(runtime):
    from emmyrt.runner import run_problem
    a = run_problem(GOLDEN / "x_r_unpinned_sum")["outputs"]["sum_1"]
    b = run_problem(GOLDEN / "x_r_unpinned_sum")["outputs"]["sum_1"]
    assert np.array_equal(a, b)


@pytest.mark.gpu
def test_row_reduce_pdl_chain(runtime, golden):
    """Programmatic dependent launch on the row template: y1 = rmsnorm(x, w) and
    y2 = rmsnorm(y1, w) launched back to back on one stream with no host sync; the second
    waits (griddepcontrol.wait) for the first before reading y1."""
    import json
    import emmyrt
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel, seeded_input
    from oracle.refs import rmsnorm
    d = golden / "x_l_rmsnorm_w"
    meta = json.loads((d / "meta.json").read_text())
    k = meta["kernels"][0]
    ck = CompiledKernel.from_ir(d / f"{k['entry']}.ir.json")
    assert ck.launch["pdl"] and ck.launch_flags == emmyrt.LAUNCH_PDL
    args = {a["name"]: a for a in k["args"]}
    host = {n: seeded_input(a) for n, a in args.items()}
    bufs = {n: DeviceBuffer(h.nbytes) for n, h in host.items()}
    for n, h in host.items():
        bufs[n].upload(h)
    y2 = DeviceBuffer(host["mul_1"].nbytes)
    for rep in range(3):
        bufs["mul_1"].upload(np.full_like(host["mul_1"], np.nan))
        y2.zero()
        first = ck.prepare(ck.params({n: b.ptr for n, b in bufs.items()}))
        second = ck.prepare(ck.params({**{n: b.ptr for n, b in bufs.items()},
                                       "x0": bufs["mul_1"].ptr, "mul_1": y2.ptr}))
        first(0)
        second(0)
        emmyrt.stream_wait(0, 60)
        got1, got2 = np.zeros_like(host["mul_1"]), np.zeros_like(host["mul_1"])
        bufs["mul_1"].download(got1)
        y2.download(got2)
        assert np.isfinite(got2).all(), f"rep {rep}: the second kernel read y1 too early"
        ref1 = rmsnorm(host["x0"], host["x1"], 1e-6)
        np.testing.assert_allclose(got1, ref1, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(got2, rmsnorm(got1, host["x1"], 1e-6), rtol=1e-5, atol=1e-6)
