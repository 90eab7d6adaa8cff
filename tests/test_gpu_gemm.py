"""Parity of the tcgen05 GEMM template on the B200 against the golden vectors and the oracle."""

import json

import numpy as np
import pytest

from conftest import GOLDEN

GEMM = ["x_h_mm_1024", "x_h_mm_256", "x_h_mm_relu", "x_h_mm_residual", "x_h_mm_t_n8", "x_h_mm_t_odd",
        "x_h_bmm_t", "x_h_linear"]


@pytest.mark.gpu
@pytest.mark.parametrize("pid", GEMM)
def test_gemm_matches_golden(runtime, pid):
    from emmyrt.runner import run_problem
    from oracle.refs import problem_expected
    d = GOLDEN / pid
    meta = json.loads((d / "meta.json").read_text())
    res = run_problem(d)
    for k in res["kernels"]:
        assert k.entry
    exp = dict(np.load(d / "expected.npz"))
    ora = problem_expected(meta)
    for name, ref in exp.items():
        got = res["outputs"][name].reshape(ref.shape)
        err = np.max(np.abs(got - ref.astype(np.float32)))
        assert np.allclose(got, ref.astype(np.float32), rtol=meta["rtol"], atol=meta["atol"]), \
            f"{pid}:{name} max abs err {err}"
        o = np.asarray(ora[name], dtype=np.float32).reshape(ref.shape)
        assert np.allclose(got, o, rtol=meta["rtol"], atol=meta["atol"])
