"""Element-map kernels on the B200 against the golden vectors: f32 add / mul, e4m3 / bf16 / f16
casts inside a kernel (all exact: rtol = atol = 0 in the fixtures)."""

import json

import numpy as np
import pytest

from conftest import GOLDEN

MAP = ["x_p_odd7", "x_p_odd1001", "x_q_fp8_e4m3", "x_q_fp8_e4m3_sat", "x_q_fp8_scaled", "x_q_bf16_cast",
       "x_q_bf16_math", "x_q_f16_scalar"]


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
        assert np.array_equal(got, np.asarray(ora[name]).reshape(ref.shape))
