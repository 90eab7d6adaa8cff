"""Second oracle: the reference compiler's own PTX (mma.sync / SIMT, built for sm_89 and
assembled for sm_100a) run on the same B200 reproduces the golden vectors, and this back
end's sm_100a kernels agree with it (GEMM, RMSNorm, L2 norm, row and global sums)."""

import json

import numpy as np
import pytest

from conftest import GOLDEN
from ref_ptx import available, run_reference

FIXTURES = ["x_h_mm_1024", "x_h_mm_256", "x_h_mm_relu", "f01_rmsnorm", "f03_l2norm", "x_l_rmsnorm_w",
            "r02_big_sum", "r04_row_sum", "x_r_unpinned_sum", "x_r_rowsum_wide"]


@pytest.mark.gpu
@pytest.mark.parametrize("pid", FIXTURES)
def test_reference_ptx_agrees(runtime, pid):
    if not available(pid):
        pytest.skip("reference PTX not built (python oracle/build_ref_ptx.py)")
    from emmyrt.runner import run_problem
    d = GOLDEN / pid
    meta = json.loads((d / "meta.json").read_text())
    ref_out, _ = run_reference(pid)
    ours = run_problem(d)["outputs"]
    exp = dict(np.load(d / "expected.npz"))
    for name, gold in exp.items():
        r = ref_out[name].reshape(gold.shape)
        o = ours[name].reshape(gold.shape)
        assert np.allclose(r, gold.astype(np.float32), rtol=meta["rtol"], atol=meta["atol"]), \
            f"reference PTX misses its own golden vector ({pid}:{name})"
        assert np.allclose(o, r, rtol=meta["rtol"], atol=meta["atol"]), \
            f"{pid}:{name}: max |ours - reference| {np.max(np.abs(o - r))}"
