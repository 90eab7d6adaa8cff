"""bench.py's command line on a machine without a GPU: the vendor-library arm answers
with an ``unavailable`` line instead of failing, and the argument choices stay as the
driver calls them."""

import json
import subprocess
import sys

import pytest

from conftest import ROOT


def _run(*args):
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True,
                       text=True, timeout=300, cwd=ROOT)
    return r.returncode, r.stdout.strip().splitlines()


def test_library_arm_without_a_gpu_reports_unavailable():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present: the arm would measure")
    rc, out = _run("--impl", "library", "--workload", "gemm_512")
    assert rc == 0
    line = json.loads(out[-1])
    assert line["impl"] == "library" and "unavailable" in line


def test_impl_choices():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True,
                       text=True, timeout=120, cwd=ROOT)
    assert r.returncode == 0
    for choice in ("ours", "reference", "library"):
        assert choice in r.stdout
