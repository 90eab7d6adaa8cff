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


def _bench():
    import importlib
    import sys
    sys.path.insert(0, str(ROOT))
    return importlib.import_module("bench")


def test_regime_follows_region_length_and_power_cap():
    b = _bench()
    assert b.regime_of(0.05, {"reasons": []}) == "burst"
    assert b.regime_of(1.2, {"reasons": []}) == "sustained"
    assert b.regime_of(0.05, {"reasons": ["sw_power_cap"]}) == "sustained"


def test_roofline_fraction_and_denominators(monkeypatch):
    """frac = achieved / the peak of the region's regime; FP8 against twice the bf16
    figures; HBM-bound workloads against the copy bandwidth; traffic from the committed
    ncu summary at one GPU only."""
    b = _bench()
    peaks = {"hbm_gbs": 6000.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0}
    monkeypatch.setattr(b, "measured_peaks", lambda: (peaks, "measured"))
    clocks = {"reasons": [], "sm_mhz": 1965.0, "sm_max_mhz": 1965}
    r = b.roofline("gemm_8192", "TFLOP/s", 1.6e12, 1.25e-3, clocks, 0.02, 1)
    assert r["bound"] == "tensor" and r["regime"] == "burst"
    assert abs(r["achieved"] - 1280.0) < 1e-6 and abs(r["frac"] - 0.8) < 1e-9
    assert r["traffic"] == b.traffic_from_profile("gemm_8192")
    r = b.roofline("gemm_8192", "TFLOP/s", 1.6e12, 1.25e-3, clocks, 0.02, 8)
    assert r["traffic"] is None
    r = b.roofline("fp8_8192", "TFLOP/s", 1.6e12, 1.0e-3, {"reasons": ["sw_power_cap"]}, 0.5, 1)
    assert r["peak"] == 2 * 1400.0 and r["regime"] == "sustained"
    assert abs(r["frac_of_burst"] - 1600.0 / 3200.0) < 1e-9
    r = b.roofline("sum", "GB/s", 6.0e9, 1.0e-3, {"reasons": []}, 0.5, 1)
    assert r["bound"] == "hbm" and r["peak"] == 6000.0 and abs(r["frac"] - 1.0) < 1e-9


def test_config_and_input_bytes_cover_every_workload():
    b = _bench()
    import baseline_configs as bc
    for name in bc.ORDER:
        for world in (1, 2, 8):
            c = b.config_of(name, world)
            assert c["workload"] == name and c["l2"]
            total = sum(b._input_bytes(name, r, world) for r in range(world))
            assert total > 0
        # GEMM / FP8 keep A whole on every GPU and RMSNorm its weight row; the other
        # inputs are partitioned
        if bc.CONFIGS[name].family not in ("gemm", "fp8"):
            replicated = 4 * bc.CONFIGS[name].dims[1] if name == "rmsnorm" else 0
            assert sum(b._input_bytes(name, r, 8) for r in range(8)) == \
                b._input_bytes(name, 0, 1) + 7 * replicated
