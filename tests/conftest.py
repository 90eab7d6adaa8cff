import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "emmy-hackathon-2026_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden" / "problems"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the sm_100a kernels)")


@pytest.fixture(scope="session")
def golden():
    return GOLDEN


@pytest.fixture(scope="session")
def runtime():
    """The native runtime with device 0 initialised (GPU tests only)."""
    import emmyrt
    emmyrt.init(0)
    return emmyrt
