"""The C-ABI library loads without a GPU and exports every symbol include/emmyrt.h declares."""

import re

from conftest import ROOT


def test_exports_match_header():
    import emmyrt
    header = (ROOT / "include" / "emmyrt.h").read_text()
    declared = set(re.findall(r"\b(emmy_rt_\w+)\s*\(", header))
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(emmyrt.lib, name), f"libemmyrt.so does not export {name}"
    assert declared == set(emmyrt.SIGNATURES), "ctypes signatures out of sync with the header"
    assert emmyrt.lib.emmy_rt_version() == 1


def test_calls_before_init_fail_cleanly():
    import ctypes
    import emmyrt
    n = ctypes.c_int()
    # no compute call without a GPU: the runtime reports "not initialised", never crashes
    if not emmyrt._initialised:
        assert emmyrt.lib.emmy_rt_device_count(ctypes.byref(n)) == -5
        assert b"emmy_rt_init" in emmyrt.lib.emmy_rt_last_error()
