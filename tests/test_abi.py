"""The C-ABI library loads without a GPU and exports every symbol include/emmyrt.h declares."""

import re

from conftest import ROOT


def test_exports_match_header():
    import emmyrt
    header = (ROOT / "include" / "emmyrt.h").read_text()
    declared = set(re.findall(r"\b(emmy_rt_\w+)\s*\(", header))
    assert declared, "no declarations found"
    static = emmyrt.static_scratch_lib()
    for name in declared:
        owner = static if name in emmyrt.STATIC_SIGNATURES else emmyrt.lib
        assert hasattr(owner, name), f"{name} is not exported"
    assert declared == set(emmyrt.SIGNATURES) | set(emmyrt.STATIC_SIGNATURES), \
        "ctypes signatures out of sync with the header"
    assert emmyrt.lib.emmy_rt_version() == 1


def test_static_scratch_rejects_oversize_without_touching_the_gpu():
    import ctypes
    import emmyrt
    static = emmyrt.static_scratch_lib()
    args = (ctypes.c_uint64 * 2)(0, 0)
    # the size check comes before any CUDA call
    rc = static.emmy_rt_full_reduce_static_scratch(0, 1, 32, args, 2, 64 * 1024 + 1, 0)
    assert rc == emmyrt.EMMY_RT_ESCRATCH


def test_static_scratch_need_follows_the_grid_not_the_claim():
    """The kernel writes 16 + 8 * grid bytes: a large grid is rejected even when the
    caller claims a small scratch, before any CUDA call."""
    import ctypes
    import emmyrt
    static = emmyrt.static_scratch_lib()
    args = (ctypes.c_uint64 * 2)(0, 0)
    fits = (64 * 1024 - 16) // 8                      # 8190 CTAs fill the 64 KiB exactly
    for grid in (fits + 1, 1 << 20):
        rc = static.emmy_rt_full_reduce_static_scratch(0, grid, 32, args, 2, 16 + 8, 0)
        assert rc == emmyrt.EMMY_RT_ESCRATCH, grid


def test_calls_before_init_fail_cleanly():
    import ctypes
    import emmyrt
    n = ctypes.c_int()
    # no compute call without a GPU: the runtime reports "not initialised", never crashes
    if not emmyrt._initialised:
        assert emmyrt.lib.emmy_rt_device_count(ctypes.byref(n)) == -5
        assert b"emmy_rt_init" in emmyrt.lib.emmy_rt_last_error()


def test_graph_holds_what_its_launches_refer_to(monkeypatch):
    """A captured graph keeps its enqueue callable and the owners named in ``keep`` alive,
    so the buffers its launches address are not freed while it can be replayed (the
    capture calls are faked: no GPU is touched)."""
    import gc
    import weakref
    import emmyrt

    class Owner:                       # stands in for a DeviceBuffer / CompiledKernel
        pass

    class FakeLib:
        def emmy_rt_graph_begin(self, stream):
            return 0

        def emmy_rt_graph_end(self, stream, out):
            return 0

        def emmy_rt_graph_destroy(self, handle):
            return 0

    monkeypatch.setattr(emmyrt, "lib", FakeLib())
    buf, kernel = Owner(), Owner()
    refs = weakref.ref(buf), weakref.ref(kernel)

    class Stream:
        handle = 0

    g = emmyrt.Graph.capture(Stream(), lambda k=kernel: None, keep=(buf,))
    del buf, kernel
    gc.collect()
    assert all(r() is not None for r in refs)
    del g
    gc.collect()
    assert all(r() is None for r in refs)
