"""The runtime's stream ordering and CUDA graph entry points on the B200."""

import numpy as np
import pytest

from conftest import GOLDEN


def _rmsnorm_kernel():
    import json
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel, seeded_input
    d = GOLDEN / "x_l_rmsnorm_w"
    meta = json.loads((d / "meta.json").read_text())
    k = meta["kernels"][0]
    ck = CompiledKernel.from_ir(d / f"{k['entry']}.ir.json")
    bufs = {}
    for a in k["args"]:
        h = seeded_input(a)
        bufs[a["name"]] = DeviceBuffer(h.nbytes)
        bufs[a["name"]].upload(h)
    out = [a for a in k["args"] if a.get("output")][0]
    return ck, bufs, out


@pytest.mark.gpu
def test_graph_replay_matches_stream_launches(runtime):
    import emmyrt
    from emmyrt import Graph, Stream
    from emmyrt.runner import NP_DTYPE
    ck, bufs, out = _rmsnorm_kernel()
    fire = ck.prepare(ck.params({n: b.ptr for n, b in bufs.items()}))
    shape = tuple(out["shape"])
    fire(0)
    emmyrt.stream_wait(0, 60)
    ref = np.zeros(shape, NP_DTYPE[out["dtype"]])
    bufs[out["name"]].download(ref)
    bufs[out["name"]].zero()
    s = Stream()
    g = Graph.capture(s, lambda: [fire(s.handle) for _ in range(3)])
    got = np.zeros_like(ref)
    bufs[out["name"]].download(got)
    assert not got.any(), "capture must record the launches, not run them"
    g.upload(0)
    g.launch(0)
    emmyrt.stream_wait(0, 60)
    bufs[out["name"]].download(got)
    assert np.array_equal(got, ref)


@pytest.mark.gpu
def test_stream_wait_event_orders_streams(runtime):
    import emmyrt
    from emmyrt import DeviceBuffer, Event, HostBuffer, Stream, check, lib
    n = 1 << 24
    src = np.arange(n, dtype=np.float32)
    hb = HostBuffer(src.nbytes)
    hb.array(np.float32, src.shape)[...] = src
    d1, d2 = DeviceBuffer(src.nbytes), DeviceBuffer(src.nbytes)
    d2.zero()
    a, b, ev = Stream(), Stream(), Event()
    check(lib.emmy_rt_memcpy_htod(d1.ptr, hb.ptr, src.nbytes, a.handle), "htod")
    ev.record(a.handle)
    b.wait(ev)                       # the device copy on b must see the upload on a
    check(lib.emmy_rt_memcpy_dtod(d2.ptr, d1.ptr, src.nbytes, b.handle), "dtod")
    emmyrt.stream_wait(b.handle, 60)
    out = np.zeros_like(src)
    d2.download(out)
    assert np.array_equal(out, src)


def _stuck_wait_kernel():
    """One thread waits on an mbarrier that nothing arrives on, through the templates' own
    bounded wait (2 s of %globaltimer): the wait gives up, records its role's status bit,
    raises the CTA's abort flag and the kernel returns -- no trap, no fault, no endless
    spin.  Bit 0x100 would mean the wait returned as if the barrier had completed."""
    from compiler.kernels.tc import Waits
    from compiler.ptx import Ptx, entry, module
    from emmyrt.runner import CompiledKernel
    p = Ptx()
    st, bar, ab, tid, pz = p.reg("b64"), p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("pred")
    done = p.label("done")
    p.emit(f"""
        ld.param.u64 {st}, [param__status]
        cvta.to.global.u64 {st}, {st}
        mov.u32 {bar}, gbar
        mov.u32 {ab}, gabort
        mov.u32 {tid}, %tid.x
        setp.ne.u32 {pz}, {tid}, 0
        @{pz} bra {done}
        mbarrier.init.shared::cta.b64 [{bar}], 1
        st.shared.u32 [{ab}], 0
        fence.mbarrier_init.release.cluster
    """)
    Waits(p, st, ab).wait(bar, "0", "mma", done)
    p.emit(f"red.global.or.b32 [{st}], 256")
    p.place(done)
    p.emit("ret")
    text = entry("k_stuck_wait", [".param .u64 param__status"], p, maxntid=32)
    text = text.replace("{\n", "{\n\t.shared .align 8 .b64 gbar;\n\t.shared .align 4 .u32 gabort;\n", 1)
    launch = {"kind": "probe", "grid": [1, 1, 1], "block": [32, 1, 1], "cluster": [1, 1, 1], "smem": 0,
              "extra_params": [{"kind": "status"}]}
    return CompiledKernel.from_module(module([text], launch), "k_stuck_wait", [])


@pytest.mark.gpu
def test_bounded_wait_reports_and_returns(runtime):
    # failure detection without a GPU fault: a wait that can never complete ends on its
    # own limit, the host reads the status, and the context keeps working
    import time
    import emmyrt
    from compiler.kernels.tc import STATUS, TIMEOUT_NS
    ck = _stuck_wait_kernel()
    t0 = time.perf_counter()
    ck({}, 0)
    emmyrt.stream_wait(0, 30)
    dt = time.perf_counter() - t0
    assert ck.status() == STATUS["mma"]
    assert TIMEOUT_NS * 1e-9 * 0.9 <= dt < 30
    rk, bufs, out = _rmsnorm_kernel()
    rk({n: b.ptr for n, b in bufs.items()}, 0)
    emmyrt.stream_wait(0, 30)
    assert rk.status() == 0
