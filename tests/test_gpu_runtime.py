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
