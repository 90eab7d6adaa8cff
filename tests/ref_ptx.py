"""Launch the reference compiler's own PTX (oracle/_ref/ptx, built by
oracle/build_ref_ptx.py) on the B200 through this repository's runtime, with meta.json's
own grid / block / dynamic shared memory and the reference runner's argument rules
(docs/API.md:40-53: seeded inputs, constants as 1-element buffers, zero_outputs
re-zeroed before every launch).  Test infrastructure: the second oracle and the
same-GPU baseline."""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
REF_PTX = ROOT / "oracle" / "_ref" / "ptx"


def available(name: str) -> bool:
    return (REF_PTX / name / "meta.json").exists()


class ReferenceKernel:
    def __init__(self, ptx_path: Path, kmeta: dict):
        import emmyrt
        from emmyrt import Module, check, lib
        self.meta = kmeta
        self.module = Module(ptx_path.read_text())
        self.function = self.module.function(kmeta["entry"])
        smem = int(kmeta.get("smem_bytes", 0))
        if smem > 48 * 1024:
            check(lib.emmy_rt_function_set_max_dynamic_smem(self.function, smem), "max smem")
        self.emmyrt = emmyrt

    def prepare(self, ptrs: dict):
        params = [ctypes.c_uint64(int(ptrs[n])) for n in self.meta["arg_order"]]
        k = self.meta
        return self.emmyrt.PreparedLaunch(self.function, k["grid"], k["block"], [1, 1, 1],
                                          int(k.get("smem_bytes", 0)), params)


def run_reference(name: str, iters: int = 0):
    """Run every kernel of a reference-built problem; returns (outputs, per-kernel us)."""
    import emmyrt
    from emmyrt import DeviceBuffer, Event
    from emmyrt.runner import NP_DTYPE, as_f32, seeded_input
    emmyrt.init(0)
    d = REF_PTX / name
    meta = json.loads((d / "meta.json").read_text())
    bufs, dtypes, times, outs = {}, {}, [], {}
    for k in meta["kernels"]:
        rk = ReferenceKernel(d / f"{k['entry']}.ptx", k)
        for a in k["args"]:
            dtypes[a["name"]] = (a["dtype"], tuple(a["shape"]) or (1,))
            if a.get("intermediate"):
                continue
            host = seeded_input(a) if not a.get("output") else \
                np.zeros(tuple(a["shape"]) or (1,), dtype=NP_DTYPE[a["dtype"]])
            if a["name"] not in bufs:
                bufs[a["name"]] = DeviceBuffer(host.nbytes)
            bufs[a["name"]].upload(host)
        fire = rk.prepare({n: b.ptr for n, b in bufs.items()})
        for z in k.get("zero_outputs", []):
            bufs[z].zero()
        fire(0)
        emmyrt.stream_wait(0, 120)
        if iters:
            e0, e1 = Event(), Event()
            e0.record(0)
            for _ in range(iters):
                for z in k.get("zero_outputs", []):
                    bufs[z].zero()
                fire(0)
            e1.record(0)
            e1.synchronize()
            times.append(e0.elapsed_ms(e1) * 1e3 / iters)
            for z in k.get("zero_outputs", []):
                bufs[z].zero()
            fire(0)
            emmyrt.stream_wait(0, 120)
        for a in k["args"]:
            if a.get("output"):
                dt, shape = dtypes[a["name"]]
                host = np.zeros(shape, dtype=NP_DTYPE[dt])
                bufs[a["name"]].download(host)
                outs[a["name"]] = as_f32(dt, host)
    return outs, times
