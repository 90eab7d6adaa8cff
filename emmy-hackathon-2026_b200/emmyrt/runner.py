"""Run Emmy problems locally on a B200: the replacement for the reference's submit.py.

For each kernel of a problem (meta.json order, ``submit.py:80``):

1. compile its IR with this back end (``compiler.load`` + ``compile_kernel``);
2. assemble with ptxas for sm_100a and load the cubin;
3. build the arguments the way the reference's runner did (``docs/API.md:40-53``):
   ``seed`` -> ``np.random.default_rng(seed).standard_normal(shape)``, ``data`` ->
   the exact values, ``output`` -> zero-filled, ``intermediate`` -> the buffer an
   earlier kernel wrote (kept on the device, ``submit.py:113-122``);
4. re-zero ``zero_outputs`` before every launch (``docs/API.md:51-53``);
5. launch with the module's own launch descriptor plus the extra parameters it
   asks for (scratch, tensor maps), wait with a deadline;
6. compare final outputs to ``expected.npz`` with ``np.allclose(rtol, atol)``
   (``submit.py:141-159``).
"""

from __future__ import annotations

import ctypes
import json
import sys
import time
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import (DeviceBuffer, Event, Module, PreparedLaunch, function_attribute, init, launch,
               stream_wait, tensor_map, CU_FUNC_ATTRIBUTE_NUM_REGS, lib, check)

_PKG = Path(__file__).resolve().parents[1]
if str(_PKG) not in sys.path:
    sys.path.insert(0, str(_PKG))

from compiler import compile_kernel, load, parse_launch  # noqa: E402

from hostfmt import NP_DTYPE, bf16_bits_to_f32, f32_to_bf16_bits  # noqa: E402,F401


def host_array(dtype: str, values) -> np.ndarray:
    """Host representation of a buffer of IR dtype ``dtype`` from float values."""
    if dtype == "bf16":
        return f32_to_bf16_bits(np.asarray(values, dtype=np.float32))
    return np.asarray(values).astype(NP_DTYPE[dtype])


def as_f32(dtype: str, a: np.ndarray) -> np.ndarray:
    """A downloaded buffer as floats for comparison: f32, except f64 and i64 buffers,
    which keep their precision as f64."""
    if dtype == "bf16":
        return bf16_bits_to_f32(a)
    if dtype in ("f64", "i64"):
        return a.astype(np.float64)
    return a.astype(np.float32)


def seeded_input(arg: dict) -> np.ndarray:
    """The runner's input fill: ``default_rng(seed).standard_normal(shape)`` (docs/API.md:46)."""
    shape = tuple(arg["shape"]) or (1,)
    if "seed" in arg:
        vals = np.random.default_rng(arg["seed"]).standard_normal(shape)
    elif "data" in arg:
        vals = np.asarray(arg["data"], dtype=np.float64).reshape(shape)
    else:
        vals = np.zeros(shape)
    return host_array(arg["dtype"], vals)


# ---------------------------------------------------------------------------
# compiled kernels


@dataclass
class CompiledKernel:
    spec: object
    ptx: str
    launch: dict
    module: Module
    function: int
    scratch: dict = field(default_factory=dict)

    @classmethod
    def from_ir(cls, ir_path) -> "CompiledKernel":
        spec = load(ir_path)
        return cls.from_spec(spec)

    @classmethod
    def from_spec(cls, spec) -> "CompiledKernel":
        ptx = compile_kernel(spec)
        return cls.from_ptx(spec, ptx)

    @classmethod
    def from_module(cls, ptx: str, entry: str, buffers) -> "CompiledKernel":
        """A template module emitted directly (not from an IR file): its parameters
        are the pointer ``buffers`` in order, then the descriptor's extras."""
        from compiler.loader import KernelSpec, Param
        spec = KernelSpec(entry, (), tuple(Param(b, "u64", ()) for b in buffers), None, None, {})
        return cls.from_ptx(spec, ptx)

    @classmethod
    def from_ptx(cls, spec, ptx: str) -> "CompiledKernel":
        desc = parse_launch(ptx)
        mod = Module(ptx)
        fn = mod.function(spec.name)
        if desc.get("smem", 0) > 48 * 1024:
            check(lib.emmy_rt_function_set_max_dynamic_smem(fn, int(desc["smem"])), "max smem")
        return cls(spec, ptx, desc, mod, fn)

    @property
    def registers(self) -> int:
        return function_attribute(self.function, CU_FUNC_ATTRIBUTE_NUM_REGS)

    def params(self, ptrs: dict) -> list:
        """Kernel parameters: meta.json arg_order pointers, then the descriptor's extras."""
        out = []
        for p in self.spec.params:
            if p.scalar:
                raise NotImplementedError("by-value scalar parameters")
            out.append(ctypes.c_uint64(int(ptrs[p.name])))
        for i, extra in enumerate(self.launch.get("extra_params", [])):
            kind = extra["kind"]
            if kind == "scratch":
                buf = self.scratch.get(i)
                if buf is None:
                    buf = DeviceBuffer(extra["bytes"])
                    buf.zero()
                    self.scratch[i] = buf
                out.append(ctypes.c_uint64(buf.ptr))
            elif kind == "tmap":
                out.append(tensor_map(int(ptrs[extra["buffer"]]) + int(extra.get("offset_bytes", 0)),
                                      extra["dtype"], extra["dims"], extra["strides"], extra["box"],
                                      extra.get("swizzle", 128)))
            elif kind == "status":
                buf = self.scratch.get(i)
                if buf is None:
                    buf = DeviceBuffer(16)
                    buf.zero()
                    self.scratch[i] = buf
                out.append(ctypes.c_uint64(buf.ptr))
            else:
                raise NotImplementedError(f"launch parameter kind {kind}")
        return out

    def __call__(self, ptrs: dict, stream: int = 0, params: list | None = None) -> None:
        d = self.launch
        launch(self.function, d["grid"], d["block"], d.get("cluster", [1, 1, 1]), d.get("smem", 0),
               stream, params if params is not None else self.params(ptrs), self.launch_flags)

    @property
    def launch_flags(self) -> int:
        """Programmatic dependent launch for modules that wait for their predecessor."""
        from . import LAUNCH_PDL
        return LAUNCH_PDL if self.launch.get("pdl") else 0

    def prepare(self, params: list) -> PreparedLaunch:
        """A ready-to-fire launch of this kernel with fixed parameters."""
        d = self.launch
        return PreparedLaunch(self.function, d["grid"], d["block"], d.get("cluster", [1, 1, 1]),
                              d.get("smem", 0), params, self.launch_flags)

    def status(self) -> int:
        """The kernel's device status word (0 = ok; non-zero = a bounded wait gave up).

        A launch that gave up may leave the counters in its scratch (split-K tickets, a
        reduction's ticket) partly counted; a non-zero status therefore re-zeroes the
        module's scratch and status word, so the next launch starts clean (its result is
        still the caller's to discard)."""
        for i, extra in enumerate(self.launch.get("extra_params", [])):
            if extra["kind"] == "status" and i in self.scratch:
                out = np.zeros(4, dtype=np.uint32)
                self.scratch[i].download(out)
                if out[0]:
                    for buf in self.scratch.values():
                        buf.zero()
                    check(lib.emmy_rt_stream_synchronize(0), "sync")
                return int(out[0])
        return 0


# ---------------------------------------------------------------------------
# problems


@dataclass
class KernelResult:
    entry: str
    registers: int
    us: float | None
    outputs: dict


def run_problem(pdir, iters: int = 0, timeout_s: float = 60.0, device: int = 0) -> dict:
    """Compile and run every kernel of a problem; returns final outputs and per-kernel info."""
    pdir = Path(pdir)
    init(device)
    meta = json.loads((pdir / "meta.json").read_text())
    bufs: dict[str, DeviceBuffer] = {}
    dtypes: dict[str, tuple] = {}
    results = []
    for k in meta["kernels"]:
        ck = CompiledKernel.from_ir(pdir / f"{k['entry']}.ir.json")
        for a in k["args"]:
            name = a["name"]
            dtypes[name] = (a["dtype"], tuple(a["shape"]) or (1,))
            if a.get("intermediate"):
                if name not in bufs:
                    raise RuntimeError(f"{k['entry']} needs {name} from an earlier kernel")
                continue
            host = seeded_input(a) if not a.get("output") else \
                np.zeros(tuple(a["shape"]) or (1,), dtype=NP_DTYPE[a["dtype"]])
            buf = bufs.get(name)
            if buf is None:
                buf = DeviceBuffer(host.nbytes)
                bufs[name] = buf
            buf.upload(host)
        ptrs = {n: b.ptr for n, b in bufs.items()}
        params = ck.params(ptrs)
        for z in k.get("zero_outputs", []):
            bufs[z].zero()
        ck(ptrs, 0, params)
        stream_wait(0, timeout_s)
        if ck.status():
            raise RuntimeError(f"{k['entry']}: kernel reported status {ck.status()}")
        us = None
        if iters:
            fire = ck.prepare(params)
            e0, e1 = Event(), Event()
            e0.record(0)
            for _ in range(iters):
                for z in k.get("zero_outputs", []):
                    bufs[z].zero()
                fire(0)
            e1.record(0)
            e1.synchronize()
            us = e0.elapsed_ms(e1) * 1e3 / iters
            for z in k.get("zero_outputs", []):   # leave the single-launch result
                bufs[z].zero()
            ck(ptrs, 0, params)
            stream_wait(0, timeout_s)
        outs = {}
        for a in k["args"]:
            if a.get("output"):
                dt, shape = dtypes[a["name"]]
                host = np.zeros(shape, dtype=NP_DTYPE[dt])
                bufs[a["name"]].download(host)
                outs[a["name"]] = as_f32(dt, host)
        results.append(KernelResult(k["entry"], ck.registers, us, outs))
    final = {}
    for r in results:
        final.update(r.outputs)
    return {"meta": meta, "kernels": results, "outputs": final}


def check_problem(pdir, **kw) -> list[tuple[str, bool, float]]:
    """Run a problem and compare its graph outputs with expected.npz."""
    pdir = Path(pdir)
    res = run_problem(pdir, **kw)
    meta = res["meta"]
    expected = dict(np.load(pdir / "expected.npz"))
    rows = []
    for name, ref in expected.items():
        got = res["outputs"][name].reshape(ref.shape)
        ok = bool(np.allclose(got, ref.astype(np.float32), rtol=meta["rtol"], atol=meta["atol"]))
        err = float(np.max(np.abs(got - ref))) if got.size else 0.0
        rows.append((name, ok, err))
    return rows


def main(argv=None) -> int:
    import argparse
    ap = argparse.ArgumentParser(description="run one Emmy problem on the local GPU")
    ap.add_argument("problem")
    ap.add_argument("--iters", type=int, default=0)
    a = ap.parse_args(argv)
    ok = True
    for name, good, err in check_problem(a.problem, iters=a.iters):
        print(f"{'PASS' if good else 'FAIL'}  {name}: max abs err {err:.3e}")
        ok &= good
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
