#!/usr/bin/env python3
"""Benchmark of the B200 back end on BASELINE.json's configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME|all]
                    [--impl ours|reference|library] [--no-cpu]

One step = one launch of the kernel ``compile.py`` emits for a configuration (its IR
synthesised from the reference's IR family at the configured size), over inputs
already resident in HBM.  The headline (the line's top-level ``value``) is the bf16
GEMM at M=N=K=8192, BASELINE.json's TFLOP/s target, timed over exactly K steps.  Every
other configuration of BASELINE.json (attention, FP8 GEMM, the other GEMM sizes,
RMSNorm, row softmax, the 2^31 sum) is measured in the same run and reported under
``workloads``, each with its own value, roofline, CPU baseline, end-to-end figure and
SM clocks; their timed regions are stretched to at least 0.3 s.

Multi-GPU (torchrun, one process per GPU): each configuration is ONE problem split
across the GPUs (strong scaling): GEMM and FP8 by N-panel (A replicated), attention by
batch (batch x head pairs), RMSNorm and softmax by rows, the sum by chunks whose f64
partials one NCCL all-reduce finishes inside every step.  ``value`` is the whole
problem's work divided by the slowest rank's time (CUDA events on the launching
stream, max over ranks).

``e2e`` is the same metric through the C-ABI runtime with host buffers: every step
copies its inputs up from pinned host memory and its result down (pipelined over two
device buffer sets and three streams).  ``cpu_baseline`` and ``--impl reference`` time
the torch-CPU evaluation of the configuration (the reference harness's own form of
the problem) on the host's cores, on the same bounded sample; the reference arm loads
none of this repository's native code.
"""

from __future__ import annotations

import argparse
import gc
import json
import math
import os
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "emmy-hackathon-2026_b200"))
sys.path.insert(0, str(ROOT))

import baseline_configs as bc  # noqa: E402  (pure numpy: no native library)

METRIC = "GEMM/attention TFLOP/s & reduction HBM GB/s vs B200 peak at 1/2/4/8 GPUs"
HEADLINE = "gemm_8192"
L2_BYTES = 126 * 2 ** 20
MIN_REGION_S = 0.3          # timed region of each non-headline workload
MAX_LAUNCHES = 50000
EXTRA = ("gemm_f32_4096",)  # measurable on request, not BASELINE configurations


# ---------------------------------------------------------------------------
# distributed plumbing (host side: gloo barrier / max; NCCL lives in the runtime)


class Dist:
    def __init__(self):
        self.rank = int(os.environ.get("RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        self.local = int(os.environ.get("LOCAL_RANK", 0))
        self.pg = None
        if self.world > 1:
            import torch.distributed as td
            # a rank that dies ends the others' next collective with an error within this
            # limit instead of a hang
            limit = float(os.environ.get("EMMY_PG_TIMEOUT_S", 300))
            td.init_process_group("gloo", timeout=timedelta(seconds=limit))
            self.pg = td

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def broadcast_bytes(self, b):
        if not self.pg:
            return b
        obj = [b]
        self.pg.broadcast_object_list(obj, src=0)
        return obj[0]

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# clocks (read-only NVML sampling during a timed region, every millisecond)


class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device: int, period_s: float = 0.001):
        self.samples, self.power, self.reasons, self.max_mhz = [], [], set(), None
        self.period = period_s
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _sample(self):
        nv = self.nv
        try:
            self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for b, n in self.REASONS.items():
                if bits & b:
                    self.reasons.add(n)
            if len(self.samples) % 8 == 1:          # power is the slow query
                self.power.append(nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0)
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            self._started.set()
            time.sleep(self.period)

    def __enter__(self):
        self._started = threading.Event()
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
            # the timed work starts only once sampling runs (a short region would
            # otherwise end before the thread's first samples)
            self._started.wait(1.0)
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self.t.join()
            self._sample()

    def summary(self) -> dict:
        s = sorted(self.samples)
        return {"sm_mhz": float(np.median(s)) if s else None, "sm_max_mhz": self.max_mhz,
                "samples": len(s), "period_ms": self.period * 1e3,
                "power_w_max": round(max(self.power), 1) if self.power else None,
                "reasons": sorted(self.reasons)}


# ---------------------------------------------------------------------------
# shared helpers


def to_rate(units: float, seconds: float, unit: str) -> float:
    return units / seconds / (1e12 if unit == "TFLOP/s" else 1e9)


def measured_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def traffic_from_profile(workload: str):
    """DRAM bytes per launch of the whole problem from the committed ncu summary
    (``profiles/<workload>_traffic.txt``)."""
    p = ROOT / "profiles" / f"{workload}_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            return float(line.split(":", 1)[1].strip().split()[0])
    return None


def config_of(name: str, world: int) -> dict:
    """The line's ``config`` (identical in both arms)."""
    c = bc.CONFIGS[name] if name in bc.CONFIGS else None
    if c is None:
        return {"workload": name}
    in_bytes = _input_bytes(name, 0, world)
    copies = 1 if in_bytes > L2_BYTES else -(-2 * L2_BYTES // max(1, in_bytes))
    return {"workload": name, "problem": list(c.dims), "dtype": c.dtype,
            "parallelism": f"{world} GPU(s); split by {c.shard_by}" if world > 1 else "1 GPU",
            "l2": ("inputs larger than L2" if copies == 1 else
                   f"inputs rotated over {copies} device copies ({copies * in_bytes >> 20} MiB, > L2)")}


def _input_bytes(name: str, rank: int, world: int) -> int:
    c = bc.CONFIGS[name]
    d = bc.shard_dims(name, rank, world)
    if c.family == "gemm":
        return 2 * (d["m"] * d["k"] + d["k"] * d["n"])
    if c.family == "fp8":
        return d["m"] * d["k"] + d["k"] * d["n"]      # the e4m3 operands the GEMM reads
    if name == "attention":
        return 3 * 2 * d["b"] * d["h"] * d["s"] * d["d"]
    if c.family == "row":
        r = d["rows"][1] - d["rows"][0]
        return 4 * r * d["cols"] + (4 * d["cols"] if name == "rmsnorm" else 0)
    if name == "sum":
        return 4 * (d["rows"][1] - d["rows"][0])
    raise KeyError(name)


def regime_of(region_s: float, clocks: dict) -> str:
    """burst: a short region at full clock; sustained: long enough to sit at the power cap."""
    if region_s >= 1.0 or "sw_power_cap" in clocks.get("reasons", []):
        return "sustained"
    return "burst"


def roofline(name: str, unit: str, units_per_launch: float, launch_s: float, clocks: dict,
             region_s: float, world: int) -> dict:
    peaks, kind = measured_peaks()
    achieved = to_rate(units_per_launch, launch_s, unit)
    regime = regime_of(region_s, clocks)
    if name == "fp8_8192":
        # no measured fp8 figure: the dense e4m3 rate is twice bf16's on this part
        burst, sust = 2 * float(peaks["bf16_tflops"]), 2 * float(peaks["bf16_tflops_sustained"])
        what = f"derived: 2 x {kind} bf16_tflops"
    elif name == "gemm_f32_4096":
        burst, sust = float(peaks["bf16_tflops"]) / 6, float(peaks["bf16_tflops_sustained"]) / 6
        what = f"derived: {kind} bf16_tflops / 2 (tf32) / 3 (MMAs per product)"
    elif unit == "TFLOP/s":
        burst, sust = float(peaks["bf16_tflops"]), float(peaks["bf16_tflops_sustained"])
        what = f"{kind} bf16_tflops"
    else:
        burst = sust = float(peaks["hbm_gbs"])
        what = f"{kind} hbm_gbs (copy)"
    peak = burst if regime == "burst" else sust
    out = {"bound": "tensor" if unit == "TFLOP/s" else "hbm", "achieved": round(achieved, 2),
           "peak": peak, "unit": unit, "frac": round(achieved / peak, 4),
           "peak_kind": f"{what} ({regime})", "regime": regime,
           "frac_of_burst": round(achieved / burst, 4),
           "traffic": traffic_from_profile(name) if world == 1 else None}
    if unit == "TFLOP/s" and clocks.get("sm_mhz") and clocks.get("sm_max_mhz"):
        # tensor-bound kernels scale with the SM clock: the rate the same launches would
        # reach at the maximum clock (time x median MHz / max MHz)
        out["achieved_at_max_clock"] = round(achieved * clocks["sm_max_mhz"] / clocks["sm_mhz"], 2)
    return out


# ---------------------------------------------------------------------------
# CPU side: the torch-CPU evaluation (cpu_baseline leg and the reference arm)


def cpu_measure(name: str, reps: int, warmup: int = 1) -> dict:
    from oracle import torch_cpu
    cores = torch_cpu.threads()
    inputs, units, sample = bc.cpu_sample_inputs(name)
    fn = torch_cpu.sample_fn(name, inputs)
    for _ in range(max(1, warmup)):
        fn()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    dt = float(np.median(times))
    unit = bc.CONFIGS[name].unit
    return {"value": round(to_rate(units, dt, unit), 4), "unit": unit, "cores": cores, "kind": "port",
            "sample": f"{sample}; torch-CPU evaluation of the problem's torch expression, "
                      f"median of {reps}", "ms_per_sample": round(dt * 1e3, 3), "_dt": dt,
            "_units": units}


def run_reference(args, dist: Dist) -> int:
    """The reference's CPU evaluation (torch on the host cores) of the same configurations."""
    if dist.rank != 0:
        return 0
    names = _names(args)
    head = names[0]
    workloads = {}
    for name in names:
        steps = args.steps if name == head else 3
        warm = args.warmup if name == head else 1
        r = cpu_measure(name, steps, warm)
        dt, units = r.pop("_dt"), r.pop("_units")
        unit = bc.CONFIGS[name].unit
        workloads[name] = {"value": r["value"], "unit": unit, "ms_per_step": r["ms_per_sample"],
                           "steps": steps, "cpu_baseline": r,
                           "e2e": {"value": r["value"], "unit": unit, "h2d_bytes_per_step": 0,
                                   "d2h_bytes_per_step": 0}}
        gc.collect()
    h = workloads[head]
    line = {"metric": METRIC, "impl": "reference", "value": h["value"], "unit": h["unit"],
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": h["ms_per_step"], "higher_is_better": True,
            "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None,
            "dtype": bc.CONFIGS[head].dtype, "data": "synthetic",
            "config": config_of(head, args.gpus), "cpu_baseline": h["cpu_baseline"],
            "e2e": h["e2e"], "workloads": workloads}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# vendor-library arm (context only): the same configurations through torch's CUDA kernels


def _library_ops(name: str, dev):
    """Closures that run one step of ``name`` with torch's CUDA kernels (cuBLAS bf16,
    cuBLASLt FP8 through ``torch._scaled_mm``, cuDNN and flash SDPA, torch's own
    normalisation / softmax / reduction kernels), output buffers allocated up front.
    Inputs are rotated over enough copies to exceed L2, like the other arm's."""
    import torch
    c = bc.CONFIGS[name]
    g = torch.Generator(device=dev).manual_seed(0)

    def copies(make, nbytes):
        n = 1 if nbytes > L2_BYTES else -(-2 * L2_BYTES // nbytes)
        return [make() for _ in range(n)]

    ops = {}
    if c.family == "gemm":
        m, n, k = c.dims
        ins = copies(lambda: ((0.05 * torch.randn(m, k, device=dev, generator=g)).bfloat16(),
                              (0.05 * torch.randn(k, n, device=dev, generator=g)).bfloat16()),
                     2 * (m * k + k * n))
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        ops["cublas"] = lambda i: torch.matmul(*ins[i % len(ins)], out=out)
    elif c.family == "fp8":
        m, n, k = c.dims
        f8 = torch.float8_e4m3fn
        # (A, B) with B column-major, as cuBLASLt takes it
        ins = copies(lambda: (torch.randn(m, k, device=dev, generator=g).to(f8),
                              torch.randn(n, k, device=dev, generator=g).to(f8).t()), m * k + k * n)
        sa = torch.tensor(1.0, device=dev)
        sb = torch.tensor(1.0, device=dev)
        ops["cublaslt_scaled_mm"] = lambda i: torch._scaled_mm(
            *ins[i % len(ins)], scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)
    elif name == "attention":
        from torch.nn.attention import SDPBackend, sdpa_kernel
        b, h, s, d = c.dims
        q, k_, v = (torch.randn(b, h, s, d, device=dev, generator=g).bfloat16() for _ in range(3))
        F = torch.nn.functional
        for label, be in (("cudnn_sdpa", SDPBackend.CUDNN_ATTENTION),
                          ("flash_sdpa", SDPBackend.FLASH_ATTENTION)):
            def run(i, be=be):
                with sdpa_kernel([be]):
                    return F.scaled_dot_product_attention(q, k_, v)
            ops[label] = run
    elif name == "rmsnorm":
        rows, cols = c.dims
        ins = copies(lambda: torch.randn(rows, cols, device=dev, generator=g), 4 * rows * cols)
        w = torch.rand(cols, device=dev, generator=g) + 0.5
        ops["torch_rms_norm"] = lambda i: torch.nn.functional.rms_norm(
            ins[i % len(ins)], (cols,), w, 1e-6)
    elif name == "softmax":
        x = torch.randn(*c.dims, device=dev, generator=g) * math.sqrt(2.0)
        out = torch.empty_like(x)
        ops["torch_softmax"] = lambda i: torch.softmax(x, dim=-1, out=out)
    elif name == "sum":
        x = torch.rand(c.dims[0], device=dev, generator=g) * 2 - 1
        out = torch.empty((), device=dev)
        ops["torch_sum"] = lambda i: torch.sum(x, dim=0, out=out)
    return ops


def run_library(args, dist: Dist) -> int:
    """``--impl library``: the configurations through NVIDIA's libraries via torch on one
    GPU (CUDA graphs of the launches, CUDA events, the same stretched regions and clock
    sampling as this back end's arm).  Context for the roofline fractions, not a
    reference arm: the reference has no GPU implementation of these kernels."""
    if dist.world > 1 or dist.rank != 0:
        if dist.rank == 0:
            print(json.dumps({"impl": "library", "unavailable": "one GPU only"}))
        return 0
    import torch
    if not torch.cuda.is_available():
        print(json.dumps({"impl": "library", "unavailable": "no CUDA device"}))
        return 0
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    results = {}
    for name in _names(args):
        if name not in bc.CONFIGS:
            continue
        unit = bc.CONFIGS[name].unit
        for label, op in _library_ops(name, dev).items():
            try:
                for i in range(max(3, args.warmup)):
                    op(i)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for i in range(3):
                    op(i)
                e1.record()
                e1.synchronize()
                est_s = e0.elapsed_time(e1) / 3e3
                steps = int(min(MAX_LAUNCHES, max(args.steps, math.ceil(MIN_REGION_S / max(est_s, 1e-7)))))
                s = torch.cuda.Stream()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.stream(s):
                    op(0)                      # library workspaces allocated outside capture
                    s.synchronize()
                    with torch.cuda.graph(graph, stream=s):
                        for i in range(steps):
                            op(i)
                torch.cuda.synchronize()
                with ClockSampler(dist.local) as clocks:
                    e0.record()
                    graph.replay()
                    e1.record()
                    e1.synchronize()
                ms = e0.elapsed_time(e1) / steps
                del graph
                value = to_rate(bc.work(name), ms / 1e3, unit)
                results[f"{name}/{label}"] = {"value": round(value, 2), "unit": unit,
                                              "ms_per_step": round(ms, 5), "steps": steps,
                                              "clocks": clocks.summary()}
            except Exception as e:      # a backend torch does not offer for this shape
                results[f"{name}/{label}"] = {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}
            print(json.dumps({f"{name}/{label}": results[f"{name}/{label}"]}), file=sys.stderr, flush=True)
        torch.cuda.empty_cache()
        gc.collect()
    print(json.dumps({"metric": METRIC, "impl": "library", "n_gpus": 1,
                      "torch": torch.__version__, "device": torch.cuda.get_device_name(dev),
                      "data": "synthetic (torch generator, BASELINE.json shapes)",
                      "workloads": results}), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm


class Workload:
    """One configuration's shard on this rank: compiled kernel, pinned host inputs,
    device buffer sets, and the prepared launches."""

    def __init__(self, name: str, dist: Dist, comm):
        import emmyrt
        from emmyrt import DeviceBuffer, HostBuffer
        from emmyrt.runner import CompiledKernel
        from compiler import synth
        self.name, self.dist, self.comm = name, dist, comm
        self.cfg = bc.CONFIGS[name] if name in bc.CONFIGS else None
        self.unit = self.cfg.unit if self.cfg else "TFLOP/s"
        if self.cfg is None:               # a non-BASELINE workload (e.g. the f32 GEMM)
            irs, meta = synth.baseline_problem(name)
        else:
            irs, meta = bc.shard_problem(name, dist.rank, dist.world)
        self.meta = meta
        k = meta["kernels"][0]
        self.fp8 = None
        if self.cfg is not None and self.cfg.family == "fp8":
            from emmyrt.fp8 import Fp8Gemm
            (m, kk), n = k["args"][0]["shape"], k["args"][1]["shape"][1]
            self.fp8 = Fp8Gemm(m, n, kk)
            self.ck = self.fp8.gemm
        else:
            d = synth.problem_dir(irs, meta)
            self.ck = CompiledKernel.from_ir(d / f"{k['entry']}.ir.json")
        self.host_bufs = []

        def pinned(nb):
            hb = HostBuffer(max(16, nb))
            self.host_bufs.append(hb)
            return hb.array(np.uint8, (max(16, nb),))[:nb]
        if self.cfg is not None:
            self.inputs = bc.shard_inputs(name, meta, dist.rank, dist.world, alloc=pinned)
        else:
            from hostfmt import NP_DTYPE
            self.inputs = {}
            for a in k["args"]:
                arr = pinned(int(np.prod(a["shape"] or [1])) * np.dtype(NP_DTYPE[a["dtype"]]).itemsize)
                arr = arr.view(NP_DTYPE[a["dtype"]]).reshape(tuple(a["shape"]) or (1,))
                arr[...] = (np.random.default_rng(a.get("seed", 0)).standard_normal(arr.shape)
                            if not a.get("output") else 0)
                self.inputs[a["name"]] = arr
        self.args = k["args"]
        self.in_names = [a["name"] for a in k["args"] if not a.get("output") and "data" not in a]
        self.out_names = [a["name"] for a in k["args"] if a.get("output")]
        self.in_bytes = sum(self.inputs[n].nbytes for n in self.in_names)
        dev_in = (_input_bytes(name, dist.rank, dist.world) if self.cfg is not None else self.in_bytes)
        self.copies = 1 if dev_in > L2_BYTES else -(-2 * L2_BYTES // max(1, dev_in))
        if self.fp8 is not None:
            self.copies = 1                 # the quantised operands are one set (> L2)
        self.bufsets = []
        for _ in range(self.copies):
            bufs = {}
            for a in k["args"]:
                h = self.inputs[a["name"]]
                b = DeviceBuffer(h.nbytes)
                b.upload(h)
                bufs[a["name"]] = b
            self.bufsets.append(bufs)
        if self.fp8 is not None:
            # quantisation is outside the timed region (BASELINE: "quantised before timing");
            # a sharded B needs the amax of all of B: one all-reduce (max) of the panels' amax
            bs = self.bufsets[0]
            self.fp8.quantize(bs["a"].ptr, bs["b"].ptr, amax_b_hook=self._amax_hook())
            self.params = [self.fp8.gemm_params(bs["c"].ptr)]
        else:
            self.params = [self.ck.params({n: b.ptr for n, b in bs.items()}) for bs in self.bufsets]
        self.fire = [self.ck.prepare(pp) for pp in self.params]
        # the sharded sum: f64 totals (scratch + 8) all-reduced into one f64 per rank
        self.total = None
        if self.cfg is not None and self.cfg.family == "sum" and comm is not None:
            ex = [i for i, e in enumerate(self.ck.launch["extra_params"]) if e["kind"] == "scratch"]
            off = self.ck.launch["extra_params"][ex[0]]["f64_total_offset"]
            self.partial_ptr = self.ck.scratch[ex[0]].ptr + off
            self.total = DeviceBuffer(16)
        emmyrt.synchronize()

    def _amax_hook(self):
        if self.comm is None:
            return None
        from emmyrt.dist import NCCL_FLOAT32, NCCL_MAX
        comm = self.comm
        return lambda ptr, stream: comm.allreduce(ptr, ptr, 1, NCCL_FLOAT32, NCCL_MAX, stream)

    def step(self, i: int, stream: int) -> None:
        self.fire[i % len(self.fire)](stream)
        if self.total is not None:
            from emmyrt.dist import NCCL_FLOAT64
            self.comm.allreduce(self.partial_ptr, self.total.ptr, 1, NCCL_FLOAT64, stream=stream)

    def free(self):
        for bs in self.bufsets:
            for b in bs.values():
                b.free()
        self.bufsets = []
        for hb in self.host_bufs:
            hb.free()
        self.host_bufs = []
        if self.total is not None:
            self.total.free()


def _time_region(w: Workload, steps: int, dist: Dist, stream: int = 0) -> tuple[float, dict, str]:
    """Time `steps` steps on one stream (a CUDA graph of the launches when no collective
    is in the step); returns (max-over-ranks ms, clock summary, launch form)."""
    import emmyrt
    from emmyrt import Event, Graph, Stream
    graph = None
    if w.total is None:
        cap = Stream()
        graph = Graph.capture(cap, lambda: [w.fire[i % len(w.fire)](cap.handle) for i in range(steps)])
        graph.upload(stream)
        emmyrt.stream_wait(stream, 120)
    dist.barrier()
    emmyrt.synchronize()
    e0, e1 = Event(), Event()
    with ClockSampler(dist.local) as clocks:
        e0.record(stream)
        if graph is not None:
            graph.launch(stream)
        else:
            for i in range(steps):
                w.step(i, stream)
        e1.record(stream)
        e1.synchronize()
    emmyrt.synchronize()
    ms = e0.elapsed_ms(e1)
    dist.barrier()
    ms = dist.max(ms)
    del graph
    return ms, clocks.summary(), ("one CUDA graph of the timed launches" if w.total is None else
                                  "stream launches, kernel + NCCL all-reduce (f64) per step")


def _e2e(w: Workload, steps: int, dist: Dist) -> dict:
    """Same metric through the C-ABI runtime with host buffers: every step copies its
    inputs up from pinned host memory and its result down."""
    import emmyrt
    from emmyrt import DeviceBuffer, Event, Stream, check, lib
    from emmyrt import HostBuffer
    host_out = {n: HostBuffer(max(16, w.inputs[n].nbytes)) for n in w.out_names}
    pipelined = w.fp8 is None and w.total is None
    extra = None
    if pipelined:
        if w.copies >= 2:
            sets, fires = w.bufsets[:2], w.fire[:2]
        else:
            extra = {}
            for a in w.args:
                h = w.inputs[a["name"]]
                extra[a["name"]] = DeviceBuffer(h.nbytes)
                extra[a["name"]].upload(h)
            sets = [w.bufsets[0], extra]
            fires = [w.fire[0], w.ck.prepare(w.ck.params({n: b.ptr for n, b in extra.items()}))]
        s_in, s_run, s_out = Stream(), Stream(), Stream()
        ev_in, ev_run, ev_out = [Event(), Event()], [Event(), Event()], [Event(), Event()]
        t_stream, end_stream = s_in.handle, s_out.handle

        def e2e_step(i):
            b = i % 2
            bs = sets[b]
            if i >= 2:
                s_in.wait(ev_run[b])          # step i-2's kernel has read this set's inputs
            for n in w.in_names:
                check(lib.emmy_rt_memcpy_htod(bs[n].ptr, w.inputs[n].ctypes.data, w.inputs[n].nbytes,
                                              s_in.handle), "htod")
            ev_in[b].record(s_in.handle)
            s_run.wait(ev_in[b])
            if i >= 2:
                s_run.wait(ev_out[b])         # step i-2's result has left this set's output
            fires[b](s_run.handle)
            ev_run[b].record(s_run.handle)
            s_out.wait(ev_run[b])
            for n in w.out_names:
                check(lib.emmy_rt_memcpy_dtoh(host_out[n].ptr, bs[n].ptr, w.inputs[n].nbytes, s_out.handle),
                      "dtoh")
            ev_out[b].record(s_out.handle)
        d2h = sum(w.inputs[n].nbytes for n in w.out_names)
    else:
        bufs = w.bufsets[0]
        t_stream = end_stream = 0
        res = w.total if w.total is not None else None

        def e2e_step(i):
            for n in w.in_names:
                check(lib.emmy_rt_memcpy_htod(bufs[n].ptr, w.inputs[n].ctypes.data, w.inputs[n].nbytes, 0),
                      "htod")
            if w.fp8 is not None:
                w.fp8.quantize(bufs["a"].ptr, bufs["b"].ptr, 0, amax_b_hook=w._amax_hook())
            w.step(0, 0)
            if res is not None:       # the all-reduced f64 sum is the step's result
                check(lib.emmy_rt_memcpy_dtoh(host_out[w.out_names[0]].ptr, res.ptr, 8, 0), "dtoh")
            else:
                for n in w.out_names:
                    check(lib.emmy_rt_memcpy_dtoh(host_out[n].ptr, bufs[n].ptr, w.inputs[n].nbytes, 0),
                          "dtoh")
        d2h = 8 if res is not None else sum(w.inputs[n].nbytes for n in w.out_names)
    for i in range(2):
        e2e_step(i)
    emmyrt.synchronize()
    dist.barrier()
    emmyrt.synchronize()
    e0, e1 = Event(), Event()
    e0.record(t_stream)
    for i in range(steps):
        e2e_step(i)
    e1.record(end_stream)
    e1.synchronize()
    ms = dist.max(e0.elapsed_ms(e1) / steps)
    if extra:
        for b in extra.values():
            b.free()
    for hb in host_out.values():
        hb.free()
    total = bc.work(w.name, 0, 1) if w.cfg is not None else _units_of(w)
    return {"value": round(to_rate(total, ms / 1e3, w.unit), 3), "unit": w.unit,
            "h2d_bytes_per_step": int(w.in_bytes), "d2h_bytes_per_step": int(d2h),
            "ms_per_step": round(ms, 4), "steps": steps, "pipelined": pipelined,
            "quantise_in_step": w.fp8 is not None}


def _units_of(w: Workload) -> float:
    L = w.ck.launch
    return float(L["flops"]) if "flops" in L else float(w.in_bytes)


def measure(name: str, args, dist: Dist, comm, headline: bool) -> dict:
    import emmyrt
    w = Workload(name, dist, comm)
    try:
        unit = w.unit
        # warm-up (one checked launch first)
        for i in range(max(1, args.warmup)):
            w.step(i, 0)
        emmyrt.stream_wait(0, 300)
        if w.ck.status():
            raise RuntimeError(f"{name}: kernel status {w.ck.status()}")
        # steps: exactly K for the headline; others stretched to >= MIN_REGION_S
        from emmyrt import Event
        e0, e1 = Event(), Event()
        e0.record(0)
        for i in range(3):
            w.step(i, 0)
        e1.record(0)
        e1.synchronize()
        est_s = dist.max(e0.elapsed_ms(e1) / 3) / 1e3
        steps = args.steps if headline else \
            int(min(MAX_LAUNCHES, max(args.steps, math.ceil(MIN_REGION_S / max(est_s, 1e-7)))))
        ms, clocks, form = _time_region(w, steps, dist)
        if w.ck.status():
            raise RuntimeError(f"{name}: kernel status {w.ck.status()} after the timed region")
        ms_step = ms / steps
        total = bc.work(name, 0, 1) if w.cfg is not None else _units_of(w)
        mine = bc.work(name, dist.rank, dist.world) if w.cfg is not None else total
        value = to_rate(total, ms_step / 1e3, unit)
        rec = {"value": round(value, 2), "unit": unit, "ms_per_step": round(ms_step, 5),
               "steps": steps, "region_ms": round(ms, 3),
               "roofline": roofline(name, unit, dist.max(mine) if dist.world > 1 else mine,
                                    ms_step / 1e3, clocks, ms / 1e3, dist.world),
               "clocks": clocks,
               "ms_x_sm_mhz": round(ms_step * clocks["sm_mhz"], 3) if clocks.get("sm_mhz") else None,
               "gpu_launches": steps, "launch": form,
               "kernel": {"entry": w.ck.spec.name, "grid": w.ck.launch["grid"],
                          "block": w.ck.launch["block"], "smem": w.ck.launch.get("smem", 0)},
               "config": config_of(name, dist.world) if w.cfg is not None else {"workload": name}}
        rec["e2e"] = _e2e(w, max(3, min(args.steps, 10)), dist)
        if dist.rank == 0 and dist.world == 1 and not args.no_cpu and w.cfg is not None:
            c = cpu_measure(name, 5, warmup=3)
            c.pop("_dt"), c.pop("_units")
            rec["cpu_baseline"] = c
        else:
            rec["cpu_baseline"] = None
        return rec
    finally:
        w.free()
        del w
        gc.collect()


def _names(args) -> list:
    if args.workload == "all":
        return list(bc.ORDER)
    return [args.workload]


def run_ours(args, dist: Dist) -> int:
    import emmyrt
    emmyrt.init(dist.local)
    comm = None
    if dist.world > 1:
        from emmyrt.dist import NcclComm, share_unique_id
        uid = share_unique_id(dist.rank, dist.broadcast_bytes)
        comm = NcclComm(uid, dist.world, dist.rank)
    names = _names(args)
    results = {}
    try:
        for name in names:
            if name in EXTRA and dist.world > 1:
                continue
            results[name] = measure(name, args, dist, comm, headline=(name == names[0]))
    finally:
        if comm is not None:
            emmyrt.synchronize()
            dist.barrier()
            comm.destroy()
    if dist.rank == 0:
        head = names[0]
        h = results[head]
        line = {"metric": METRIC, "value": h["value"], "unit": h["unit"], "n_gpus": dist.world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": h["ms_per_step"],
                "higher_is_better": True, "scaling": "strong" if dist.world > 1 else "weak",
                "vs_baseline": None,
                "dtype": bc.CONFIGS[head].dtype if head in bc.CONFIGS else "f32",
                "data": "synthetic (seeded, BASELINE.json distributions)",
                "config": h["config"], "e2e": h["e2e"], "roofline": h["roofline"],
                "cpu_baseline": h["cpu_baseline"], "clocks": h["clocks"],
                "gpu_launches": h["gpu_launches"], "launch": h["launch"], "kernel": h["kernel"]}
        if len(results) > 1:
            line["workloads"] = results
        print(json.dumps(line), flush=True)
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "library"], default="ours")
    ap.add_argument("--workload", choices=["all", *bc.ORDER, *EXTRA], default="all")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline samples")
    args = ap.parse_args(argv)
    args.warmup = max(3, args.warmup)
    if args.workload in EXTRA and args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": f"{args.workload} is not a BASELINE "
                          "configuration; no CPU evaluation is defined for it"}))
        return 0
    dist = Dist()
    try:
        if args.impl == "reference":
            return run_reference(args, dist)
        if args.impl == "library":
            return run_library(args, dist)
        return run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    sys.exit(main())
