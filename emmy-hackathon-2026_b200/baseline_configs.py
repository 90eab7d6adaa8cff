"""BASELINE.json's configurations: problem shapes, seeded inputs, shards and work.

Pure Python + numpy (no native library), shared by the benchmark's two arms, the
parity tests and the multi-GPU checks, so every one of them sees the same inputs.

Inputs are seeded synthetic data with BASELINE.json's distributions.  A tensor is
generated in chunks of whole leading-axis rows (about 2^22 elements a chunk); chunk
``c`` of the tensor with seed ``s`` comes from ``numpy.random.default_rng([s, c])``.
Any rows of any tensor can therefore be produced on their own, in parallel, and a
shard is bit-identical to the same rows of the whole tensor whatever the number of
GPUs.

Shards (one process per GPU): GEMM and FP8 by N-panel (each GPU holds all of A and
the columns [n0, n1) of B and C), attention by batch (batch x heads pairs), RMSNorm
and softmax by rows, the global sum by contiguous chunks whose f64 partials one
all-reduce finishes.  ``panel(n, rank, world)`` is the split of n units.
"""

from __future__ import annotations

import math
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np

from hostfmt import NP_DTYPE, f32_to_bf16_bits

CHUNK_ELEMS = 1 << 22


def panel(n: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of rank's share of n units split into contiguous panels."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


# ---------------------------------------------------------------------------
# seeded tensors


@dataclass(frozen=True)
class Tensor:
    """A seeded input: ``scale * N(0,1)`` (``dist='normal'``) or ``U(lo, hi)``."""
    shape: tuple
    seed: int
    dist: str = "normal"
    scale: float = 1.0
    lo: float = 0.0
    hi: float = 1.0

    @property
    def row_elems(self) -> int:
        return math.prod(self.shape[1:])

    @property
    def chunk_rows(self) -> int:
        return max(1, CHUNK_ELEMS // max(1, self.row_elems))

    def _chunk(self, c: int, out: np.ndarray) -> None:
        g = np.random.default_rng([self.seed, c])
        if self.dist == "normal":
            g.standard_normal(out=out, dtype=np.float32)
            if self.scale != 1.0:
                out *= np.float32(self.scale)
        else:
            g.random(out=out, dtype=np.float32)
            out *= np.float32(self.hi - self.lo)
            out += np.float32(self.lo)

    def rows(self, r0: int, r1: int, out: np.ndarray | None = None) -> np.ndarray:
        """Rows [r0, r1) of the leading axis as f32, generated chunk by chunk in parallel."""
        n_rows = r1 - r0
        out = np.empty((n_rows, *self.shape[1:]), np.float32) if out is None else out
        flat = out.reshape(n_rows, -1) if self.row_elems else out.reshape(n_rows, 1)
        cr = self.chunk_rows
        first, last = r0 // cr, (r1 - 1) // cr if n_rows else -1

        def one(c):
            c0, c1 = c * cr, min((c + 1) * cr, self.shape[0])
            lo, hi = max(c0, r0), min(c1, r1)
            if lo == c0 and hi == c1:
                self._chunk(c, flat[lo - r0:hi - r0].reshape(-1))
            else:
                tmp = np.empty((c1 - c0) * max(1, self.row_elems), np.float32)
                self._chunk(c, tmp)
                flat[lo - r0:hi - r0] = tmp.reshape(c1 - c0, -1)[lo - c0:hi - c0]

        workers = min(os.cpu_count() or 1, max(1, last - first + 1), 32)
        if workers == 1:
            for c in range(first, last + 1):
                one(c)
        else:
            with ThreadPoolExecutor(workers) as ex:
                list(ex.map(one, range(first, last + 1)))
        return out

    def full(self) -> np.ndarray:
        return self.rows(0, self.shape[0])


# ---------------------------------------------------------------------------
# configurations


@dataclass(frozen=True)
class Config:
    name: str
    unit: str          # "TFLOP/s" (tensor-core work) or "GB/s" (HBM streams)
    family: str        # gemm | attention | fp8 | row | sum
    dtype: str         # the arithmetic type of the path
    dims: tuple        # the configuration's sizes
    shard_by: str      # what the GPUs split

    @property
    def describe(self) -> str:
        return f"{self.name} {'x'.join(map(str, self.dims))}"


GEMM_SIZES = {"gemm_512": (512, 512, 512), "gemm_2048": (2048, 2048, 2048),
              "gemm_8192": (8192, 8192, 8192), "gemm_4096x14336x4096": (4096, 14336, 4096)}

CONFIGS = {
    **{n: Config(n, "TFLOP/s", "gemm", "bf16", d, "N-panels of B and C, A replicated")
       for n, d in GEMM_SIZES.items()},
    "attention": Config("attention", "TFLOP/s", "attention", "bf16", (8, 32, 4096, 128),
                        "batch (batch x heads pairs)"),
    "fp8_8192": Config("fp8_8192", "TFLOP/s", "fp8", "e4m3", (8192, 8192, 8192),
                       "N-panels of B and C, A replicated; one all-reduce (max) of B's amax"),
    "rmsnorm": Config("rmsnorm", "GB/s", "row", "f32", (4096, 4096), "rows"),
    "softmax": Config("softmax", "GB/s", "row", "f32", (65536, 8192), "rows"),
    "sum": Config("sum", "GB/s", "sum", "f32", (1 << 31,),
                  "contiguous chunks; one NCCL all-reduce of the f64 partials"),
}

# the order the benchmark measures them in (the headline first)
ORDER = ("gemm_8192", "attention", "fp8_8192", "gemm_4096x14336x4096", "gemm_2048", "gemm_512",
         "rmsnorm", "softmax", "sum")


def tensors(name: str) -> dict:
    """The seeded input tensors of a configuration, by role."""
    c = CONFIGS[name]
    if c.family == "gemm":
        m, n, k = c.dims
        return {"A": Tensor((m, k), 0, scale=0.05), "B": Tensor((k, n), 1, scale=0.05)}
    if c.family == "fp8":
        m, n, k = c.dims
        return {"A": Tensor((m, k), 0), "B": Tensor((k, n), 1)}
    if name == "attention":
        return {r: Tensor(c.dims, s) for r, s in (("Q", 0), ("K", 1), ("V", 2))}
    if name == "rmsnorm":
        rows, cols = c.dims
        return {"X": Tensor((rows, cols), 0), "W": Tensor((cols,), 1, dist="uniform", lo=0.5, hi=1.5)}
    if name == "softmax":
        return {"X": Tensor(c.dims, 0, scale=math.sqrt(2.0))}
    if name == "sum":
        return {"X": Tensor(c.dims, 0, dist="uniform", lo=-1.0, hi=1.0)}
    raise KeyError(name)


def shard_dims(name: str, rank: int, world: int) -> dict:
    """The rank's part of the problem: its sizes and where it sits in the whole."""
    c = CONFIGS[name]
    if c.family in ("gemm", "fp8"):
        m, n, k = c.dims
        n0, n1 = panel(n, rank, world)
        return {"m": m, "n": n1 - n0, "k": k, "cols": (n0, n1)}
    if name == "attention":
        b, h, s, d = c.dims
        b0, b1 = panel(b, rank, world)
        return {"b": b1 - b0, "h": h, "s": s, "d": d, "rows": (b0, b1)}
    if c.family == "row":
        rows, cols = c.dims
        r0, r1 = panel(rows, rank, world)
        return {"rows": (r0, r1), "cols": cols}
    if name == "sum":
        r0, r1 = panel(c.dims[0], rank, world)
        return {"rows": (r0, r1)}
    raise KeyError(name)


def work(name: str, rank: int = 0, world: int = 1) -> float:
    """Algorithmic work of the rank's shard (the whole problem at world 1): flops for
    tensor-core configurations; bytes read once plus bytes written once for streams."""
    c = CONFIGS[name]
    d = shard_dims(name, rank, world)
    if c.family in ("gemm", "fp8"):
        return 2.0 * d["m"] * d["n"] * d["k"]
    if name == "attention":
        return 4.0 * d["b"] * d["h"] * d["s"] * d["s"] * d["d"]
    if name == "rmsnorm":
        r = d["rows"][1] - d["rows"][0]
        return float(2 * r * d["cols"] * 4 + d["cols"] * 4)
    if name == "softmax":
        r = d["rows"][1] - d["rows"][0]
        return float(2 * r * d["cols"] * 4)
    if name == "sum":
        return float((d["rows"][1] - d["rows"][0]) * 4)
    raise KeyError(name)


def shard_problem(name: str, rank: int = 0, world: int = 1) -> tuple[dict, dict]:
    """The IR + meta of the rank's shard, synthesised from the configuration's family
    (fp8 has no IR family: its meta describes the pipeline's buffers only)."""
    from compiler import synth
    c = CONFIGS[name]
    d = shard_dims(name, rank, world)
    tag = f"{name}_r{rank}of{world}" if world > 1 else name
    if c.family == "gemm":
        return synth.gemm_family(d["m"], d["n"], d["k"], tag)
    if name == "attention":
        return synth.attention_family(d["b"], d["h"], d["s"], d["d"], tag)
    if name == "rmsnorm":
        return synth.rmsnorm_family(d["rows"][1] - d["rows"][0], d["cols"], tag)
    if name == "softmax":
        return synth.softmax_family(d["rows"][1] - d["rows"][0], d["cols"], tag)
    if name == "sum":
        return synth.sum_family(d["rows"][1] - d["rows"][0], tag)
    if c.family == "fp8":
        meta = {"id": tag, "kernels": [{"entry": "k_gemm_e4m3", "args": [
            {"name": "a", "dtype": "f32", "shape": [d["m"], d["k"]]},
            {"name": "b", "dtype": "f32", "shape": [d["k"], d["n"]]},
            {"name": "c", "dtype": "bf16", "shape": [d["m"], d["n"]], "output": True}]}]}
        return {}, meta
    raise KeyError(name)


# IR argument name -> tensor role, per family
_ROLES = {"gemm": {"x0": "A", "x1": "B"}, "fp8": {"a": "A", "b": "B"},
          "attention": {"x0": "Q", "x1": "K", "x2": "V"},
          "rmsnorm": {"x0": "X", "x1": "W"}, "softmax": {"x": "X"}, "sum": {"x": "X"}}


def _roles(name: str) -> dict:
    c = CONFIGS[name]
    return _ROLES[c.family if c.family in ("gemm", "fp8") else name]


def shard_inputs(name: str, meta: dict, rank: int = 0, world: int = 1, alloc=None) -> dict:
    """Host arrays for every argument of the shard's kernel (meta.json args): the seeded
    inputs cut to the shard, constants from their ``data``, zeroed outputs.
    ``alloc(nbytes) -> writable uint8 array`` places them (e.g. in pinned memory)."""
    alloc = alloc or (lambda nb: np.empty(nb, np.uint8))
    c = CONFIGS[name]
    d = shard_dims(name, rank, world)
    ts = tensors(name)
    roles = _roles(name)
    out = {}
    for a in meta["kernels"][0]["args"]:
        shape = tuple(a["shape"]) or (1,)
        npt = NP_DTYPE[a["dtype"]]
        buf = alloc(int(np.prod(shape)) * np.dtype(npt).itemsize).view(npt).reshape(shape)
        if a.get("output"):
            buf[...] = 0
        elif "data" in a:
            buf[...] = np.asarray(a["data"], dtype=npt).reshape(shape)
        else:
            t = ts[roles[a["name"]]]
            if c.family in ("gemm", "fp8") and roles[a["name"]] == "B":
                n0, n1 = d["cols"]
                vals = t.full()[:, n0:n1] if (n0, n1) != (0, t.shape[1]) else t.full()
            elif c.family in ("gemm", "fp8"):
                vals = t.full()
            elif name == "rmsnorm" and roles[a["name"]] == "W":
                vals = t.full()
            else:
                r0, r1 = d["rows"]
                if a["dtype"] == "f32":
                    t.rows(r0, r1, out=buf)
                    out[a["name"]] = buf
                    continue
                vals = t.rows(r0, r1)
            if a["dtype"] == "bf16":
                f32_to_bf16_bits(vals, out=buf)
            else:
                buf[...] = vals
        out[a["name"]] = buf
    return out


def output_name(meta: dict) -> str:
    return next(a["name"] for a in meta["kernels"][0]["args"] if a.get("output"))


# ---------------------------------------------------------------------------
# the bounded CPU sample (the same in the CPU baseline and the reference arm)


def cpu_sample_inputs(name: str) -> tuple[dict, float, str]:
    """(f32 / bf16-valued inputs of the sample, its algorithmic work, description).

    GEMM / FP8: the first rows of A against the whole B (about 2^38 flops, a quarter
    of the 8192^3 problem); attention: all queries of the 32 batch x head pairs of
    batch 0 (an eighth); RMSNorm: the whole problem; softmax: the first 16384 rows (a
    quarter); sum: the first 2^29 elements (a quarter)."""
    c = CONFIGS[name]
    ts = tensors(name)
    if c.family in ("gemm", "fp8"):
        m, n, k = c.dims
        rows = min(m, max(8, (1 << 38) // (2 * n * k)))
        A, B = ts["A"].rows(0, rows), ts["B"].full()
        return {"A": A, "B": B}, 2.0 * rows * n * k, f"first {rows} of {m} rows of A against all of B"
    if name == "attention":
        b, h, s, d = c.dims
        q, k_, v = (ts[r].rows(0, 1) for r in ("Q", "K", "V"))
        return {"Q": q, "K": k_, "V": v}, 4.0 * h * s * s * d, \
            f"batch 0 ({h} of {b * h} batch x head pairs), all {s} queries and keys"
    if name == "rmsnorm":
        X, W = ts["X"].full(), ts["W"].full()
        return {"X": X, "W": W}, float(2 * X.nbytes + W.nbytes), "the whole 4096 x 4096 problem"
    if name == "softmax":
        X = ts["X"].rows(0, 16384)
        return {"X": X}, float(2 * X.nbytes), f"first 16384 of {c.dims[0]} rows"
    if name == "sum":
        X = ts["X"].rows(0, 1 << 29)
        return {"X": X}, float(X.nbytes), "first 2^29 of the 2^31 elements"
    raise KeyError(name)
