"""BASELINE-sized problems synthesised from the reference's IR families.

Emmy cannot run here, so no IR exists at the benchmark sizes.  A benchmark problem
is made from a small problem of its family (the emmy dumps under ``families/``, one
folder per family: the kernels' IR json and ``meta.json``) by rescaling it:

* ``axes`` names the loop axes that change, as ``(axis name, old extent) -> new
  extent``; only ``Axis(name=..., extent=Dim(old))`` records of that name and extent
  in the kernel body are rewritten (a constant that merely equals an extent is left
  alone, and a windowed axis keeps its window size while its parent grows);
* ``shapes`` gives the new shape of each named tensor (graph node outputs and
  meta.json args), ``dtypes`` retypes buffers, ``constants`` replaces ConstantOp
  values (``mean_count`` follows the new row length);
* the kernel keeps its statement structure.  The templates read sizes from the
  buffer shapes and the family from the statements, so the rescaled IR compiles
  exactly as an emmy dump of that size would.

Families (folder -> BASELINE config):

* ``x_l_rmsnorm_w``   -> RMSNorm fp32 4096 x 4096, eps 1e-6
* ``f02_row_softmax`` -> row softmax fp32 65536 x 8192
* ``x_r_unpinned_sum`` -> global fp32 sum over 2^31 elements
* ``x_h_mm_1024``     -> bf16 GEMM, M=N=K in {512, 2048, 8192} and 4096 x 14336 x 4096
* ``x_h_sdpa``        -> bf16 attention B8 H32 S4096 D128
"""

from __future__ import annotations

import copy
import json
import os
import re
import tempfile
from pathlib import Path

from .loader import load

FAMILIES = Path(__file__).resolve().parent / "families"

_DT_NP = {"f32": "float32", "f16": "float16", "bf16": "uint16", "f64": "float64"}
# shared-memory buffers (Smem) carry the C type name of their elements
_DT_C = {"f32": "float", "f16": "__half", "bf16": "__nv_bfloat16", "f64": "double"}


def _rewrite_body(text: str, axes: dict, dtypes: dict) -> str:
    def axis(m):
        name, old = m.group(1), int(m.group(2))
        return f"Axis(name='{name}', extent=Dim({axes.get((name, old), old)})"
    text = re.sub(r"Axis\(name='(\w+)', extent=Dim\((\d+)\)", axis, text)
    for old, new in dtypes.items():
        text = text.replace(f"DataType(name='{old}', np=dtype('{_DT_NP[old]}')",
                            f"DataType(name='{new}', np=dtype('{_DT_NP[new]}')")
        text = text.replace(f"ab_dtype='{old}'", f"ab_dtype='{new}'")
        text = text.replace(f"dtype='{old}'", f"dtype='{new}'")
        text = text.replace(f"dtype='{_DT_C[old]}'", f"dtype='{_DT_C[new]}'")
    return text


def rescale(src_dir: Path, axes: dict | None = None, dtypes: dict | None = None,
            constants: dict | None = None, shapes: dict | None = None,
            problem_id: str | None = None, const_dtypes: dict | None = None) -> tuple[dict, dict]:
    """Rescale one family problem; returns (ir_json_by_entry, meta).  Every tensor whose
    shape changes must be named in ``shapes``; ``const_dtypes`` gives named constant
    buffers their own dtype (e.g. an exact f32 softmax scale in a bf16 problem)."""
    axes = axes or {}
    dtypes = dtypes or {}
    constants = constants or {}
    shapes = shapes or {}
    const_dtypes = const_dtypes or {}
    meta = json.loads((src_dir / "meta.json").read_text())
    irs = {}
    for k in meta["kernels"]:
        ir = json.loads((src_dir / f"{k['entry']}.ir.json").read_text())
        for node in ir["nodes"].values():
            for o in node["outputs"]:
                o["shape"] = list(shapes.get(o["name"], o["shape"]))
                o["dtype"] = const_dtypes.get(o["name"], dtypes.get(o["dtype"], o["dtype"]))
            if node["op"] == "ConstantOp":
                nid = node["op_fields"]["name"]
                if nid in constants:
                    node["op_fields"]["value"] = constants[nid]
            if node["op"] == "KernelOp":
                node["op_fields"]["body"] = [_rewrite_body(s, axes, dtypes)
                                             for s in node["op_fields"]["body"]]
        irs[k["entry"]] = ir
        for a in k["args"]:
            a["shape"] = list(shapes.get(a["name"], a["shape"]))
            a["dtype"] = const_dtypes.get(a["name"], dtypes.get(a["dtype"], a["dtype"]))
            if a["name"] in constants:
                a["data"] = [constants[a["name"]]]
    meta = copy.deepcopy(meta)
    if problem_id:
        meta["id"] = problem_id
    meta.pop("code", None)
    return irs, meta


def _write_atomic(path: Path, text: str) -> None:
    """Write to a file of this process's own, then rename it over ``path``: processes
    that write the same problem at once (one per GPU under torchrun) never read a
    half-written file."""
    tmp = path.with_name(f".{path.name}.{os.getpid()}.tmp")
    tmp.write_text(text)
    os.replace(tmp, path)


def write_problem(irs: dict, meta: dict, out_dir: Path) -> Path:
    out_dir.mkdir(parents=True, exist_ok=True)
    for entry, ir in irs.items():
        _write_atomic(out_dir / f"{entry}.ir.json", json.dumps(ir))
    _write_atomic(out_dir / "meta.json", json.dumps(meta, indent=1))
    return out_dir


# BASELINE configurations -------------------------------------------------------

GEMM_SIZES = {"gemm_512": (512, 512, 512), "gemm_2048": (2048, 2048, 2048),
              "gemm_8192": (8192, 8192, 8192), "gemm_4096x14336x4096": (4096, 14336, 4096)}


def rmsnorm_family(rows: int, cols: int, problem_id: str) -> tuple[dict, dict]:
    """x_l_rmsnorm_w: y = x * rsqrt(mean(x^2) + eps) * w over rows of x [rows, cols];
    axis a0 walks the rows, a1 (the mean's stream) and a2 (the scaling pass) the columns."""
    return rescale(FAMILIES / "x_l_rmsnorm_w",
                   axes={("a0", 64): rows, ("a1", 512): cols, ("a2", 512): cols},
                   shapes={"x0": [rows, cols], "x1": [cols], "mul_1": [rows, cols]},
                   constants={"mean_count": float(cols)}, problem_id=problem_id)


def sum_family(n: int, problem_id: str) -> tuple[dict, dict]:
    """x_r_unpinned_sum: the global sum of x [n], split by emmy over ``_ksplit`` windows
    of 1024 elements of the axis a0 (so n / 1024 of them)."""
    if n % 1024:
        raise ValueError("the sum family splits its axis into windows of 1024")
    return rescale(FAMILIES / "x_r_unpinned_sum",
                   axes={("_ksplit", 64): n // 1024, ("a0", 65536): n},
                   shapes={"x": [n]}, problem_id=problem_id)


def softmax_family(rows: int, cols: int, problem_id: str) -> tuple[dict, dict]:
    """f02_row_softmax: softmax over the rows of x [rows, cols] (a0 rows; a1 the max /
    sum stream and a3 the normalising pass over the columns)."""
    return rescale(FAMILIES / "f02_row_softmax",
                   axes={("a0", 64): rows, ("a1", 256): cols, ("a3", 256): cols},
                   shapes={"x": [rows, cols], "softmax": [rows, cols]}, problem_id=problem_id)


def gemm_family(m: int, n: int, k: int, problem_id: str) -> tuple[dict, dict]:
    """x_h_mm_1024 retyped to bf16: C [m, n] = A [m, k] . B [k, n] (x0 is A, x1 is B).
    The tensor-core templates take the sizes from the buffer shapes."""
    return rescale(FAMILIES / "x_h_mm_1024", dtypes={"f16": "bf16"},
                   shapes={"x0": [m, k], "x1": [k, n], "matmul": [m, n]}, problem_id=problem_id)


def attention_family(b: int, h: int, s: int, d: int, problem_id: str) -> tuple[dict, dict]:
    """x_h_sdpa retyped to bf16: O = softmax(Q K^T / sqrt(d)) V over [b, h, s, d], with
    the softmax scale as an exact f32 constant."""
    shp = [b, h, s, d]
    return rescale(FAMILIES / "x_h_sdpa", dtypes={"f16": "bf16"},
                   shapes={"x0": shp, "x1": shp, "x2": shp, "scaled_dot_product_attention": shp},
                   constants={"scaled_dot_product_attention_scale": d ** -0.5},
                   const_dtypes={"scaled_dot_product_attention_scale": "f32"},
                   problem_id=problem_id)


def baseline_problem(name: str) -> tuple[dict, dict]:
    if name == "rmsnorm":
        return rmsnorm_family(4096, 4096, "rmsnorm_4096x4096")
    if name == "softmax":
        return softmax_family(65536, 8192, "softmax_65536x8192")
    if name == "sum":
        return sum_family(1 << 31, "sum_2p31")
    if name in GEMM_SIZES:
        return gemm_family(*GEMM_SIZES[name], problem_id=name)
    if name == "gemm_f32_4096":
        # not a BASELINE config: the reference's own f32 matmul (m01, emmy's SIMT FMA
        # schedule) at 4096^3, for the 3xTF32 template's measurements
        return rescale(FAMILIES / "m01_matmul_512",
                       axes={("a0", 512): 4096, ("a1", 512): 4096, ("_ks", 512): 4096},
                       shapes={"x0": [4096, 4096], "x1": [4096, 4096], "matmul": [4096, 4096]},
                       problem_id=name)
    if name == "attention":
        return attention_family(8, 32, 4096, 128, "attention_b8h32s4096d128")
    raise KeyError(name)


BASELINE_NAMES = ("rmsnorm", "softmax", "sum", *GEMM_SIZES, "attention")


def baseline_dir(name: str, root: Path | None = None) -> Path:
    irs, meta = baseline_problem(name)
    root = root or Path(tempfile.gettempdir()) / "emmy_baseline"
    return write_problem(irs, meta, root / name)


def problem_dir(irs: dict, meta: dict, root: Path | None = None) -> Path:
    """Write a synthesised problem under the temporary problem root, named by its id."""
    root = root or Path(tempfile.gettempdir()) / "emmy_baseline"
    return write_problem(irs, meta, root / meta["id"])


def baseline_specs(names=BASELINE_NAMES) -> dict:
    """KernelSpecs of the BASELINE configurations whose family compiles."""
    out = {}
    for n in names:
        d = baseline_dir(n)
        meta = json.loads((d / "meta.json").read_text())
        for k in meta["kernels"]:
            try:
                spec = load(d / f"{k['entry']}.ir.json")
                from . import compile_kernel
                compile_kernel(spec)
            except NotImplementedError:
                continue
            out[f"{n}:{k['entry']}"] = spec
    return out
