"""BASELINE-sized problems synthesised from the reference's IR families.

Emmy cannot run here, so no IR exists at the benchmark sizes.  A benchmark problem
is made from the fixture of its family by rescaling it: every extent in the graph,
in meta.json and in the body's ``Dim(...)`` values is mapped through ``dims``
(old extent -> new extent), buffer dtypes through ``dtypes``, constants are
replaced (``mean_count`` follows the new row length), and the kernel keeps its
statement structure.  The templates read sizes from the buffer shapes and the
family from the statements, so the rescaled IR compiles exactly as an emmy dump of
that size would.

Families (fixture -> BASELINE config):

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

ROOT = Path(__file__).resolve().parents[2]
GOLDEN = ROOT / "tests" / "golden" / "problems"

_DT_NP = {"f32": "float32", "f16": "float16", "bf16": "uint16", "f64": "float64"}


def _rewrite_body(text: str, dims: dict, dtypes: dict) -> str:
    def dim(m):
        v = int(m.group(1))
        return f"Dim({dims.get(v, v)})"
    text = re.sub(r"Dim\((\d+)\)", dim, text)
    for old, new in dtypes.items():
        text = text.replace(f"DataType(name='{old}', np=dtype('{_DT_NP[old]}')",
                            f"DataType(name='{new}', np=dtype('{_DT_NP[new]}')")
        text = text.replace(f"ab_dtype='{old}'", f"ab_dtype='{new}'")
        text = text.replace(f"dtype='{old}'", f"dtype='{new}'")
    return text


def rescale(src_dir: Path, dims: dict, dtypes: dict | None = None, constants: dict | None = None,
            shapes: dict | None = None, problem_id: str | None = None,
            const_dtypes: dict | None = None) -> tuple[dict, dict]:
    """Rescale one fixture problem; returns (ir_json_by_entry, meta).  ``const_dtypes``
    gives named constant buffers their own dtype (e.g. an exact f32 softmax scale in a
    bf16 problem)."""
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
                o["shape"] = shapes.get(o["name"], [dims.get(int(d), int(d)) for d in o["shape"]])
                o["dtype"] = const_dtypes.get(o["name"], dtypes.get(o["dtype"], o["dtype"]))
            if node["op"] == "ConstantOp":
                nid = node["op_fields"]["name"]
                if nid in constants:
                    node["op_fields"]["value"] = constants[nid]
            if node["op"] == "KernelOp":
                node["op_fields"]["body"] = [_rewrite_body(s, dims, dtypes)
                                             for s in node["op_fields"]["body"]]
        irs[k["entry"]] = ir
        for a in k["args"]:
            a["shape"] = shapes.get(a["name"], [dims.get(int(d), int(d)) for d in a["shape"]])
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


def baseline_problem(name: str, golden: Path = GOLDEN) -> tuple[dict, dict]:
    if name == "rmsnorm":
        return rescale(golden / "x_l_rmsnorm_w", {64: 4096, 512: 4096},
                       constants={"mean_count": 4096.0}, problem_id="rmsnorm_4096x4096")
    if name == "softmax":
        return rescale(golden / "f02_row_softmax", {64: 65536, 256: 8192},
                       problem_id="softmax_65536x8192")
    if name == "sum":
        return rescale(golden / "x_r_unpinned_sum", {64: 1 << 21, 65536: 1 << 31},
                       problem_id="sum_2p31")
    if name in GEMM_SIZES:
        m, n, k = GEMM_SIZES[name]
        # x_h_mm_1024: x0 is A [M, K], x1 is B [K, N], matmul is C [M, N]
        return rescale(golden / "x_h_mm_1024", {}, dtypes={"f16": "bf16"},
                       shapes={"x0": [m, k], "x1": [k, n], "matmul": [m, n]}, problem_id=name)
    if name == "gemm_f32_4096":
        # not a BASELINE config: the reference's own f32 matmul (m01, emmy's SIMT FMA
        # schedule) at 4096^3, for the 3xTF32 template's measurements
        return rescale(golden / "m01_matmul_512", {512: 4096}, problem_id=name)
    if name == "attention":
        shp = [8, 32, 4096, 128]
        return rescale(golden / "x_h_sdpa", {}, dtypes={"f16": "bf16"},
                       shapes={"x0": shp, "x1": shp, "x2": shp, "scaled_dot_product_attention": shp},
                       constants={"scaled_dot_product_attention_scale": 128 ** -0.5},
                       const_dtypes={"scaled_dot_product_attention_scale": "f32"},
                       problem_id="attention_b8h32s4096d128")
    raise KeyError(name)


BASELINE_NAMES = ("rmsnorm", "softmax", "sum", *GEMM_SIZES, "attention")


def baseline_dir(name: str, root: Path | None = None) -> Path:
    irs, meta = baseline_problem(name)
    root = root or Path(tempfile.gettempdir()) / "emmy_baseline"
    return write_problem(irs, meta, root / name)


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
