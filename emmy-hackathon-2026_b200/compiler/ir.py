"""Emmy Kernel IR: typed statement tree and a ``Graph.from_dict`` loader.

The reference deserialises IR json through the third-party ``emmy-ml==0.3.11``
package (``compiler/loader.py:14,78`` in the reference: ``Graph.from_dict``).
That package is not installable here, so this module provides a compatible
loader of its own:

* a graph json holds ``inputs``, ``outputs`` and ``nodes``; every node has an
  ``op`` name (``InputOp``, ``ConstantOp``, ``KernelOp``), ``op_fields``,
  ``inputs`` and ``outputs`` (``name``, ``shape``, ``dtype``);
* a ``KernelOp`` body is a list of Python-repr strings over the IR constructors
  (``Tile(axes=(Axis(...),), body=(...))``).  They are parsed with ``ast`` -- never
  ``eval`` -- into frozen dataclasses with the constructor's own class name and
  field names, because every consumer (the reference's handlers and ours)
  dispatches on ``type(stmt).__name__`` and reads plain attributes.

``ElementwiseImpl`` carries the identity a reduction accumulator starts from
(add 0, max -1e30, min +1e30, mul 1); the ``-1e30`` max identity is the one the
reference's generated CUDA uses (``problems/f02_row_softmax/*.ref.cu:9``).

When the real ``emmy`` package is importable it is preferred, so a machine with
emmy installed deserialises exactly as the reference does.
"""

from __future__ import annotations

import ast
import dataclasses
from dataclasses import dataclass, field
from typing import Any

__all__ = ["Graph", "Node", "TensorInfo", "parse_stmt", "IR_CLASSES", "DataType",
           "ElementwiseImpl", "Dim", "NpDType"]


# --------------------------------------------------------------------------
# leaf value types


@dataclass(frozen=True)
class NpDType:
    """Stand-in for ``numpy.dtype('float32')`` inside ``DataType(np=...)``."""
    name: str


@dataclass(frozen=True)
class Dim:
    """A static extent.  ``Dim(64).value == 64``."""
    value: int

    def __int__(self) -> int:
        return int(self.value)


_IDENTITY = {"add": 0.0, "maximum": -1e30, "minimum": 1e30, "multiply": 1.0,
             "bitwise_or": 0, "bitwise_and": -1, "bitwise_xor": 0}


@dataclass(frozen=True)
class ElementwiseImpl:
    """An elementwise operation by name (``ElementwiseImpl('add')``)."""
    name: str

    @property
    def identity(self):
        try:
            return _IDENTITY[self.name]
        except KeyError:
            raise NotImplementedError(f"no reduction identity for {self.name!r}") from None


@dataclass(frozen=True)
class DataType:
    """``DataType(name='f32', np=dtype('float32'), nbytes=4)``."""
    name: str
    np: Any = None
    nbytes: int = 0


# --------------------------------------------------------------------------
# statement / expression constructors.  Field lists follow the IR vocabulary;
# every field defaults to None so an older or newer dump with a missing
# keyword still loads.

_FIELDS = {
    # expressions
    "Var": ("name",),
    "Literal": ("value", "dtype"),
    "BinaryExpr": ("op", "left", "right"),
    "TernaryExpr": ("cond", "if_true", "if_false"),
    "Builtin": ("name",),
    "FuncCallExpr": ("name", "args"),
    "CastExpr": ("dtype", "expr"),
    "FlatIndex": ("buffer", "index"),
    # launch structure
    "Axis": ("name", "extent", "window"),
    "Window": ("base", "bound", "parent", "partition"),
    "Tile": ("axes", "body", "block_threads", "aux_threads", "raster_axes",
             "raster_group", "raster_orient"),
    "Loop": ("axis", "body", "unroll", "seed"),
    "StridedLoop": ("axis", "start", "step", "body", "unroll", "end", "seed"),
    "Cond": ("cond", "body", "else_body"),
    # scalar compute
    "Load": ("names", "input", "index", "dtype"),
    "Write": ("output", "index", "values", "value_dtype", "atomic", "swizzle"),
    "Assign": ("name", "op", "args", "dtype"),
    "Let": ("name", "value", "dtype"),
    "Accum": ("name", "value", "op", "dtype", "axes", "base"),
    "Init": ("name", "identity", "dtype"),
    "Select": ("name", "branches"),
    "SelectBranch": ("select", "value"),
    "Lambda": ("params", "body", "results"),
    "Pre": ("name", "carrier", "index"),
    "Carry": ("name", "value", "index", "seed", "dtype"),
    "ZeroPrologue": ("dst", "words"),
    # shared memory, barriers, copies
    "Smem": ("name", "extents", "dtype", "align"),
    "Sync": ("barrier_id", "count", "warp"),
    "CpAsyncCopy": ("smem", "smem_index", "src", "src_index", "nbytes", "swizzle",
                    "lane_index", "lane_rows"),
    "CpAsyncCommit": (),
    "CpAsyncWait": ("group",),
    "TmaDescriptor": ("name", "src_buf", "src_shape", "box_extents", "swizzle", "dtype"),
    "TmaLoad": ("smem", "smem_index", "desc", "coords", "mbar", "mbar_slot"),
    "MbarrierInit": ("mbar", "count", "slot"),
    "MbarrierArriveExpectTx": ("mbar", "bytes_", "slot"),
    "MbarrierArrive": ("mbar", "slot"),
    "MbarrierWait": ("mbar", "phase", "slot"),
    "SetMaxNReg": ("count", "direction"),
    # cross-thread combine
    "WarpShuffle": ("state", "state_b", "combine_states", "length", "dtype"),
    "TreeHalve": ("bufs", "state", "state_b", "combine_states", "length", "tid_var",
                  "dtype", "barrier_id", "barrier_count", "inner"),
    # register-fragment tensor core
    "RegFragment": ("name", "role", "shape", "dtype", "count", "nregs"),
    "LdmatrixLoad": ("frag", "src_buffer", "src_index", "role", "ldm", "swizzle", "staged",
                     "gmem_guard", "k_zero", "b_trans", "pair_frag", "byte_slab",
                     "scale_buffer", "scale_index", "scale_ldm", "fragment_layout",
                     "fragment_index"),
    "BlockScaleLoad": ("frag", "src_buffer", "src_index", "role", "ldm"),
    "MmaSyncPtx": ("c_frag", "a_frag", "b_frag", "shape", "ab_dtype", "c_dtype",
                   "b_row_major", "sfa_frag", "sfb_frag"),
    "FragmentPromote": ("dst", "src"),
    "FragmentApply": ("out", "op", "args", "kinds", "in_place", "layout", "post",
                      "row_base", "col_base"),
    "FragmentRowReduce": ("top", "bot", "frags", "op", "layout", "dtype"),
    "FragmentRepack": ("frag", "srcs", "ab_dtype", "fragment_layout", "part"),
    "RegStore": ("dst_buffer", "dst_index", "frag", "shape", "ldm", "epilogue", "extra_frags",
                 "m_guard", "n_guard", "atomic", "fragment_layout", "volta_interleaved",
                 "fragment_index", "swizzle", "row_dim", "col_dim"),
    "FragLayout": ("n_elems", "elem_row", "reduce_xors", "lane_decl", "lane_names",
                   "row_off", "col_off"),
    # warp-group tensor core (listed in the vocabulary; never emitted by emmy 0.3.11)
    "WgmmaDescriptor": ("name", "smem", "smem_index", "swizzle", "lbo_bytes", "sbo_bytes"),
    "WgmmaMma": ("c_frags", "b_desc", "shape", "ab_dtype", "a_desc", "a_frag", "scale_d",
                 "trans_a", "trans_b"),
    "WgmmaFence": (),
    "WgmmaCommit": (),
    "WgmmaWait": ("group",),
}


def _make_class(name: str, fields: tuple[str, ...]) -> type:
    cls = dataclasses.make_dataclass(
        name, [(f, Any, field(default=None)) for f in fields], frozen=True)
    cls.__module__ = __name__
    return cls


IR_CLASSES: dict[str, type] = {n: _make_class(n, f) for n, f in _FIELDS.items()}
globals().update(IR_CLASSES)
__all__ += list(IR_CLASSES)


# --------------------------------------------------------------------------
# repr-string parser


class IRParseError(ValueError):
    pass


def _convert(node: ast.AST):
    if isinstance(node, ast.Constant):
        return node.value
    if isinstance(node, ast.Tuple):
        return tuple(_convert(e) for e in node.elts)
    if isinstance(node, ast.List):
        return tuple(_convert(e) for e in node.elts)
    if isinstance(node, ast.Dict):
        return {_convert(k): _convert(v) for k, v in zip(node.keys, node.values)}
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, ast.USub):
        return -_convert(node.operand)
    if isinstance(node, ast.Name) and node.id in ("inf", "nan"):
        return float(node.id)
    if isinstance(node, ast.Call) and isinstance(node.func, ast.Name):
        name = node.func.id
        args = [_convert(a) for a in node.args]
        kwargs = {k.arg: _convert(k.value) for k in node.keywords}
        if name == "dtype":
            return NpDType(*args)
        if name == "Dim":
            return Dim(int(args[0]))
        if name == "ElementwiseImpl":
            return ElementwiseImpl(*args, **kwargs)
        if name == "DataType":
            return DataType(*args, **kwargs)
        cls = IR_CLASSES.get(name)
        if cls is None:
            # An unknown constructor still loads; the back end rejects it with
            # NotImplementedError when (and only when) it has to lower it.
            cls = _make_class(name, tuple(kwargs))
            IR_CLASSES[name] = cls
        try:
            return cls(*args, **kwargs)
        except TypeError as exc:
            raise IRParseError(f"{name}: {exc}") from None
    raise IRParseError(f"unsupported IR syntax: {ast.dump(node)[:120]}")


def parse_stmt(text: str):
    """Parse one body statement repr into its dataclass tree."""
    try:
        tree = ast.parse(text.strip(), mode="eval")
    except SyntaxError as exc:
        raise IRParseError(f"body statement is not a constructor expression: {exc}") from None
    return _convert(tree.body)


# --------------------------------------------------------------------------
# graph


@dataclass(frozen=True)
class TensorInfo:
    name: str
    shape: tuple[Dim, ...]
    dtype: DataType


@dataclass(frozen=True)
class _OpRecord:
    """The op of one node: its type name plus its ``op_fields`` as attributes."""
    kind: str
    fields: dict

    def __getattr__(self, item):
        try:
            return self.__dict__["fields"][item]
        except KeyError:
            raise AttributeError(item) from None


def _op_class(kind: str) -> type:
    return type(kind, (_OpRecord,), {})


_OP_CLASSES: dict[str, type] = {}


@dataclass(frozen=True)
class Node:
    id: str
    op: Any
    inputs: tuple[str, ...]
    outputs: tuple[TensorInfo, ...]


_DTYPE_BYTES = {"f32": 4, "f16": 2, "bf16": 2, "f64": 8, "i32": 4, "i64": 8, "u8": 1,
                "i8": 1, "bool": 1, "u16": 2, "e4m3": 1, "e5m2": 1}


class Graph:
    """Deserialised graph: ``nodes`` maps node id -> :class:`Node`."""

    def __init__(self, inputs, outputs, nodes):
        self.inputs = tuple(inputs)
        self.outputs = tuple(outputs)
        self.nodes = nodes

    @classmethod
    def from_dict(cls, data: dict) -> "Graph":
        nodes = {}
        for nid, rec in data["nodes"].items():
            kind = rec["op"]
            fields = dict(rec.get("op_fields", {}))
            if kind == "KernelOp":
                fields["body"] = tuple(parse_stmt(s) for s in fields.get("body", ()))
            opcls = _OP_CLASSES.setdefault(kind, _op_class(kind))
            outs = tuple(
                TensorInfo(o["name"], tuple(Dim(int(d)) for d in o.get("shape") or ()),
                           DataType(o["dtype"], None, _DTYPE_BYTES.get(o["dtype"], 0)))
                for o in rec.get("outputs", ()))
            nodes[nid] = Node(nid, opcls(kind, fields), tuple(rec.get("inputs", ())), outs)
        return cls(data.get("inputs", ()), data.get("outputs", ()), nodes)


def load_graph_class():
    """``Graph`` from the real emmy package when importable, else this module's."""
    try:  # pragma: no cover - emmy is not installable in this image
        from emmy.compiler.graph import Graph as EmmyGraph  # type: ignore
        return EmmyGraph
    except Exception:
        return Graph
