"""Load one Kernel IR json plus its ``meta.json`` launch contract into a KernelSpec.

Mirrors the reference's ``compiler/loader.py``:

* ``Param`` / ``KernelSpec`` carry the same fields (``loader.py:17-39``);
* the KernelOp is found by file stem when a graph holds several (``:42-52``);
* ``ConstantOp`` values are collected so their 1-element buffers can be folded
  to immediates (``:65-73``);
* ``meta.json``'s ``arg_order`` is the parameter order, and its grid/block/smem
  the prescribed launch (``:83-96``); without a meta.json the node's inputs
  followed by its outputs are used (``:97-103``).

Added for this back end: ``buffers`` (shape/dtype of every tensor the graph
names) and ``args_meta`` (meta.json's arg records, whose ``seed``/``data``
fields the runner uses to build inputs the way the reference's runner does).
"""

from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from pathlib import Path

from .ir import load_graph_class


@dataclass(frozen=True)
class Param:
    name: str
    dtype: str
    shape: tuple[int, ...]
    scalar: bool = False    # passed by value instead of as a buffer pointer


@dataclass(frozen=True)
class KernelSpec:
    name: str
    body: tuple                 # top-level IR statements
    params: tuple[Param, ...]   # in launch order (meta.json arg_order)
    grid: tuple[int, int, int] | None
    block: tuple[int, int, int] | None
    constants: dict             # ConstantOp buffer -> its value (also passed at launch)
    smem_bytes: int = 0         # dynamic shared memory of emmy's own launch (meta.json)
    buffers: dict = field(default_factory=dict)    # every graph tensor -> Param
    args_meta: tuple = ()       # meta.json arg records (seed / data / output)
    zero_outputs: tuple = ()    # buffers the reference runner re-zeroes before each launch

    @property
    def threads_launched(self) -> int | None:
        if self.grid is None or self.block is None:
            return None
        return math.prod(self.grid) * math.prod(self.block)

    def param(self, name: str) -> Param:
        for p in self.params:
            if p.name == name:
                return p
        return self.buffers[name]


def _find_kernel_node(graph, stem: str):
    kernels = [n for n in graph.nodes.values() if type(n.op).__name__ == "KernelOp"]
    if not kernels:
        raise ValueError("IR contains no KernelOp")
    if len(kernels) == 1:
        return kernels[0]
    for n in kernels:
        if n.op.name == stem:
            return n
    raise ValueError(f"cannot tell which of {[n.op.name for n in kernels]} to compile")


def _dtype_name(dt) -> str:
    return getattr(dt, "name", str(dt))


def _graph_buffers(graph) -> dict:
    out = {}
    for node in graph.nodes.values():
        for o in node.outputs:
            out[o.name] = Param(o.name, _dtype_name(o.dtype),
                                tuple(int(getattr(d, "value", d)) for d in o.shape))
    return out


def _constants(graph) -> dict:
    out = {}
    for node in graph.nodes.values():
        if type(node.op).__name__ != "ConstantOp":
            continue
        value = getattr(node.op, "value", None)
        if isinstance(value, (int, float)) and not isinstance(value, bool):
            out[node.id] = value
    return out


def load(ir_path) -> KernelSpec:
    """Read ``<entry>.ir.json`` and the ``meta.json`` beside it."""
    ir_path = Path(ir_path)
    Graph = load_graph_class()
    graph = Graph.from_dict(json.loads(ir_path.read_text(encoding="utf-8")))
    stem = ir_path.name.removesuffix(".ir.json")
    node = _find_kernel_node(graph, stem)
    kernel = node.op
    buffers = _graph_buffers(graph)

    meta_path = ir_path.parent / "meta.json"
    entry = None
    if meta_path.exists():
        meta = json.loads(meta_path.read_text(encoding="utf-8"))
        entry = next((k for k in meta.get("kernels", ()) if k["entry"] == kernel.name), None)

    if entry is not None:
        params = tuple(Param(a["name"], a["dtype"], tuple(a["shape"]), bool(a.get("scalar", False)))
                       for a in entry["args"])
        by_name = {p.name: p for p in params}
        missing = [n for n in entry["arg_order"] if n not in by_name]
        if missing:
            raise ValueError(f"meta.json arg_order names unknown args {missing}")
        params = tuple(by_name[n] for n in entry["arg_order"])
        grid, block = tuple(entry["grid"]), tuple(entry["block"])
        smem_bytes = int(entry.get("smem_bytes", 0))
        args_meta = tuple(entry["args"])
        zero_outputs = tuple(entry.get("zero_outputs", ()))
    else:
        names = list(node.inputs) + [o.name for o in node.outputs]
        params = tuple(buffers[n] for n in names)
        grid = block = None
        smem_bytes = 0
        args_meta = ()
        zero_outputs = ()

    return KernelSpec(kernel.name, tuple(kernel.body), params, grid, block, _constants(graph),
                      smem_bytes, buffers, args_meta, zero_outputs)
