"""``load(path)``: one Kernel IR json plus the ``meta.json`` beside it -> a KernelSpec.

The record types keep the reference's field names (``compiler/loader.py:17-39`` there),
because the compiler's callers read them; the way they are filled is this back end's own:

* one pass over the graph (:class:`_GraphIndex`) collects every tensor the graph names
  (shape and dtype, used by the templates to size tiles and tensor maps), the scalar
  value of every ``ConstantOp`` (folded to immediates) and the ``KernelOp`` nodes;
* the kernel to compile is the one named like the file (``<entry>.ir.json``), or the
  graph's only kernel;
* the launch contract (:class:`_Contract`) comes from the ``meta.json`` record whose
  ``entry`` is that kernel: parameter order (``arg_order``), emmy's grid / block /
  dynamic shared memory, the argument records the runner builds inputs from and the
  buffers re-zeroed before each launch.  A graph without a record is launched with its
  kernel's inputs followed by its outputs as parameters and no prescribed geometry.
"""

from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from pathlib import Path

from .ir import load_graph_class


@dataclass(frozen=True)
class Param:
    """One kernel parameter: a device buffer (``.u64`` pointer), or a by-value scalar."""
    name: str
    dtype: str
    shape: tuple[int, ...]
    scalar: bool = False


@dataclass(frozen=True)
class KernelSpec:
    """Everything the templates need to emit one kernel module."""
    name: str                   # the .entry symbol
    body: tuple                 # the KernelOp's statements
    params: tuple[Param, ...]   # parameter list, in the order the launcher passes them
    grid: tuple[int, int, int] | None    # emmy's own launch geometry, if meta.json gives it
    block: tuple[int, int, int] | None
    constants: dict             # ConstantOp tensor name -> scalar value
    smem_bytes: int = 0         # emmy's dynamic shared memory request
    buffers: dict = field(default_factory=dict)    # tensor name -> Param, for the whole graph
    args_meta: tuple = ()       # meta.json argument records (seed / data / output flags)
    zero_outputs: tuple = ()    # tensors cleared before every launch

    @property
    def threads_launched(self) -> int | None:
        if self.grid is None or self.block is None:
            return None
        return math.prod(self.grid) * math.prod(self.block)

    def param(self, name: str) -> Param:
        """A tensor by name: a parameter first, else any tensor of the graph."""
        return next((p for p in self.params if p.name == name), None) or self.buffers[name]


def _extent(d) -> int:
    return int(d.value) if hasattr(d, "value") else int(d)


class _GraphIndex:
    """Tensors, constants and kernels of a deserialised graph, gathered in one pass."""

    def __init__(self, graph):
        self.tensors: dict[str, Param] = {}
        self.constants: dict[str, float] = {}
        self.kernels: list = []
        for node in graph.nodes.values():
            kind = type(node.op).__name__
            for t in node.outputs:
                dtype = t.dtype.name if hasattr(t.dtype, "name") else str(t.dtype)
                self.tensors[t.name] = Param(t.name, dtype, tuple(_extent(d) for d in t.shape))
            if kind == "KernelOp":
                self.kernels.append(node)
            elif kind == "ConstantOp":
                v = getattr(node.op, "value", None)
                if type(v) in (int, float):          # bools and arrays are not scalars
                    self.constants[node.id] = v

    def kernel(self, wanted: str):
        by_name = {n.op.name: n for n in self.kernels}
        if wanted in by_name:
            return by_name[wanted]
        if len(self.kernels) == 1:
            return self.kernels[0]
        if not self.kernels:
            raise ValueError("the graph holds no KernelOp to compile")
        raise ValueError(f"several kernels in one graph ({sorted(by_name)}) and none is "
                         f"named {wanted!r} like the file")


@dataclass(frozen=True)
class _Contract:
    """The launch contract of one kernel."""
    params: tuple[Param, ...]
    grid: tuple | None = None
    block: tuple | None = None
    smem_bytes: int = 0
    args_meta: tuple = ()
    zero_outputs: tuple = ()

    @classmethod
    def from_meta(cls, record: dict) -> "_Contract":
        declared = {a["name"]: a for a in record["args"]}
        unknown = [n for n in record["arg_order"] if n not in declared]
        if unknown:
            raise ValueError(f"meta.json: arg_order lists {unknown}, which args does not declare")
        params = []
        for n in record["arg_order"]:
            a = declared[n]
            params.append(Param(n, a["dtype"], tuple(a["shape"]), bool(a.get("scalar", False))))
        return cls(tuple(params), tuple(record["grid"]), tuple(record["block"]),
                   int(record.get("smem_bytes", 0)), tuple(record["args"]),
                   tuple(record.get("zero_outputs", ())))

    @classmethod
    def from_graph(cls, node, index: _GraphIndex) -> "_Contract":
        names = [*node.inputs, *(t.name for t in node.outputs)]
        return cls(tuple(index.tensors[n] for n in names))


def _meta_record(meta_path: Path, entry: str) -> dict | None:
    if not meta_path.is_file():
        return None
    meta = json.loads(meta_path.read_text(encoding="utf-8"))
    for record in meta.get("kernels", ()):
        if record.get("entry") == entry:
            return record
    return None


def load(ir_path) -> KernelSpec:
    """Read ``<entry>.ir.json`` and its launch contract from ``meta.json`` in the same folder."""
    ir_path = Path(ir_path)
    graph = load_graph_class().from_dict(json.loads(ir_path.read_text(encoding="utf-8")))
    index = _GraphIndex(graph)
    node = index.kernel(ir_path.name.removesuffix(".ir.json"))
    record = _meta_record(ir_path.with_name("meta.json"), node.op.name)
    contract = _Contract.from_meta(record) if record is not None else _Contract.from_graph(node, index)
    return KernelSpec(name=node.op.name, body=tuple(node.op.body), params=contract.params,
                      grid=contract.grid, block=contract.block, constants=index.constants,
                      smem_bytes=contract.smem_bytes, buffers=index.tensors,
                      args_meta=contract.args_meta, zero_outputs=contract.zero_outputs)
