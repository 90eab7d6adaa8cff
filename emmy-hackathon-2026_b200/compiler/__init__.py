"""Emmy Kernel IR -> sm_100a PTX compiler (B200 back end).

Same surface as the reference's ``compiler`` package (``compiler/__init__.py:35-52``):
``load(path) -> KernelSpec`` and ``compile_kernel(spec) -> str``, plus the
``@handles`` statement registry in :mod:`compiler.stmts`.

``compile_kernel`` recognises which kernel family the IR describes and emits that
family's hand-written sm_100a template (tcgen05 GEMM / attention, streaming
reductions), computing the IR's own arithmetic.  The module starts with the
``.version``/``.target`` header; a ``// @launch {json}`` comment right after it
is the launch descriptor (grid, block, cluster, dynamic shared memory and the
parameters appended after meta.json's ``arg_order``), because the templates do not
run under emmy's sm_89 launch geometry.  IR outside the supported families raises
``NotImplementedError`` -- there is no scalar fallback.
"""

from __future__ import annotations

from .loader import KernelSpec, Param, load
from .stmts import HANDLERS, handles, lower_body
from .ptx import HEADER, parse_launch


def compile_kernel(spec: KernelSpec) -> str:
    """Lower one kernel to a complete sm_100a PTX module."""
    from .kernels import select
    return select(spec)


__all__ = ["compile_kernel", "load", "KernelSpec", "Param", "HANDLERS", "handles",
           "lower_body", "HEADER", "parse_launch"]
