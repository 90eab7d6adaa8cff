"""Multi-GPU plumbing: one process per GPU, NCCL through the native runtime.

The reference has no multi-GPU path.  Here every partitioned problem shards without
communication on the data path (GEMM by N-panel, attention by batch x head, row kernels
by rows), and the whole-array reduction finishes with one all-reduce of the per-rank
f64 partials (the FP8 GEMM's per-tensor scale of a sharded B takes one all-reduce with
max of the panels' amax, before the timed GEMM):
``emmy_rt_nccl_*`` wraps ncclGetUniqueId / ncclCommInitRank / ncclAllReduce; rank 0's
unique id travels to the other ranks over the host process group (``torch.distributed``
with gloo), which carries no tensor data.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

from . import check, lib

NCCL_FLOAT32, NCCL_FLOAT64 = 7, 8
NCCL_SUM, NCCL_MAX, NCCL_MIN = 0, 2, 3


def nccl_library() -> str:
    """The NCCL shared library: $EMMY_NCCL_LIB, torch's bundled copy, or the loader path."""
    env = os.environ.get("EMMY_NCCL_LIB")
    if env:
        return env
    try:
        import nvidia.nccl as nn
        for base in nn.__path__:
            cand = Path(base) / "lib" / "libnccl.so.2"
            if cand.exists():
                return str(cand)
    except Exception:
        pass
    return "libnccl.so.2"


def load_nccl() -> None:
    check(lib.emmy_rt_nccl_load(nccl_library().encode()), "nccl load")


def unique_id() -> bytes:
    load_nccl()
    buf = (ctypes.c_ubyte * 128)()
    check(lib.emmy_rt_nccl_unique_id(buf), "ncclGetUniqueId")
    return bytes(buf)


def share_unique_id(rank: int, broadcast) -> bytes:
    """Rank 0 makes the NCCL unique id; ``broadcast(obj)`` (host collective) returns
    rank 0's object on every rank."""
    uid = unique_id() if rank == 0 else None
    uid = broadcast(uid)
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("NCCL unique id exchange failed")
    return bytes(uid)


class NcclComm:
    """A communicator over ``world`` ranks, one GPU each (device already current)."""

    def __init__(self, uid: bytes, world: int, rank: int):
        load_nccl()
        buf = (ctypes.c_ubyte * 128).from_buffer_copy(uid)
        c = ctypes.c_uint64()
        check(lib.emmy_rt_nccl_comm_init(ctypes.byref(c), world, buf, rank), "ncclCommInitRank")
        self.handle = c.value
        self.world, self.rank = world, rank

    def allreduce(self, send: int, recv: int, count: int, dtype: int = NCCL_FLOAT32,
                  op: int = NCCL_SUM, stream: int = 0) -> None:
        check(lib.emmy_rt_nccl_allreduce(self.handle, send, recv, count, dtype, op, stream),
              "ncclAllReduce")

    def destroy(self) -> None:
        if self.handle:
            lib.emmy_rt_nccl_comm_destroy(self.handle)
            self.handle = 0


from baseline_configs import panel  # noqa: E402,F401  (the one definition of the split)
