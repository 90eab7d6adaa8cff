"""Multi-process host logic of the multi-GPU path, as gloo ranks on CPU (world size 2):
rank 0's NCCL unique id reaches every rank, the max-over-ranks of the timings, a rank that
dies (the survivor's next collective errors instead of hanging), and the panel partition
used for N-panel / batch x head / row / chunk sharding."""

import os
import socket

import pytest
import torch.multiprocessing as mp

from conftest import PKG, ROOT


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys
    for p in (str(PKG), str(ROOT)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import bench
    from emmyrt.dist import share_unique_id
    d = bench.Dist()
    try:
        uid = share_unique_id(d.rank, d.broadcast_bytes)
        m = d.max(float(rank + 1) * 1.5)
        d.barrier()
        q.put((rank, uid.hex(), m))
    finally:
        d.close()


def test_gloo_ranks_share_nccl_id_and_max():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ids = {u for _, u, _ in out}
    assert len(ids) == 1 and len(next(iter(ids))) == 256      # 128-byte ncclUniqueId
    assert all(m == 3.0 for _, _, m in out)                   # max over ranks


def _failing_worker(rank, world, port, q):
    import sys
    for p in (str(PKG), str(ROOT)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), EMMY_PG_TIMEOUT_S="10")
    import bench
    d = bench.Dist()
    d.barrier()
    if rank == 1:
        os._exit(3)                     # a rank that dies between steps
    try:
        d.max(1.0)
        q.put((rank, "completed"))
    except Exception as e:              # noqa: BLE001
        q.put((rank, type(e).__name__))


def test_surviving_rank_errors_instead_of_hanging():
    # failure detection on the host: rank 1 dies after a barrier, rank 0's next collective
    # ends with an error (connection lost or the short process-group timeout), not a hang
    import time
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    t0 = time.time()
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and outcome != "completed"
    assert procs[1].exitcode == 3
    assert time.time() - t0 < 110


@pytest.mark.parametrize("n,world", [(8192, 8), (65536, 3), (7, 4), (256, 1)])
def test_panels_partition(n, world):
    from emmyrt.dist import panel
    spans = [panel(n, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1
