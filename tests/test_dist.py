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


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_cover_every_configuration(world):
    """The shards of each BASELINE configuration tile the whole problem, and their
    algorithmic work adds up to the whole problem's."""
    import baseline_configs as bc
    for name, c in bc.CONFIGS.items():
        dims = [bc.shard_dims(name, r, world) for r in range(world)]
        key = "cols" if c.family in ("gemm", "fp8") else "rows"
        spans = [d[key] for d in dims]
        extent = c.dims[1] if c.family in ("gemm", "fp8") else c.dims[0]
        assert spans[0][0] == 0 and spans[-1][1] == extent, name
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:])), name
        total = sum(bc.work(name, r, world) for r in range(world))
        whole = bc.work(name)
        if name == "rmsnorm":          # every shard reads the whole weight vector
            whole += (world - 1) * c.dims[1] * 4
        assert total == whole, name


def test_shard_inputs_are_slices_of_the_whole_inputs():
    import numpy as np
    import baseline_configs as bc
    _, meta1 = bc.shard_problem("gemm_512")
    whole = bc.shard_inputs("gemm_512", meta1)
    panels = []
    for r in range(2):
        _, meta = bc.shard_problem("gemm_512", r, 2)
        x = bc.shard_inputs("gemm_512", meta, r, 2)
        assert np.array_equal(x["x0"], whole["x0"])            # A replicated
        panels.append(x["x1"])
    assert np.array_equal(np.concatenate(panels, axis=1), whole["x1"])
    t = bc.tensors("sum")["X"]
    n = (1 << 23) + 12345
    ref = t.rows(0, n)
    parts = [t.rows(*bc.panel(n, r, 3)) for r in range(3)]
    assert np.array_equal(np.concatenate(parts), ref)


def _sum_worker(rank, world, port, n, q):
    import sys
    for p in (str(PKG), str(ROOT)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import numpy as np
    import torch
    import baseline_configs as bc
    import bench
    d = bench.Dist()
    try:
        r0, r1 = bc.panel(n, rank, world)
        part = torch.tensor([bc.tensors("sum")["X"].rows(r0, r1).sum(dtype=np.float64)],
                            dtype=torch.float64)
        d.pg.all_reduce(part)                 # the f64 all-reduce that finishes the sum
        q.put((rank, float(part.item())))
    finally:
        d.close()


def test_sharded_sum_partials_reduce_in_f64():
    """The sum's chunks, reduced per rank in f64 and all-reduced in f64 (gloo here, NCCL
    on the GPUs), give the whole array's f64 sum on every rank."""
    import math
    import numpy as np
    import baseline_configs as bc
    world, n = 2, 1 << 24
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sum_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x = bc.tensors("sum")["X"].rows(0, n)
    exact = math.fsum(x.astype(np.float64))
    assert out[0] == out[1]
    assert abs(out[0] - exact) <= 1e-12 * abs(exact) + 1e-9
