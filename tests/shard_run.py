"""One rank of a sharded run of BASELINE configurations (test infrastructure).

Launched by ``test_gpu_multi.py`` under torchrun, one process per GPU:

    torchrun --nproc-per-node 2 tests/shard_run.py OUT_DIR NAME[,NAME...]

Each rank sets up its shard of every named configuration exactly as ``bench.py`` does
(``bench.Workload``: the shard's kernel, its seeded inputs, the FP8 amax all-reduce,
the sum's f64 all-reduce), runs one step and writes its output to
``OUT_DIR/<name>_r<rank>.npy`` (for the sum: the all-reduced f64 total).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "emmy-hackathon-2026_b200"))
sys.path.insert(0, str(ROOT))


def main() -> int:
    import bench
    import emmyrt
    from emmyrt.dist import NcclComm, share_unique_id
    out_dir, names = Path(sys.argv[1]), sys.argv[2].split(",")
    dist = bench.Dist()
    emmyrt.init(dist.local)
    uid = share_unique_id(dist.rank, dist.broadcast_bytes)
    comm = NcclComm(uid, dist.world, dist.rank)
    try:
        for name in names:
            w = bench.Workload(name, dist, comm)
            try:
                w.step(0, 0)
                emmyrt.stream_wait(0, 120)
                if w.ck.status():
                    raise RuntimeError(f"{name}: kernel status {w.ck.status()}")
                if w.total is not None:
                    res = np.zeros(2, np.float64)
                    w.total.download(res)
                    res = res[:1]
                else:
                    o = w.out_names[0]
                    res = np.zeros_like(w.inputs[o])
                    w.bufsets[0][o].download(res)
                np.save(out_dir / f"{name}_r{dist.rank}.npy", res)
            finally:
                w.free()
            dist.barrier()
    finally:
        emmyrt.synchronize()
        dist.barrier()
        comm.destroy()
        dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
