"""Sharded BASELINE configurations on 2 GPUs reassemble into the 1-GPU result.

Two ranks (torchrun, one process per GPU, NCCL through the runtime) each run their
shard of the configured problems (``tests/shard_run.py``, the benchmark's own set-up);
the test then puts the pieces back together and checks them against the same problem
run whole on one GPU and against the oracle:

* GEMM 8192^3 / FP8 8192^3: the two N-panels of C side by side;
* attention: the two halves of the batch;
* RMSNorm / softmax: the two halves of the rows;
* the 2^31 sum: the f64 all-reduce of the two chunks' f64 totals, against the exact
  f64 sum of all 2^31 inputs.

Skipped on a box with fewer than 2 GPUs.
"""

from __future__ import annotations

import math
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT
from parity import assert_parity, sample_rows

NAMES = ["gemm_8192", "fp8_8192", "attention", "rmsnorm", "softmax", "sum"]


def _gpus() -> int:
    import emmyrt
    import ctypes
    n = ctypes.c_int()
    emmyrt.check(emmyrt.lib.emmy_rt_device_count(ctypes.byref(n)), "device count")
    return n.value


@pytest.fixture(scope="module")
def shards(runtime, tmp_path_factory):
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path_factory.mktemp("shards")
    env = {**os.environ, "PYTHONPATH": ""}
    cmd = ["timeout", "-k", "60", "900", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29531",
           str(ROOT / "tests" / "shard_run.py"), str(out), ",".join(NAMES)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return out


def _pieces(out, name):
    return [np.load(out / f"{name}_r{r}.npy") for r in range(2)]


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["gemm_8192", "attention", "rmsnorm", "softmax"])
def test_shards_reassemble_into_the_one_gpu_result(runtime, shards, name):
    from test_gpu_baseline import _run
    axis = {"gemm_8192": 1, "attention": 0, "rmsnorm": 0, "softmax": 0}[name]
    whole = np.concatenate(_pieces(shards, name), axis=axis)
    _, one = _run(name)
    assert whole.shape == one.shape
    if name == "gemm_8192":
        # a tile's K order depends on its place in the CTA's tile sequence (the serpentine
        # order), which differs between a panel and the whole: within one bf16 rounding
        from hostfmt import bf16_bits_to_f32
        assert_parity(bf16_bits_to_f32(whole), bf16_bits_to_f32(one), rel=5e-3, ulps=1,
                      what="2-GPU panels vs 1-GPU gemm_8192")
    else:
        # the same kernel code path per output element: the pieces equal the whole run
        assert np.array_equal(whole, one), f"{name}: {np.count_nonzero(whole != one)} elements differ"


@pytest.mark.gpu
def test_sharded_gemm_against_the_oracle(runtime, shards):
    import baseline_configs as bc
    from hostfmt import bf16_bits_to_f32
    from oracle.refs import mm_bf16
    C = bf16_bits_to_f32(np.concatenate(_pieces(shards, "gemm_8192"), axis=1))
    ts = bc.tensors("gemm_8192")
    rows = sample_rows(C.shape[0], 24, seed=5)
    A = bf16_bits_to_f32(bc.f32_to_bf16_bits(ts["A"].full()[rows]))
    B = bf16_bits_to_f32(bc.f32_to_bf16_bits(ts["B"].full()))
    assert_parity(C[rows], mm_bf16(A, B), rel=1e-2, what="2-GPU gemm_8192")


@pytest.mark.gpu
def test_sharded_fp8_uses_the_whole_b_scale(runtime, shards):
    import baseline_configs as bc
    from hostfmt import bf16_bits_to_f32
    from oracle.refs import e4m3_round, mm_fp8
    C = bf16_bits_to_f32(np.concatenate(_pieces(shards, "fp8_8192"), axis=1))
    ts = bc.tensors("fp8_8192")
    A, B = ts["A"].full(), ts["B"].full()
    sa = np.float32(np.abs(A).max()) / np.float32(448.0)
    sb = np.float32(np.abs(B).max()) / np.float32(448.0)       # all of B, not one panel
    rows = sample_rows(C.shape[0], 16, seed=6)
    ref = mm_fp8(e4m3_round(A[rows] / sa), e4m3_round(B / sb), sa, sb)
    assert_parity(C[rows], ref, rel=5e-2, what="2-GPU fp8_8192")


@pytest.mark.gpu
def test_sharded_sum_is_one_f64_allreduce(runtime, shards):
    import baseline_configs as bc
    t0, t1 = (float(p[0]) for p in _pieces(shards, "sum"))
    assert t0 == t1                                   # every rank holds the same total
    x = bc.tensors("sum")["X"]
    n, c = x.shape[0], 1 << 26
    exact = math.fsum(float(x.rows(i, min(n, i + c)).sum(dtype=np.float64)) for i in range(0, n, c))
    assert abs(t0 - exact) <= 1e-6 * max(abs(exact), 1.0), f"{t0} vs {exact}"
