"""Parity at BASELINE.json's full sizes, on the exact inputs bench.py times.

Every benchmark configuration runs once at its full size through the same compiled
kernel and the same seeded inputs as ``bench.py`` (``baseline_configs``).  The oracle
cannot redo a whole 8192^3 GEMM or the whole attention in seconds, so the checks are
the ones that do not depend on size, with the criterion of ``parity.py``
(``||out - ref|| / ||ref||`` within BASELINE.json's relative bar, and every element
within 4 bf16 ulps of the output's largest magnitude, no absolute floor):

* GEMM: the whole output at 512^3 and 2048^3, sampled rows at the larger sizes,
  recomputed by the oracle in f64, rel 1e-2;
* attention: 16 or more query rows of EVERY one of the 256 batch x head pairs, rel 1e-2;
* FP8: sampled rows, rel 5e-2, the quantised operands bit-exact with the oracle's cast;
* RMSNorm: the whole 4096 x 4096 output within 1e-5 relative per element;
* row softmax: sampled rows within 1e-5 relative, and every one of the 65536 rows
  sums to 1;
* global sum: the f64 sum of all 2^31 inputs, within 1e-5 relative.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from parity import assert_parity, sample_rows


def _run(name: str):
    """Compile the configuration's kernel, upload its inputs, launch once; returns
    (host inputs by IR argument, output as a host array)."""
    import baseline_configs as bc
    import emmyrt
    from compiler import synth
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel
    irs, meta = bc.shard_problem(name)
    d = synth.problem_dir(irs, meta)
    k = meta["kernels"][0]
    inputs = bc.shard_inputs(name, meta)
    ck = CompiledKernel.from_ir(d / f"{k['entry']}.ir.json")
    bufs = {}
    for a in k["args"]:
        h = inputs[a["name"]]
        bufs[a["name"]] = DeviceBuffer(h.nbytes)
        bufs[a["name"]].upload(h)
    ck({n: b.ptr for n, b in bufs.items()})
    emmyrt.stream_wait(0, 120)
    assert ck.status() == 0, f"kernel status {ck.status()}"
    out_name = bc.output_name(meta)
    out = np.zeros_like(inputs[out_name])
    bufs[out_name].download(out)
    for b in bufs.values():
        b.free()
    return inputs, out


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["gemm_8192", "gemm_4096x14336x4096", "gemm_2048", "gemm_512"])
def test_gemm_full_size_sampled_rows(runtime, name):
    from hostfmt import bf16_bits_to_f32
    from oracle.refs import mm_bf16
    inputs, out = _run(name)
    A = bf16_bits_to_f32(inputs["x0"])
    B = bf16_bits_to_f32(inputs["x1"])
    C = bf16_bits_to_f32(out)
    # every row where the f64 oracle takes seconds (512^3, 2048^3), sampled rows above
    rows = np.arange(A.shape[0]) if A.shape[0] * B.shape[1] <= 2048 * 2048 else sample_rows(A.shape[0], 48)
    assert_parity(C[rows], mm_bf16(A[rows], B), rel=1e-2, what=name)
    assert np.isfinite(C).all()


@pytest.mark.gpu
def test_attention_full_size_every_head(runtime):
    from hostfmt import bf16_bits_to_f32
    from oracle.refs import attn_bf16
    inputs, out = _run("attention")
    q, kk, v = (bf16_bits_to_f32(inputs[n]) for n in ("x0", "x1", "x2"))
    o = bf16_bits_to_f32(out)
    B, H, S, D = q.shape
    scale = 1.0 / math.sqrt(D)
    got, ref = [], []
    for b in range(B):
        for h in range(H):
            rows = sample_rows(S, 16, seed=b * H + h)
            got.append(o[b, h, rows])
            ref.append(attn_bf16(q[b, h, rows], kk[b, h], v[b, h], scale))
            # each pair on its own too: a head-indexing mistake shows up where it happens
            assert_parity(got[-1], ref[-1], rel=1e-2, what=f"(b={b}, h={h})")
    assert_parity(np.concatenate(got), np.concatenate(ref), rel=1e-2, what="all pairs")
    assert np.isfinite(o).all()


@pytest.mark.gpu
def test_fp8_full_size_sampled_rows(runtime):
    import baseline_configs as bc
    import emmyrt
    from emmyrt import DeviceBuffer
    from emmyrt.fp8 import Fp8Gemm, e4m3_decode
    from hostfmt import bf16_bits_to_f32
    from oracle.refs import e4m3_round, mm_fp8
    _, meta = bc.shard_problem("fp8_8192")
    inputs = bc.shard_inputs("fp8_8192", meta)
    A, B = inputs["a"], inputs["b"]
    n = A.shape[0]
    g = Fp8Gemm(n, n, n)
    da, db, dc = DeviceBuffer(A.nbytes), DeviceBuffer(B.nbytes), DeviceBuffer(n * n * 2)
    da.upload(A)
    db.upload(B)
    g.quantize(da.ptr, db.ptr)
    g.gemm(None, 0, g.gemm_params(dc.ptr))
    emmyrt.stream_wait(0, 120)
    assert g.gemm.status() == 0
    sa, sb = g.scales()
    assert sa == np.float32(np.abs(A).max()) / np.float32(448.0)
    assert sb == np.float32(np.abs(B).max()) / np.float32(448.0)
    qa = np.zeros((n, n), np.uint8)
    qb = np.zeros((n, n), np.uint8)
    g.qa.download(qa)
    g.qb.download(qb)
    rows = sample_rows(n, 24)
    # quantisation of the sampled rows is bit-exact with the oracle's e4m3 cast
    assert np.array_equal(e4m3_decode(qa[rows]), e4m3_round(A[rows] / np.float32(sa)))
    assert np.array_equal(e4m3_decode(qb[rows]), e4m3_round(B[rows] / np.float32(sb)))
    out = np.zeros((n, n), np.uint16)
    dc.download(out)
    C = bf16_bits_to_f32(out)
    ref = mm_fp8(e4m3_decode(qa[rows]), e4m3_decode(qb), sa, sb)
    assert_parity(C[rows], ref, rel=5e-2, what="fp8_8192")
    for b in (da, db, dc):
        b.free()


@pytest.mark.gpu
def test_rmsnorm_full_size(runtime):
    from oracle.refs import rmsnorm
    inputs, out = _run("rmsnorm")
    ref = rmsnorm(inputs["x0"], inputs["x1"], 1e-6).astype(np.float64)
    err = np.abs(out.astype(np.float64) - ref)
    assert np.all(err <= 1e-5 * np.abs(ref) + 1e-6), f"max abs err {err.max()}"


@pytest.mark.gpu
def test_softmax_full_size(runtime):
    from oracle.refs import softmax
    inputs, out = _run("softmax")
    x = inputs["x"]
    rows = sample_rows(x.shape[0], 256)
    ref = softmax(x[rows]).astype(np.float64)
    err = np.abs(out[rows].astype(np.float64) - ref)
    assert np.all(err <= 1e-5 * np.abs(ref) + 1e-9), f"max abs err {err.max()}"
    # every row is a distribution
    s = out.sum(axis=1, dtype=np.float64)
    assert np.all(np.abs(s - 1.0) <= 1e-5), f"row sums off by {np.max(np.abs(s - 1.0))}"
    assert (out >= 0).all()


@pytest.mark.gpu
def test_sum_full_size(runtime):
    inputs, out = _run("sum")
    x = inputs["x"]
    c = 1 << 24
    ref = math.fsum(float(x[i:i + c].sum(dtype=np.float64)) for i in range(0, x.size, c))
    got = float(out.reshape(-1)[0])
    assert abs(got - ref) <= 1e-5 * max(abs(ref), 1.0), f"{got} vs {ref}"
