"""Parity at BASELINE.json's full sizes, on the exact inputs bench.py times.

Every benchmark configuration runs once at its full size through the same compiled
kernel and the same seeded input generator as ``bench.py`` (``bench.problem`` /
``bench.host_inputs``).  The oracle cannot redo a whole 8192^3 GEMM or the whole
attention in seconds, so the checks are the ones that do not depend on size:

* GEMM / FP8 / attention: sampled rows (and batch x head pairs) recomputed by the
  oracle in f64, within the BASELINE tolerances (bf16 1e-2, fp8 5e-2);
* RMSNorm: the whole 4096 x 4096 output, within 1e-5 relative;
* row softmax: sampled rows against the oracle within 1e-5 relative, and every one
  of the 65536 rows sums to 1;
* global sum: the f64 sum of all 2^31 inputs, within 1e-5 relative.
"""

from __future__ import annotations

import math

import numpy as np
import pytest


def _run(name: str):
    """Compile the workload's kernel, upload bench.py's inputs, launch once; returns
    (host inputs, output name, device output as host array, kernel)."""
    import bench
    import emmyrt
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel, NP_DTYPE
    d, meta = bench.problem(name)
    k = meta["kernels"][0]
    inputs = bench.host_inputs(name, meta, 0)
    ck = CompiledKernel.from_ir(d / f"{k['entry']}.ir.json")
    bufs = {}
    for a in k["args"]:
        h = inputs[a["name"]]
        bufs[a["name"]] = DeviceBuffer(h.nbytes)
        bufs[a["name"]].upload(h)
    ck({n: b.ptr for n, b in bufs.items()})
    emmyrt.stream_wait(0, 120)
    assert ck.status() == 0, f"kernel status {ck.status()}"
    out_arg = [a for a in k["args"] if a.get("output")][0]
    out = np.zeros(tuple(out_arg["shape"]) or (1,), dtype=NP_DTYPE[out_arg["dtype"]])
    bufs[out_arg["name"]].download(out)
    return inputs, k, out


def _rows(n: int, count: int, seed: int = 0) -> np.ndarray:
    """First, last and random rows of an n-row output."""
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, count)]))


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["gemm_8192", "gemm_4096x14336x4096", "gemm_2048", "gemm_512"])
def test_gemm_full_size_sampled_rows(runtime, name):
    from emmyrt.runner import bf16_bits_to_f32
    from oracle.refs import mm_bf16
    inputs, k, out = _run(name)
    A = bf16_bits_to_f32(inputs["x0"])
    B = bf16_bits_to_f32(inputs["x1"])
    C = bf16_bits_to_f32(out)
    rows = _rows(A.shape[0], 48)
    ref = mm_bf16(A[rows], B)
    # fp32-accumulated bf16: within 1e-2 relative (BASELINE tolerance)
    assert np.allclose(C[rows], ref, rtol=1e-2, atol=1e-2), \
        f"{name}: max abs err {np.max(np.abs(C[rows] - ref))}"
    assert np.isfinite(C).all()


@pytest.mark.gpu
def test_attention_full_size_sampled_heads(runtime):
    from emmyrt.runner import bf16_bits_to_f32
    from oracle.refs import attn_bf16
    inputs, k, out = _run("attention")
    q, kk, v = (bf16_bits_to_f32(inputs[n]) for n in ("x0", "x1", "x2"))
    o = bf16_bits_to_f32(out)
    B, H, S, D = q.shape
    scale = 1.0 / math.sqrt(D)
    for b, h in ((0, 0), (B - 1, H - 1), (3, 17)):
        rows = _rows(S, 200, seed=b * H + h)
        ref = attn_bf16(q[b, h, rows], kk[b, h], v[b, h], scale)
        assert np.allclose(o[b, h, rows], ref, rtol=1e-2, atol=1e-2), \
            f"(b={b}, h={h}) max abs err {np.max(np.abs(o[b, h, rows] - ref))}"
    assert np.isfinite(o).all()


@pytest.mark.gpu
def test_fp8_full_size_sampled_rows(runtime):
    import emmyrt
    from emmyrt import DeviceBuffer
    from emmyrt.fp8 import Fp8Gemm, e4m3_decode
    from emmyrt.runner import bf16_bits_to_f32
    from oracle.refs import e4m3_round, mm_fp8
    import bench
    _, meta = bench.problem("fp8_8192")
    inputs = bench.host_inputs("fp8_8192", meta, 0)
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
    rows = _rows(n, 24)
    # quantisation of the sampled rows is bit-exact with the oracle's e4m3 cast
    assert np.array_equal(e4m3_decode(qa[rows]), e4m3_round(A[rows] / np.float32(sa)))
    out = np.zeros((n, n), np.uint16)
    dc.download(out)
    C = bf16_bits_to_f32(out)
    ref = mm_fp8(e4m3_decode(qa[rows]), e4m3_decode(qb), sa, sb)
    assert np.allclose(C[rows], ref, rtol=5e-2, atol=5e-2 * np.abs(ref).max()), \
        f"max abs err {np.max(np.abs(C[rows] - ref))}"


@pytest.mark.gpu
def test_rmsnorm_full_size(runtime):
    from oracle.refs import rmsnorm
    inputs, k, out = _run("rmsnorm")
    ref = rmsnorm(inputs["x0"], inputs["x1"], 1e-6).astype(np.float64)
    err = np.abs(out.astype(np.float64) - ref)
    assert np.all(err <= 1e-5 * np.abs(ref) + 1e-6), f"max abs err {err.max()}"


@pytest.mark.gpu
def test_softmax_full_size(runtime):
    from oracle.refs import softmax
    inputs, k, out = _run("softmax")
    x = inputs["x"]
    rows = _rows(x.shape[0], 256)
    ref = softmax(x[rows]).astype(np.float64)
    err = np.abs(out[rows].astype(np.float64) - ref)
    assert np.all(err <= 1e-5 * np.abs(ref) + 1e-9), f"max abs err {err.max()}"
    # every row is a distribution
    s = out.sum(axis=1, dtype=np.float64)
    assert np.all(np.abs(s - 1.0) <= 1e-5), f"row sums off by {np.max(np.abs(s - 1.0))}"
    assert (out >= 0).all()


@pytest.mark.gpu
def test_sum_full_size(runtime):
    inputs, k, out = _run("sum")
    x = inputs["x"]
    c = 1 << 24
    ref = math.fsum(float(x[i:i + c].sum(dtype=np.float64)) for i in range(0, x.size, c))
    got = float(out.reshape(-1)[0])
    assert abs(got - ref) <= 1e-5 * max(abs(ref), 1.0), f"{got} vs {ref}"
