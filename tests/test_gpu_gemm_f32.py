"""f32 matmuls on the B200: emmy's SIMT FMA schedule (``problems/m01_matmul_512``,
``problems/m02_matmul_rect``, ``tests/problems/x_m_*``) lowered to the tcgen05 GEMM
with 3xTF32 operands, against the golden vectors and the f64 oracle."""

import json

import numpy as np
import pytest

from conftest import GOLDEN

F32_MM = ["m01_matmul_512", "m02_matmul_rect", "x_m_small", "x_m_tall", "x_m_wide", "x_m_longk",
          "x_m_256", "x_m_batched", "x_m_bias_relu", "x_m_scaled",
          # f32 operands cast to bf16 / f16: one exact tf32 MMA of the rounded values
          "x_q_bf16_mm", "x_q_bf16_mm_t", "x_q_f16_mm_t",
          # rows not 16-byte aligned, 16-bit and mixed operands: loaded by the converter warps
          "x_q_bf16_mm_odd", "x_h_mm_odd", "x_h_mm_odd2", "x_h_mm_mixed", "x_m_odd",
          # f64 buffers whose products the IR takes in f32
          "x_d_f64_mm"]


@pytest.mark.gpu
@pytest.mark.parametrize("pid", F32_MM)
def test_f32_matmul_matches_golden(runtime, pid):
    from emmyrt.runner import run_problem
    from oracle.refs import problem_expected
    d = GOLDEN / pid
    meta = json.loads((d / "meta.json").read_text())
    res = run_problem(d)
    exp = dict(np.load(d / "expected.npz"))
    ora = problem_expected(meta)
    for name, ref in exp.items():
        got = res["outputs"][name].reshape(ref.shape)
        err = np.max(np.abs(got - ref))
        assert np.allclose(got, ref, rtol=meta["rtol"], atol=meta["atol"]), f"{pid}:{name} max abs err {err}"
        assert np.allclose(got, np.asarray(ora[name]).reshape(ref.shape), rtol=meta["rtol"], atol=meta["atol"])


def _run_f32(m, n, k, b_kmajor=False, batch=1, bias=False, seed=0, BN=None, ksplit=0, launches=1):
    import emmyrt
    from compiler.kernels.gemm import GemmConfig, choose_tiling_f32, emit_gemm_module
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel
    tiling = choose_tiling_f32(m, n, batch)
    if BN is not None:
        tiling = dict(tiling, BN=BN, stages=min(4, (232448 - 256 - 1024) // (2 * (128 * 128 + BN * 128))))
    epi = (("bias", "bias"),) if bias else ()
    cfg = GemmConfig(M=m, N=n, K=k, batch=batch, ab="f32", c="f32", b_kmajor=b_kmajor, **tiling,
                     epilogue=epi, name="k_gemm_f32_test", buffers=("a", "b", "c", "bias"),
                     operand_dtypes=(("bias", "f32"),), ksplit=ksplit)
    ck = CompiledKernel.from_module(emit_gemm_module(cfg), "k_gemm_f32_test", ["a", "b", "c", "bias"])
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((batch, m, k)).astype(np.float32)
    B = rng.standard_normal((batch, n, k) if b_kmajor else (batch, k, n)).astype(np.float32)
    bv = rng.standard_normal(n).astype(np.float32)
    da, db, dc, dbias = DeviceBuffer(A.nbytes), DeviceBuffer(B.nbytes), DeviceBuffer(batch * m * n * 4), \
        DeviceBuffer(bv.nbytes)
    da.upload(A)
    db.upload(B)
    dbias.upload(bv)
    first = None
    for launch in range(launches):
        # the same module again: split-K tickets left at zero by the last slice serve the
        # next launch with the once-zeroed scratch
        dc.zero()
        ck({"a": da.ptr, "b": db.ptr, "c": dc.ptr, "bias": dbias.ptr})
        emmyrt.stream_wait(0, 60)
        assert ck.status() == 0
        out = np.zeros((batch, m, n), np.float32)
        dc.download(out)
        if first is None:
            first = out
        assert np.array_equal(out, first), f"launch {launch} differs from the first"
    Bm = np.swapaxes(B, -1, -2) if b_kmajor else B
    ref = A.astype(np.float64) @ Bm.astype(np.float64)
    scale = np.abs(A.astype(np.float64)) @ np.abs(Bm.astype(np.float64))
    if bias:
        ref = ref + bv
        scale = scale + np.abs(bv)
    return out, ref, scale


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,b_kmajor,batch,BN", [
    (512, 512, 512, False, 1, None),
    (1000, 600, 300, False, 1, None),       # partial M and N tiles, K not a multiple of 32
    (384, 256, 1024, True, 1, None),        # B stored [N, K]
    (200, 96, 64, False, 3, 64),            # batched, partial M tile
    (2048, 2048, 2048, False, 1, 128),
])
def test_3xtf32_accuracy(runtime, m, n, k, b_kmajor, batch, BN):
    out, ref, scale = _run_f32(m, n, k, b_kmajor, batch, BN=BN)
    # hi*hi + hi*lo + lo*hi misses each product by about 2^-21 of its size and the f32
    # accumulation adds about 2^-24 per step: 2^-16 of sum |a||b| holds with room, while
    # single tf32 products (2^-11 each) would miss it
    err = np.abs(out - ref) / scale
    assert np.max(err) <= 2.0 ** -16, f"max error {np.max(err)} of sum |a||b|"


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,batch,bias,ksplit", [(130, 100, 512, 1, True, 4), (200, 96, 256, 3, False, 2)])
def test_3xtf32_split_k(runtime, m, n, k, batch, bias, ksplit):
    """Forced K slices: the bias epilogue runs once, after the ordered sum of the slices;
    batched tiles take their own tickets."""
    out, ref, scale = _run_f32(m, n, k, batch=batch, bias=bias, BN=64, ksplit=ksplit, launches=3)
    assert np.max(np.abs(out - ref) / scale) <= 2.0 ** -16


@pytest.mark.gpu
def test_3xtf32_bias_on_ragged_tiles(runtime):
    out, ref, scale = _run_f32(130, 100, 64, bias=True, BN=64)
    assert np.max(np.abs(out - ref) / scale) <= 2.0 ** -16


def _run_direct(m, n, k, a_dt, b_dt, b_kmajor, rnd, seed=1):
    """The converter warps' own operand loads (no TMA) on odd shapes: several tiles, several
    stages, partial tiles on every edge."""
    import emmyrt
    from compiler.kernels.gemm import GemmConfig, choose_tiling_f32, emit_gemm_module
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel, f32_to_bf16_bits, bf16_bits_to_f32
    cfg = GemmConfig(M=m, N=n, K=k, ab="f32", c="f32", b_kmajor=b_kmajor,
                     **choose_tiling_f32(m, n, 1, split3=rnd is None), name="k_gemm_direct",
                     buffers=("a", "b", "c"), operand_round=rnd, direct=True, a_dtype=a_dt, b_dtype=b_dt)
    ck = CompiledKernel.from_module(emit_gemm_module(cfg), "k_gemm_direct", ["a", "b", "c"])
    rng = np.random.default_rng(seed)

    def host(shape, dt):
        x = rng.standard_normal(shape).astype(np.float32)
        if dt == "f16":
            return x.astype(np.float16), x.astype(np.float16).astype(np.float64)
        if dt == "bf16":
            bits = f32_to_bf16_bits(x)
            return bits, bf16_bits_to_f32(bits).astype(np.float64)
        return x, x.astype(np.float64)
    A, Af = host((m, k), a_dt)
    B, Bf = host((n, k) if b_kmajor else (k, n), b_dt)
    da, db, dc = DeviceBuffer(A.nbytes), DeviceBuffer(B.nbytes), DeviceBuffer(m * n * 4)
    da.upload(A)
    db.upload(B)
    dc.zero()
    ck({"a": da.ptr, "b": db.ptr, "c": dc.ptr})
    emmyrt.stream_wait(0, 60)
    assert ck.status() == 0
    out = np.zeros((m, n), np.float32)
    dc.download(out)
    Bm = Bf.T if b_kmajor else Bf
    return out, Af @ Bm, np.abs(Af) @ np.abs(Bm)


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,a_dt,b_dt,b_kmajor,rnd", [
    (300, 173, 229, "f32", "f32", False, None),     # 3xTF32, every row length odd
    (257, 130, 101, "f32", "f32", True, None),
    (200, 77, 135, "f16", "f16", False, "f16"),     # 16-bit rows of 154 / 270 bytes
    (129, 95, 67, "bf16", "bf16", True, "bf16"),
    (70, 50, 45, "f16", "f32", False, None),        # mixed: f16 A exact, f32 B split
])
def test_direct_loads_on_odd_shapes(runtime, m, n, k, a_dt, b_dt, b_kmajor, rnd):
    out, ref, scale = _run_direct(m, n, k, a_dt, b_dt, b_kmajor, rnd)
    # 16-bit operands are exact in tf32: only the f32 accumulation differs
    assert np.max(np.abs(out - ref) / scale) <= 2.0 ** -16
