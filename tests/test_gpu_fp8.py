"""FP8 e4m3 pipeline on the B200: amax, quantisation (bit-exact with torch's cast
semantics, restated in the oracle) and the tcgen05 kind::f8f6f4 GEMM."""

import numpy as np
import pytest


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(256, 512, 384), (1024, 1024, 1024), (300, 272, 160)])
def test_fp8_gemm_pipeline(runtime, m, n, k):
    import emmyrt
    from emmyrt import DeviceBuffer
    from emmyrt.fp8 import Fp8Gemm, e4m3_decode
    from emmyrt.runner import bf16_bits_to_f32
    from oracle.refs import e4m3_round, mm_fp8
    rng = np.random.default_rng(3)
    A = rng.standard_normal((m, k), dtype=np.float32)
    B = rng.standard_normal((k, n), dtype=np.float32)
    g = Fp8Gemm(m, n, k)
    da, db, dc = DeviceBuffer(A.nbytes), DeviceBuffer(B.nbytes), DeviceBuffer(m * n * 2)
    da.upload(A)
    db.upload(B)
    g.quantize(da.ptr, db.ptr)
    g.gemm(None, 0, g.gemm_params(dc.ptr))
    emmyrt.stream_wait(0, 60)
    assert g.gemm.status() == 0
    sa, sb = g.scales()
    # scales: amax / 448 in f32
    assert sa == np.float32(np.abs(A).max()) / np.float32(448.0)
    assert sb == np.float32(np.abs(B).max()) / np.float32(448.0)
    qa = np.zeros(m * k, np.uint8)
    g.qa.download(qa)
    ref_qa = e4m3_round(A.reshape(-1) / np.float32(sa))
    assert np.array_equal(e4m3_decode(qa), ref_qa), "quantisation is not bit-exact"
    qb = np.zeros(k * n, np.uint8)
    g.qb.download(qb)
    out = np.zeros((m, n), np.uint16)
    dc.download(out)
    got = bf16_bits_to_f32(out)
    ref = mm_fp8(e4m3_decode(qa).reshape(m, k), e4m3_decode(qb).reshape(k, n), sa, sb)
    # the BASELINE fp8 bar: within 5e-2 relative
    assert np.allclose(got, ref, rtol=5e-2, atol=5e-2 * np.abs(ref).max()), \
        f"max abs err {np.max(np.abs(got - ref))}"
