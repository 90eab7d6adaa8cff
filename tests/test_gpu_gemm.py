"""Parity of the tcgen05 GEMM template on the B200 against the golden vectors and the oracle."""

import json

import numpy as np
import pytest

from conftest import GOLDEN

GEMM = ["x_h_mm_1024", "x_h_mm_256", "x_h_mm_relu", "x_h_mm_residual", "x_h_mm_t_n8", "x_h_mm_t_odd",
        "x_h_mm_rect", "x_h_bmm", "x_h_mm_bias", "x_h_linear_bias_gelu",
        "x_h_mm_16", "x_h_mm_64", "x_h_mm_128", "x_h_mm_t", "x_h_mm_vec", "x_q_f16_mm_t",
        "x_h_bmm_t", "x_h_linear",
        # two contractions in one kernel (element maps of the same arithmetic)
        "x_h_mlp", "x_l_swiglu_h"]


@pytest.mark.gpu
@pytest.mark.parametrize("pid", GEMM)
def test_gemm_matches_golden(runtime, pid):
    from emmyrt.runner import run_problem
    from oracle.refs import problem_expected
    d = GOLDEN / pid
    meta = json.loads((d / "meta.json").read_text())
    res = run_problem(d)
    for k in res["kernels"]:
        assert k.entry
    exp = dict(np.load(d / "expected.npz"))
    ora = problem_expected(meta)
    for name, ref in exp.items():
        got = res["outputs"][name].reshape(ref.shape)
        err = np.max(np.abs(got - ref.astype(np.float32)))
        assert np.allclose(got, ref.astype(np.float32), rtol=meta["rtol"], atol=meta["atol"]), \
            f"{pid}:{name} max abs err {err}"
        o = np.asarray(ora[name], dtype=np.float32).reshape(ref.shape)
        assert np.allclose(got, o, rtol=meta["rtol"], atol=meta["atol"])


def _direct_gemm(m, n, k, pair, b_kmajor, seed=0, batch=1, ksplit=0, launches=1, tail_split=0):
    from compiler.kernels.gemm import GemmConfig, emit_gemm_module
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel, bf16_bits_to_f32, f32_to_bf16_bits
    import emmyrt
    cfg = GemmConfig(M=m, N=n, K=k, batch=batch, ab="bf16", c="bf16", b_kmajor=b_kmajor, BN=256,
                     stages=6 if pair else 4, pair=pair, name="k_gemm_test", buffers=("a", "b", "c"),
                     ksplit=ksplit, tail_split=tail_split)
    if tail_split > 1:
        from compiler import parse_launch
        assert parse_launch(emit_gemm_module(cfg))["tail_split"] == tail_split
    ck = CompiledKernel.from_module(emit_gemm_module(cfg), "k_gemm_test", ["a", "b", "c"])
    rng = np.random.default_rng(seed)
    A = f32_to_bf16_bits(rng.standard_normal((batch, m, k), dtype=np.float32) * np.float32(0.05))
    bshape = (batch, n, k) if b_kmajor else (batch, k, n)
    B = f32_to_bf16_bits(rng.standard_normal(bshape, dtype=np.float32) * np.float32(0.05))
    da, db, dc = DeviceBuffer(A.nbytes), DeviceBuffer(B.nbytes), DeviceBuffer(batch * m * n * 2)
    da.upload(A)
    db.upload(B)
    first = None
    for launch in range(launches):
        # the same module again: split-K tickets left at zero by the last slice serve the
        # next launch with the once-zeroed scratch
        dc.zero()
        ck({"a": da.ptr, "b": db.ptr, "c": dc.ptr})
        emmyrt.stream_wait(0, 60)
        assert ck.status() == 0
        out = np.zeros((batch, m, n), np.uint16)
        dc.download(out)
        if first is None:
            first = out
        assert np.array_equal(out, first), f"launch {launch} differs from the first"
    Bf = bf16_bits_to_f32(B)
    if b_kmajor:
        Bf = np.swapaxes(Bf, -1, -2)
    return bf16_bits_to_f32(out), bf16_bits_to_f32(A), Bf


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,pair,kmaj", [(512, 512, 512, True, False), (640, 384, 320, True, False),
                                             (768, 512, 448, True, True), (512, 768, 256, False, False),
                                             (300, 200, 136, False, True)])
def test_gemm_direct_bf16(runtime, m, n, k, pair, kmaj):
    from oracle.refs import mm_bf16
    from parity import assert_parity
    got, A, B = _direct_gemm(m, n, k, pair, kmaj)
    assert_parity(got[0], mm_bf16(A[0], B[0]), rel=1e-2, what=f"{m}x{n}x{k}")


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,kmaj,ksplit", [(512, 512, 1024, False, 4), (300, 200, 512, True, 2)])
def test_gemm_split_k_bf16(runtime, m, n, k, kmaj, ksplit):
    """K slices forced on 16-bit tiles (the automatic choice keeps them for the f32 path):
    partials through the workspace, the last slice's ordered sum, ragged M and N tiles."""
    from oracle.refs import mm_bf16
    from parity import assert_parity
    got, A, B = _direct_gemm(m, n, k, False, kmaj, ksplit=ksplit, launches=3)
    assert_parity(got[0], mm_bf16(A[0], B[0]), rel=1e-2, what=f"split-K {ksplit}")


@pytest.mark.gpu
def test_pdl_chain_waits_for_the_previous_gemm(runtime):
    """Programmatic dependent launch: the second GEMM reads the first one's C as its A,
    launched right behind it on one stream with no host sync in between; its prologue may
    overlap the first GEMM, its loads must not (griddepcontrol.wait)."""
    import emmyrt
    from compiler.kernels.gemm import GemmConfig, emit_gemm_module
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel, bf16_bits_to_f32, f32_to_bf16_bits
    from oracle.refs import mm_bf16
    from parity import assert_parity
    n = 512
    cks = []
    for name in ("k_pdl_first", "k_pdl_second"):
        cfg = GemmConfig(M=n, N=n, K=n, ab="bf16", c="bf16", name=name, buffers=("a", "b", "c"))
        ck = CompiledKernel.from_module(emit_gemm_module(cfg), name, ["a", "b", "c"])
        assert ck.launch["pdl"] and ck.launch_flags == emmyrt.LAUNCH_PDL
        cks.append(ck)
    rng = np.random.default_rng(3)
    A = f32_to_bf16_bits(rng.standard_normal((n, n), dtype=np.float32) * np.float32(0.05))
    B = f32_to_bf16_bits(rng.standard_normal((n, n), dtype=np.float32) * np.float32(0.05))
    da, db, dc1, dc2 = (DeviceBuffer(n * n * 2) for _ in range(4))
    da.upload(A)
    db.upload(B)
    for rep in range(3):
        dc1.upload(np.full((n, n), 0x7FC0, np.uint16))          # NaN until the first GEMM writes
        dc2.zero()
        first = cks[0].prepare(cks[0].params({"a": da.ptr, "b": db.ptr, "c": dc1.ptr}))
        second = cks[1].prepare(cks[1].params({"a": dc1.ptr, "b": db.ptr, "c": dc2.ptr}))
        first(0)
        second(0)
        emmyrt.stream_wait(0, 60)
        assert cks[0].status() == 0 and cks[1].status() == 0
        c1 = np.zeros((n, n), np.uint16)
        c2 = np.zeros((n, n), np.uint16)
        dc1.download(c1)
        dc2.download(c2)
        C1, C2 = bf16_bits_to_f32(c1), bf16_bits_to_f32(c2)
        assert np.isfinite(C2).all(), f"rep {rep}: the second GEMM read the first's C too early"
        assert_parity(C1, mm_bf16(bf16_bits_to_f32(A), bf16_bits_to_f32(B)), rel=1e-2, what="first")
        assert_parity(C2, mm_bf16(C1, bf16_bits_to_f32(B)), rel=1e-2, what="second")


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,pair,ts", [(2560, 2048, 1024, True, 4),    # 80 pair tiles: 74 + 6 sliced
                                            (1280, 4096, 512, False, 2),    # 160 CTA tiles: 148 + 12
                                            (2560, 2048, 2048, True, 8)])
def test_gemm_tail_split(runtime, m, n, k, pair, ts):
    """The tiles past the last full wave cut into K slices (partials through the workspace,
    the last slice's ordered sum): against the oracle on rows of every M tile, against
    the same GEMM with whole tiles (within one bf16 rounding: only the tail's order
    differs), bit-identical over three launches of one module (the tickets reset)."""
    from oracle.refs import mm_bf16
    from parity import assert_parity
    got, A, B = _direct_gemm(m, n, k, pair, False, seed=7, launches=3, tail_split=ts)
    whole, _, _ = _direct_gemm(m, n, k, pair, False, seed=7, tail_split=1)
    rows = np.arange(0, m, 37)
    assert_parity(got[0][rows], mm_bf16(A[0][rows], B[0]), rel=1e-2, what=f"tail split {ts}")
    assert_parity(got[0], whole[0], rel=5e-3, ulps=1, what="tail split vs whole tiles")
