"""Parity of the tcgen05 attention template on the B200."""

import json
import math

import numpy as np
import pytest

from conftest import GOLDEN

ATTN = ["x_h_sdpa", "x_h_attn", "x_h_attn_128", "x_h_attn_b", "x_h_sdpa_causal", "x_h_sdpa_mask",
        # emmy's unrolled SIMT masked attention (pre-transposed K; odd 100 x 120 with a mask)
        "x_h_attn_mask", "x_h_sdpa_mask_odd",
        # Q K^T and softmax @ V as two kernels (50 x 70 keys); softmax of input scores @ V
        "x_h_attn_odd", "x_h_softmax_mm", "x_h_softmax_mm_odd"]


@pytest.mark.gpu
@pytest.mark.parametrize("pid", ATTN)
def test_attention_matches_golden(runtime, pid):
    from emmyrt.runner import run_problem
    from oracle.refs import problem_expected
    d = GOLDEN / pid
    meta = json.loads((d / "meta.json").read_text())
    res = run_problem(d)
    exp = dict(np.load(d / "expected.npz"))
    ora = problem_expected(meta)
    for name, ref in exp.items():
        got = res["outputs"][name].reshape(ref.shape)
        err = np.max(np.abs(got - ref.astype(np.float32)))
        assert np.allclose(got, ref.astype(np.float32), rtol=meta["rtol"], atol=meta["atol"]), \
            f"{pid}:{name} max abs err {err}"
        o = np.asarray(ora[name], dtype=np.float32).reshape(ref.shape)
        assert np.allclose(got, o, rtol=meta["rtol"], atol=meta["atol"])


def _run_direct(bh, sq, sk, d, seed=0):
    from compiler.kernels.attention import AttnConfig, emit_attention_module
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel, bf16_bits_to_f32, f32_to_bf16_bits
    cfg = AttnConfig(BH=bh, Sq=sq, Sk=sk, D=d, dtype="bf16", scale=1 / math.sqrt(d),
                     name="k_attn_test", buffers=("q", "k", "v", "o"))
    ck = CompiledKernel.from_module(emit_attention_module(cfg), "k_attn_test", ["q", "k", "v", "o"])
    rng = np.random.default_rng(seed)
    host = {n: f32_to_bf16_bits(rng.standard_normal((bh, s, d), dtype=np.float32))
            for n, s in (("q", sq), ("k", sk), ("v", sk))}
    bufs = {n: DeviceBuffer(a.nbytes) for n, a in host.items()}
    for n, a in host.items():
        bufs[n].upload(a)
    bufs["o"] = DeviceBuffer(bh * sq * d * 2)
    bufs["o"].zero()
    ptrs = {n: b.ptr for n, b in bufs.items()}
    ck(ptrs)
    import emmyrt
    emmyrt.stream_wait(0, 60)
    assert ck.status() == 0
    out = np.zeros((bh, sq, d), np.uint16)
    bufs["o"].download(out)
    f = {n: bf16_bits_to_f32(a) for n, a in host.items()}
    return bf16_bits_to_f32(out), f, cfg


@pytest.mark.gpu
@pytest.mark.parametrize("bh,sq,sk,d", [(2, 256, 512, 128), (3, 384, 640, 128), (1, 128, 200, 64)])
def test_attention_direct_bf16(runtime, bh, sq, sk, d):
    from oracle.refs import attn_bf16
    got, f, cfg = _run_direct(bh, sq, sk, d)
    ref = attn_bf16(f["q"], f["k"], f["v"], cfg.scale)
    # fp32-accumulated bf16: within 1e-2 relative (BASELINE tolerance), P rounded to bf16
    assert np.allclose(got, ref, rtol=1e-2, atol=1e-2), f"max abs err {np.max(np.abs(got - ref))}"


def _run_cfg(cfg, host, extra_bufs=()):
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel, bf16_bits_to_f32
    import emmyrt
    names = list(cfg.buffers)
    ck = CompiledKernel.from_module(emit_module(cfg), cfg.name, names)
    bufs = {n: DeviceBuffer(a.nbytes) for n, a in host.items()}
    for n, a in host.items():
        bufs[n].upload(a)
    bufs["o"] = DeviceBuffer(cfg.BH * cfg.Sq * cfg.D * 2)
    bufs["o"].zero()
    ck({n: b.ptr for n, b in bufs.items()})
    emmyrt.stream_wait(0, 60)
    assert ck.status() == 0
    out = np.zeros((cfg.BH, cfg.Sq, cfg.D), np.uint16)
    bufs["o"].download(out)
    return bf16_bits_to_f32(out)


def emit_module(cfg):
    from compiler.kernels.attention import emit_attention_module
    return emit_attention_module(cfg)


@pytest.mark.gpu
@pytest.mark.parametrize("bh,sq,sk,d", [(2, 384, 384, 128), (3, 512, 512, 64), (2, 256, 640, 128),
                                        (1, 300, 300, 64)])
def test_attention_causal_bf16(runtime, bh, sq, sk, d):
    """Causal attention (key > query masked, top-left aligned): the per-tile block counts,
    the diagonal masking, ragged query / key ends and the reversed CTA order."""
    from compiler.kernels.attention import AttnConfig
    from emmyrt.runner import bf16_bits_to_f32, f32_to_bf16_bits
    from oracle.refs import attn_bf16
    cfg = AttnConfig(BH=bh, Sq=sq, Sk=sk, D=d, dtype="bf16", scale=1 / math.sqrt(d), causal=True,
                     name="k_attn_causal", buffers=("q", "k", "v", "o"))
    rng = np.random.default_rng(5)
    host = {n: f32_to_bf16_bits(rng.standard_normal((bh, s, d), dtype=np.float32))
            for n, s in (("q", sq), ("k", sk), ("v", sk))}
    got = _run_cfg(cfg, host)
    f = {n: bf16_bits_to_f32(a) for n, a in host.items()}
    ref = attn_bf16(f["q"], f["k"], f["v"], cfg.scale, causal=True)
    assert np.allclose(got, ref, rtol=1e-2, atol=1e-2), f"max abs err {np.max(np.abs(got - ref))}"


@pytest.mark.gpu
@pytest.mark.parametrize("bh,sq,sk,d,per_head", [(2, 256, 384, 128, False), (3, 384, 256, 64, True)])
def test_attention_additive_mask_bf16(runtime, bh, sq, sk, d, per_head):
    """Additive score mask, shared by every batch x head or one per batch x head, with
    some entries at -1e4 (masked-out keys)."""
    from compiler.kernels.attention import AttnConfig
    from emmyrt.runner import bf16_bits_to_f32, f32_to_bf16_bits
    from oracle.refs import attn_bf16
    cfg = AttnConfig(BH=bh, Sq=sq, Sk=sk, D=d, dtype="bf16", scale=1 / math.sqrt(d),
                     name="k_attn_mask", buffers=("q", "k", "v", "mask", "o"), mask_param="mask",
                     mask_dtype="bf16", mask_bh_stride=sq * sk if per_head else 0)
    rng = np.random.default_rng(6)
    host = {n: f32_to_bf16_bits(rng.standard_normal((bh, s, d), dtype=np.float32))
            for n, s in (("q", sq), ("k", sk), ("v", sk))}
    mshape = (bh, sq, sk) if per_head else (sq, sk)
    m = rng.standard_normal(mshape, dtype=np.float32)
    m[rng.random(mshape) < 0.2] = -1e4
    host["mask"] = f32_to_bf16_bits(m)
    got = _run_cfg(cfg, host)
    f = {n: bf16_bits_to_f32(a) for n, a in host.items()}
    ref = attn_bf16(f["q"], f["k"], f["v"], cfg.scale, mask=f["mask"])
    assert np.allclose(got, ref, rtol=1e-2, atol=1e-2), f"max abs err {np.max(np.abs(got - ref))}"


@pytest.mark.gpu
@pytest.mark.parametrize("b,hq,g,s,d,causal", [(2, 8, 4, 256, 128, False), (1, 6, 3, 384, 64, True)])
def test_attention_grouped_query_bf16(runtime, b, hq, g, s, d, causal):
    """Grouped-query attention: query head h reads key / value head h // g (the
    repeat_interleave semantics of x_l_gqa), plain and causal."""
    from compiler.kernels.attention import AttnConfig
    from emmyrt.runner import bf16_bits_to_f32, f32_to_bf16_bits
    from oracle.refs import attn_bf16
    hk = hq // g
    cfg = AttnConfig(BH=b * hq, Sq=s, Sk=s, D=d, dtype="bf16", scale=1 / math.sqrt(d), causal=causal,
                     heads=hq, kv_group=g, name="k_attn_gqa", buffers=("q", "k", "v", "o"))
    rng = np.random.default_rng(7)
    host = {"q": f32_to_bf16_bits(rng.standard_normal((b * hq, s, d), dtype=np.float32)),
            "k": f32_to_bf16_bits(rng.standard_normal((b * hk, s, d), dtype=np.float32)),
            "v": f32_to_bf16_bits(rng.standard_normal((b * hk, s, d), dtype=np.float32))}
    got = _run_cfg(cfg, host)
    f = {n: bf16_bits_to_f32(a) for n, a in host.items()}
    kk = np.repeat(f["k"].reshape(b, hk, s, d), g, axis=1).reshape(b * hq, s, d)
    vv = np.repeat(f["v"].reshape(b, hk, s, d), g, axis=1).reshape(b * hq, s, d)
    ref = attn_bf16(f["q"], kk, vv, cfg.scale, causal=causal)
    assert np.allclose(got, ref, rtol=1e-2, atol=1e-2), f"max abs err {np.max(np.abs(got - ref))}"
