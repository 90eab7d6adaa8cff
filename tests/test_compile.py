"""Offline contract checks of compile.py (the reference's tests/check_local.py gate):
ASCII, .version first, the .entry name, one .param per arg_order entry (plus the
launch descriptor's extras), ptxas assembles for sm_100a, fast compile."""

import json
import subprocess
import sys
import time

import pytest

from compiler import compile_kernel, load, parse_launch
from compiler.ir import Graph, parse_stmt
from compiler.synth import baseline_dir

from conftest import GOLDEN, ROOT

IRS = sorted(GOLDEN.glob("*/*.ir.json"))


def _supported(path):
    try:
        return compile_kernel(load(path))
    except NotImplementedError:
        return None


@pytest.mark.parametrize("ir", IRS, ids=[f"{p.parent.name}/{p.stem}" for p in IRS])
def test_module_contract(ir):
    spec = load(ir)
    t0 = time.time()
    ptx = _supported(ir)
    if ptx is None:
        pytest.skip("family not supported yet")
    assert time.time() - t0 < 1.0
    ptx.encode("ascii")
    lines = [l.strip() for l in ptx.splitlines() if l.strip() and not l.strip().startswith("//")]
    assert lines[0] == ".version 8.8" and lines[1] == ".target sm_100a"
    assert f".visible .entry {spec.name}(" in ptx
    launch = parse_launch(ptx)
    sig = ptx.split(f".visible .entry {spec.name}(")[1].split(")")[0]
    nparams = sig.count(".param")
    assert nparams == len(spec.params) + len(launch.get("extra_params", []))
    # meta.json arg_order is the parameter order
    names = [l.split()[-1].rstrip(",") for l in sig.strip().splitlines()]
    for p, n in zip(spec.params, names):
        assert n.endswith(p.name.replace(".", "_"))


@pytest.mark.parametrize("ir", IRS, ids=[f"{p.parent.name}/{p.stem}" for p in IRS])
def test_ptxas_assembles(ir):
    ptx = _supported(ir)
    if ptx is None:
        pytest.skip("family not supported yet")
    from emmyrt import assemble
    cubin, log = assemble(ptx)
    assert len(cubin) > 0


def test_cli_contract(tmp_path):
    r = subprocess.run([sys.executable, str(ROOT / "compile.py")], capture_output=True, text=True)
    assert r.returncode == 2 and "compile.py" in r.stderr
    ir = next((GOLDEN / "f02_row_softmax").glob("*.ir.json"))
    r = subprocess.run([sys.executable, str(ROOT / "compile.py"), str(ir)], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.startswith(".version")


def test_unsupported_raises_not_implemented():
    # an f32 SIMT matmul (no tensor-core family) is rejected loudly, not lowered scalar
    from compiler.ir import parse_stmt
    body = (parse_stmt("Tile(axes=(Axis(name='a0', extent=Dim(4), window=None),), body=(), "
                       "block_threads=4, aux_threads=0, raster_axes=None, raster_group=None, "
                       "raster_orient='m')"),)
    from compiler.loader import KernelSpec
    spec = KernelSpec("k_x", body, (), None, None, {})
    with pytest.raises(NotImplementedError):
        compile_kernel(spec)


def test_loader_parses_all_fixture_statements():
    for ir in IRS:
        g = Graph.from_dict(json.loads(ir.read_text()))
        k = [n for n in g.nodes.values() if type(n.op).__name__ == "KernelOp"]
        assert len(k) == 1
        assert all(hasattr(s, "__dataclass_fields__") for s in k[0].op.body)


def test_reduce_identities():
    s = parse_stmt("Accum(name='a', value='v', op=ElementwiseImpl('maximum'), dtype=None, axes=(), base=None)")
    assert s.op.identity == -1e30


@pytest.mark.parametrize("name", ["rmsnorm", "softmax", "sum"])
def test_baseline_reductions_compile(name):
    d = baseline_dir(name)
    meta = json.loads((d / "meta.json").read_text())
    spec = load(d / f"{meta['kernels'][0]['entry']}.ir.json")
    ptx = compile_kernel(spec)
    from emmyrt import assemble
    assemble(ptx)


@pytest.mark.parametrize("pid,scale,kt,d", [("x_h_sdpa", 32 ** -0.5, False, 32), ("x_h_attn", 1 / 8, True, 64),
                                            ("x_h_attn_128", 1 / 8, True, 64)])
def test_attention_recognizer(pid, scale, kt, d):
    from compiler.kernels.attention import analyze
    cfg = analyze(load(next((GOLDEN / pid).glob("*.ir.json"))))
    assert abs(cfg.scale - scale) < 1e-12 and cfg.kt_layout == kt and cfg.D == d


@pytest.mark.parametrize("pid,kmajor", [("x_h_mm_1024", False), ("x_h_linear", True), ("x_h_mm_t_odd", True),
                                        ("x_h_bmm_t", True)])
def test_gemm_recognizer(pid, kmajor):
    from compiler.kernels.gemm import analyze
    cfg = analyze(load(next((GOLDEN / pid).glob("*.ir.json"))))
    assert cfg.b_kmajor == kmajor


@pytest.mark.parametrize("pid,scale,kt,causal", [("x_h_sdpa_causal", 32 ** -0.5, False, True),
                                                 ("x_h_attn_b", 1 / 5.66, True, False)])
def test_attention_recognizer_staged_and_causal(pid, scale, kt, causal):
    # operands staged through shared memory by cp.async are traced to their buffers;
    # where(__frow < __fcol, -1e30, s) is the causal mask, a uniform add is a shift
    from compiler.kernels.attention import analyze
    cfg = analyze(load(next((GOLDEN / pid).glob("*.ir.json"))))
    assert abs(cfg.scale - scale) < 1e-4 and cfg.kt_layout == kt and cfg.causal == causal


def test_simt_attention_recognizer():
    from compiler.kernels.attention import analyze_simt
    cfg = analyze_simt(load(next((GOLDEN / "x_h_sdpa_mask").glob("*.ir.json"))))
    assert (cfg.BH, cfg.Sq, cfg.Sk, cfg.D) == (2, 64, 64, 32)
    assert cfg.mask_param == "x3" and cfg.mask_bh_stride == 0 and abs(cfg.scale - 32 ** -0.5) < 1e-12
    assert (cfg.q_param, cfg.k_param, cfg.v_param) == ("x0", "x1", "x2")
    # no reduction fixture is taken for attention
    for ir in IRS:
        if ir.parent.name not in ("x_h_sdpa_mask", "x_h_attn_mask", "x_h_sdpa_mask_odd"):
            with pytest.raises(NotImplementedError):
                analyze_simt(load(ir))


F32_ATTN = {"a01_attention": (1, 64, 64, 64, 64, True), "a02_attention_128": (1, 128, 128, 32, 32, True),
            "x_a_256x64": (1, 256, 256, 64, 64, True), "x_a_32x16": (1, 32, 32, 16, 16, True),
            "x_a_batched": (4, 64, 64, 32, 32, True), "x_a_rect": (1, 64, 192, 32, 48, False),
            "x_l_gqa": (8, 64, 64, 32, 32, False)}


def test_f32_attention_recognizer():
    """The register-tiled f32 attention forms (q @ kt scaled by a 1-element buffer or its
    inverse) go to the warp-per-row template, and so does the online softmax over a score
    buffer of the split attention (its f16 rounding and f16 scale lowered from the IR);
    nothing else in the fixtures does."""
    from compiler.kernels.attention_f32 import analyze
    for ir in sorted(GOLDEN.glob("*/*.ir.json")):
        pid = ir.parent.name
        if pid == "x_h_attn_odd" and "softmax" in ir.name:
            cfg = analyze(load(ir))
            assert (cfg.scores, cfg.B, cfg.Sq, cfg.Sk, cfg.Dv) == ("matmul_1__place_03e2a34518_0", 1, 50, 70, 24)
            assert dict(cfg.dtypes) == {"v": "f16", "matmul_1": "f16"}
            assert [x.op.name for x in cfg.s_chain] == ["copy", "multiply"]
            assert parse_launch(compile_kernel(load(ir)))["kind"] == "attention_f32"
        elif pid in F32_ATTN:
            cfg = analyze(load(ir))
            b, sq, sk, d, dv, recip = F32_ATTN[pid]
            assert (cfg.B, cfg.Sq, cfg.Sk, cfg.D, cfg.Dv, cfg.scale_recip) == (b, sq, sk, d, dv, recip)
            if pid == "x_l_gqa":      # sdpa: key-major k, 4 query heads per k / v head
                assert (cfg.kt, cfg.group, cfg.k) == (False, 4, "x1")
            else:
                assert (cfg.q, cfg.k, cfg.v, cfg.kt, cfg.group) == ("q", "kt", "v", True, 1)
            assert cfg.scale_param is not None
            assert parse_launch(compile_kernel(load(ir)))["kind"] == "attention_f32"
        else:
            with pytest.raises(NotImplementedError):
                analyze(load(ir))


def test_f32_attention_rejects_score_transforms():
    """A softcap between the scaled score and the softmax (planted into a01's statements)
    is not computed by the template, so the recogniser must hand the kernel back."""
    from dataclasses import replace
    from compiler.kernels.attention_f32 import analyze
    spec = load(next((GOLDEN / "a01_attention").glob("*.ir.json")))

    def plant(body):
        out = []
        for x in body:
            if type(x).__name__ == "Assign" and x.name == "v4__gn__c0_0":
                out.append(parse_stmt("Assign(name='tc', op=ElementwiseImpl('tanh'), args=('v4__c0_0',), "
                                      "dtype=None)"))
                x = replace(x, args=("acc1__c0_0", "tc"))
            sub = getattr(x, "body", None)
            out.append(replace(x, body=plant(sub)) if isinstance(sub, tuple) else x)
        return tuple(out)
    with pytest.raises(NotImplementedError, match="tanh"):
        analyze(replace(spec, body=plant(spec.body)))


def test_f32_attention_rejects_rounded_p():
    """p rounded to f16 before it multiplies v (planted into a01's statements) is a step the
    template does not take, so the recogniser must hand the kernel back."""
    from dataclasses import replace
    from compiler.kernels.attention_f32 import analyze
    spec = load(next((GOLDEN / "a01_attention").glob("*.ir.json")))

    def plant(body):
        out = []
        for x in body:
            if type(x).__name__ == "Assign" and x.name == "v4__acc5__sum_sb__c0_0":
                out.append(parse_stmt("Assign(name='p16', op=ElementwiseImpl('copy'), "
                                      "args=('v4__beta__c0_0',), dtype=DataType(name='f16', "
                                      "np=dtype('float16'), nbytes=2))"))
                x = replace(x, args=(x.args[0], "p16"))
            sub = getattr(x, "body", None)
            out.append(replace(x, body=plant(sub)) if isinstance(sub, tuple) else x)
        return tuple(out)
    with pytest.raises(NotImplementedError, match="key sum"):
        analyze(replace(spec, body=plant(spec.body)))


def _odd_scores_spec():
    return load(next(p for p in (GOLDEN / "x_h_attn_odd").glob("*.ir.json") if "softmax" in p.name))


def _replant(body, fn):
    from dataclasses import replace
    out = []
    for x in body:
        for y in fn(x):
            sub = getattr(y, "body", None)
            out.append(replace(y, body=_replant(sub, fn)) if isinstance(sub, tuple) else y)
    return tuple(out)


def test_f32_attention_scores_reject_rounded_p():
    """x_h_attn_odd's online softmax over a score buffer with p rounded to f16 before it
    multiplies v (planted): the template multiplies the f32 p, so it must hand back."""
    from dataclasses import replace
    from compiler.kernels.attention_f32 import analyze
    spec = _odd_scores_spec()

    def fn(x):
        if type(x).__name__ == "Assign" and x.name == "v5__ws03e2a34518__acc5__sum_sb__c1_0":
            yield parse_stmt("Assign(name='p16', op=ElementwiseImpl('copy'), "
                             "args=('v5__ws03e2a34518__beta__c1_0',), dtype=DataType(name='f16', "
                             "np=dtype('float16'), nbytes=2))")
            yield replace(x, args=(x.args[0], "p16"))
        else:
            yield x
    with pytest.raises(NotImplementedError, match="key sum"):
        analyze(replace(spec, body=_replant(spec.body, fn)))


def test_f32_attention_scores_reject_a_copy_with_another_transform():
    """One register copy (row 2, column 1) scales its score twice (planted): the template
    lowers the first copy's transform for every row, so it must hand back."""
    from dataclasses import replace
    from compiler.kernels.attention_f32 import analyze
    spec = _odd_scores_spec()

    def fn(x):
        if type(x).__name__ == "Assign" and x.name == "v5__ws03e2a34518__c2_1":
            yield replace(x, name="tw", args=("v2", "v4__ws03e2a34518__c2_1"))
            yield replace(x, args=("v2", "tw"))
        else:
            yield x
    with pytest.raises(NotImplementedError, match="different score transforms"):
        analyze(replace(spec, body=_replant(spec.body, fn)))


@pytest.mark.parametrize("axis", [-2, -1])
def test_f32_attention_scores_reject_a_shifted_output(axis):
    """A Write one row (or one value column) away from its copy's score row / v column
    (planted) would be miscompiled by the template, so it must hand back."""
    from dataclasses import replace
    from compiler.kernels.attention_f32 import analyze
    spec = _odd_scores_spec()

    def fn(x):
        if type(x).__name__ == "Write" and x.values == ("acc5__c1_1",):
            idx = list(x.index)
            idx[axis] = parse_stmt(f"BinaryExpr(op='+', left={idx[axis]!r}, "
                                   "right=Literal(value=1, dtype='int'))")
            yield replace(x, index=tuple(idx))
        else:
            yield x
    with pytest.raises(NotImplementedError, match="written away"):
        analyze(replace(spec, body=_replant(spec.body, fn)))


def test_gemm_ksplit_choice():
    """K slices only where they remove many converter stages: the f32 512^3 matmul (64
    tiles, 16 K blocks) takes 2, the 64x64x2048 one (2 tiles) 16; 16-bit GEMMs none."""
    from compiler.synth import baseline_dir
    want = {"m01_matmul_512": 2, "x_m_longk": 16, "x_h_mm_256": 1, "m02_matmul_rect": 1}
    for pid, ks in want.items():
        ir = sorted((GOLDEN / pid).glob("*.ir.json"))[-1]
        assert parse_launch(compile_kernel(load(ir))).get("ksplit", 1) == ks, pid
    for name in ("gemm_512", "gemm_2048"):
        for ir in baseline_dir(name).glob("*.ir.json"):
            assert parse_launch(compile_kernel(load(ir)))["ksplit"] == 1


@pytest.mark.parametrize("pid,mnk,batch,a,b,epi", [
    ("m01_matmul_512", (512, 512, 512), 1, "x0", "x1", None),
    ("m02_matmul_rect", (128, 64, 256), 1, "x0", "x1", None),      # split-K atomics: one pass
    ("x_m_batched", (64, 48, 32), 4, "x0", "x1", None),
    ("x_m_bias_relu", (128, 96, 64), 1, "a", "b", ("add", "relu")),
    ("x_m_scaled", (64, 64, 128), 1, "x0", "x1", ("multiply",)),
])
def test_f32_matmul_recognizer(pid, mnk, batch, a, b, epi):
    # emmy's SIMT f32 matmul (operands staged by cp.async, FMA accumulators) goes to the
    # tcgen05 GEMM with 3xTF32 operands
    from compiler.kernels.gemm import analyze_f32
    cfg = analyze_f32(load(next((GOLDEN / pid).glob("*.ir.json"))))
    assert (cfg.M, cfg.N, cfg.K) == mnk and cfg.batch == batch and cfg.ab == "f32" and cfg.split3
    assert (cfg.a_param, cfg.b_param) == (a, b) and not cfg.b_kmajor and not cfg.pair
    if epi is None:
        assert cfg.epilogue == ()
    else:
        lam = cfg.epilogue[0][1]
        assert tuple(s.op.name for s in lam.body if type(s).__name__ == "Assign") == epi
    ptx = compile_kernel(load(next((GOLDEN / pid).glob("*.ir.json"))))
    assert "kind::tf32" in ptx and "cvt.rna.tf32.f32" in ptx


def test_f32_matmul_recognizer_rejects_other_kernels():
    from compiler.kernels.gemm import analyze_f32
    taken = set()
    for ir in IRS:
        try:
            analyze_f32(load(ir))
            taken.add(ir.parent.name)
        except NotImplementedError:
            pass
    # x_q_f16_mm_t / x_q_bf16_mm_t: operands cast to f16 / bf16, a warp-shuffle dot product
    # writing split-K partial slices
    assert taken == {"m01_matmul_512", "m02_matmul_rect", "x_m_small", "x_m_tall", "x_m_wide", "x_m_longk",
                     "x_m_256", "x_m_batched", "x_m_bias_relu", "x_m_scaled", "x_q_f16_mm_t", "x_q_bf16_mm_t",
                     "x_q_bf16_mm_odd", "x_h_mm_mixed", "x_m_odd", "x_d_f64_mm"}


def _synth_and_read(i):
    import json as _json
    from compiler.synth import baseline_dir
    for _ in range(5):
        d = baseline_dir("gemm_8192")
        _json.loads((d / "meta.json").read_text())
        for f in d.glob("*.ir.json"):
            _json.loads(f.read_text())
    return i


def test_baseline_problems_written_concurrently():
    # one process per GPU under torchrun synthesises the same BASELINE problem at once:
    # every reader must see whole files
    import multiprocessing as mp
    with mp.get_context("spawn").Pool(8) as pool:
        assert sorted(pool.map(_synth_and_read, range(8))) == list(range(8))


def test_compilation_is_deterministic():
    """The same IR compiles to the same PTX text in a fresh process (no dependence on hash
    seeds, set order or the order in which modules were compiled), so a module built here
    is the one the B200 runs and the judge can rebuild."""
    import os
    import random
    sample = [p for p in IRS if _supported(p) is not None]
    random.Random(3).shuffle(sample)
    sample = sample[:24]
    texts = {str(p): compile_kernel(load(p)) for p in sample}
    code = ("import sys, json; sys.path[:0] = [%r, %r]\n"
            "from compiler import compile_kernel, load\n"
            "paths = json.loads(sys.argv[1])\n"
            "print(json.dumps({p: compile_kernel(load(p)) for p in reversed(paths)}))"
            % (str(ROOT / "emmy-hackathon-2026_b200"), str(ROOT)))
    env = {**os.environ, "PYTHONHASHSEED": "12345"}
    r = subprocess.run([sys.executable, "-c", code, json.dumps(list(texts))], capture_output=True,
                       text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    again = json.loads(r.stdout)
    for p, t in texts.items():
        assert again[p] == t, f"{p}: PTX differs between runs"
