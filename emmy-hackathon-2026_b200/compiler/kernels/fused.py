"""Fused double matmuls of emmy's tensor-core form, lowered as element maps.

Two families of the reference's matmul IR chain or pair their contractions inside one
kernel (tests/problems/x_l_swiglu_h, tests/problems/x_h_mlp):

* a dual GEMM -- two accumulators share the A operand, ``C1 = A B1`` and ``C2 = A B2``,
  and the store's epilogue Lambda combines them (``silu(x W1) * (x W3)``);
* a chained GEMM -- the A tile of the second contraction is computed in the kernel from a
  first one (``relu(f16(x W1))`` written to shared memory, then ``H W2``).

Both are recognised from the statements (which buffers feed which accumulators, which
statements compute the stored values) and rewritten as one Tile over the output elements
whose serial loops do the same arithmetic: products of 16-bit values exact in f32 (the
MMA's), sums in f32, and the IR's own statements for the roundings and activations in
between.  The kernels are small; the element-map template runs them one output per
thread.
"""

from __future__ import annotations

from dataclasses import replace

from ..ir import parse_stmt
from .gemm import _walk

_DT = {"f32": "DataType(name='f32', np=dtype('float32'), nbytes=4)",
       "f16": "DataType(name='f16', np=dtype('float16'), nbytes=2)",
       "bf16": "DataType(name='bf16', np=dtype('uint16'), nbytes=2)"}


def _names(frag) -> tuple:
    return tuple(frag) if isinstance(frag, (tuple, list)) else (frag,)


def _sources(stmts, spec) -> dict:
    """Fragment name -> the global buffer its LdmatrixLoad reads (through cp.async)."""
    staged = {x.smem: x.src for x in stmts if type(x).__name__ == "CpAsyncCopy"}
    out = {}
    for x in stmts:
        if type(x).__name__ == "LdmatrixLoad":
            buf = staged.get(x.src_buffer, x.src_buffer)
            for f in _names(x.frag):
                out[f.split("[")[0]] = buf
    return out


def _tile(axes: list, body_text: str) -> object:
    ax = ", ".join(f"Axis(name='{n}', extent=Dim({e}), window=None)" for n, e in axes)
    return parse_stmt(f"Tile(axes=({ax},), body=({body_text},), block_threads=256, aux_threads=0, "
                      f"raster_axes=None, raster_group=None, raster_orient='m')")


def dual_gemm_spec(spec):
    """``out = f(A B1, A B2)``: the store's fragment and its extra fragments are the Lambda's
    parameters in order; each accumulates A times its own B."""
    stmts = list(_walk(spec.body))
    stores = [x for x in stmts if type(x).__name__ == "RegStore"]
    if len(stores) != 1 or not getattr(stores[0], "extra_frags", None) or stores[0].epilogue is None:
        raise NotImplementedError("not a dual GEMM")
    st = stores[0]
    lam = st.epilogue
    frags = (st.frag,) + tuple(st.extra_frags)
    if len(lam.params) != len(frags):
        raise NotImplementedError("epilogue parameters and fragments differ")
    src = _sources(stmts, spec)
    mmas = [x for x in stmts if type(x).__name__ == "MmaSyncPtx"]
    b_of, a_bufs = {}, set()
    for m in mmas:
        c = m.c_frag.split("[")[0]
        a_bufs.add(src.get(m.a_frag.split("[")[0]))
        b_of.setdefault(c, set()).add(src.get(m.b_frag.split("[")[0]))
    if len(a_bufs) != 1 or None in a_bufs or any(len(v) != 1 or None in v for v in b_of.values()):
        raise NotImplementedError("dual GEMM operands not traced")
    A = spec.param(next(iter(a_bufs)))
    Bs = []
    for f in frags:
        bset = b_of.get(f.split("[")[0])
        if not bset:
            raise NotImplementedError(f"no MMA accumulates into {f}")
        Bs.append(spec.param(next(iter(bset))))
    O = spec.param(st.dst_buffer)
    if len(A.shape) != 2 or any(tuple(B.shape) != (A.shape[1], O.shape[1]) for B in Bs) or \
            tuple(O.shape) != (A.shape[0], Bs[0].shape[1]) or O.dtype not in _DT:
        raise NotImplementedError("dual GEMM shapes")
    M, K, N = A.shape[0], A.shape[1], O.shape[1]
    f32 = _DT["f32"]
    loop = [f"Load(names=('_a',), input='{A.name}', index=(Var(name='i'), Var(name='k')), dtype=None)"]
    for pname, B in zip(lam.params, Bs):
        loop += [f"Load(names=('_b_{pname}',), input='{B.name}', index=(Var(name='k'), Var(name='n')), dtype=None)",
                 f"Assign(name='_p_{pname}', op=ElementwiseImpl('multiply'), args=('_a', '_b_{pname}'), dtype={f32})",
                 f"Accum(name='{pname}', value='_p_{pname}', op=ElementwiseImpl('add'), dtype={f32}, "
                 f"axes=('k',), base=None)"]
    kloop = (f"Loop(axis=Axis(name='k', extent=Dim({K}), window=None), body=({', '.join(loop)},), "
             f"unroll=False, seed=True)")
    write = (f"Write(output='{O.name}', index=(Var(name='i'), Var(name='n')), values=('{lam.results[0]}',), "
             f"value_dtype={_DT[O.dtype]}, atomic=False, swizzle='NONE')")
    tile = _tile([("i", M), ("n", N)], kloop)
    write_stmt = parse_stmt(write)
    tile = replace(tile, body=tile.body + tuple(lam.body) + (write_stmt,))
    return replace(spec, body=(tile,))


def chained_gemm_spec(spec):
    """``out = g(H) W2`` with ``H = f(x W1)`` computed in the kernel: the shared A tile of
    the MMAs is written from values computed from a dot product of two global buffers.  The
    first written value's statements (back to its accumulator) are the per-element f."""
    X, W1, W2, O, a0, chain, hname = chained_parts(spec)
    M, K1 = X.shape
    J, N = W1.shape[1], W2.shape[1]
    f32 = _DT["f32"]
    inner = (f"Loop(axis=Axis(name='k', extent=Dim({K1}), window=None), body=("
             f"Load(names=('_x',), input='{X.name}', index=(Var(name='i'), Var(name='k')), dtype=None), "
             f"Load(names=('_w1',), input='{W1.name}', index=(Var(name='k'), Var(name='j')), dtype=None), "
             f"Assign(name='_p1', op=ElementwiseImpl('multiply'), args=('_x', '_w1'), dtype={f32}), "
             f"Accum(name='{a0}', value='_p1', op=ElementwiseImpl('add'), dtype={f32}, axes=('k',), "
             f"base=None)), unroll=False, seed=True)")
    tail = (f"Load(names=('_w2',), input='{W2.name}', index=(Var(name='j'), Var(name='n')), dtype=None), "
            f"Assign(name='_p2', op=ElementwiseImpl('multiply'), args=('{hname}', '_w2'), dtype={f32}), "
            f"Accum(name='_acc2', value='_p2', op=ElementwiseImpl('add'), dtype={f32}, axes=('j',), base=None)")
    outer = parse_stmt(f"Loop(axis=Axis(name='j', extent=Dim({J}), window=None), body=({inner}, {tail}), "
                       f"unroll=False, seed=True)")
    # H's own statements (16-bit rounding, the activation) between the two contractions
    outer = replace(outer, body=(outer.body[0],) + tuple(chain) + outer.body[1:])
    tile = _tile([("i", M), ("n", N)], "Let(name='_unused', value=Literal(value=0, dtype='int'), dtype=None)")
    write = parse_stmt(f"Write(output='{O.name}', index=(Var(name='i'), Var(name='n')), values=('_acc2',), "
                       f"value_dtype={_DT[O.dtype]}, atomic=False, swizzle='NONE')")
    tile = replace(tile, body=(outer, write))
    return replace(spec, body=(tile,))


def chained_parts(spec):
    """(x, W1, W2, out, H's accumulator name, H's statements in program order, H's name)
    of a chained GEMM; NotImplementedError for anything else."""
    stmts = list(_walk(spec.body))
    src = _sources(stmts, spec)
    mmas = [x for x in stmts if type(x).__name__ == "MmaSyncPtx"]
    a_smem = {x.src_buffer for x in stmts if type(x).__name__ == "LdmatrixLoad" and x.role == "a"}
    if len(a_smem) != 1:
        raise NotImplementedError("not a chained GEMM")
    a_smem = next(iter(a_smem))
    writes = [x for x in stmts if type(x).__name__ == "Write" and x.output == a_smem]
    if not writes:
        raise NotImplementedError("the A tile is not computed in the kernel")
    defs, order = {}, {id(x): i for i, x in enumerate(stmts)}
    for x in stmts:
        k = type(x).__name__
        if k == "Load":
            for n in x.names:
                defs[n] = x
        elif k == "Assign":
            defs[x.name] = x
    accs = {x.name: x for x in stmts if type(x).__name__ == "Accum"}
    # the computed value of H and its chain back to one accumulator
    chain, seen, acc = [], set(), []

    def visit(n):
        if n in accs:
            acc.append(n)
            return
        d = defs.get(n)
        if d is None or type(d).__name__ != "Assign" or id(d) in seen:
            if d is None:
                raise NotImplementedError(f"{n} not traced")
            return
        seen.add(id(d))
        for x in d.args:
            visit(x)
        chain.append(d)
    visit(writes[0].values[0])
    if len(set(acc)) != 1:
        raise NotImplementedError("H not computed from one dot product")
    a0 = accs[acc[0]]
    prod = defs.get(a0.value)
    if prod is None or type(prod).__name__ != "Assign" or prod.op.name != "multiply":
        raise NotImplementedError("H's accumulator is not a dot product")
    lx = [defs.get(x) for x in prod.args]
    if any(d is None or type(d).__name__ != "Load" for d in lx):
        raise NotImplementedError("H's dot product does not read two buffers")
    # which loaded operand is x (indexed by the H row) and which W1 (by the H column):
    # x's last index is the contraction variable
    kv = set(a0.axes or ())
    from ..stmts import expr_vars
    xs = [d for d in lx if expr_vars(d.index[-1]) & kv]
    ws = [d for d in lx if expr_vars(d.index[0]) & kv]
    if len(xs) != 1 or len(ws) != 1 or xs[0] is ws[0]:
        raise NotImplementedError("H's operands not identified")
    X, W1 = spec.param(xs[0].input), spec.param(ws[0].input)
    b_bufs = {src.get(m.b_frag.split("[")[0]) for m in mmas}
    stores = {x.dst_buffer for x in stmts if type(x).__name__ == "RegStore"}
    if len(b_bufs) != 1 or None in b_bufs or len(stores) != 1:
        raise NotImplementedError("second GEMM operands not traced")
    W2, O = spec.param(next(iter(b_bufs))), spec.param(next(iter(stores)))
    st = next(x for x in stmts if type(x).__name__ == "RegStore")
    if st.epilogue is not None and any(type(x).__name__ != "Assign" or x.op.name != "copy" for x in st.epilogue.body):
        raise NotImplementedError("an epilogue on the chained GEMM")
    M, K1 = X.shape
    if tuple(W1.shape[:1]) != (K1,) or len(W1.shape) != 2 or W2.shape[0] != W1.shape[1] or \
            tuple(O.shape) != (M, W2.shape[1]) or O.dtype not in _DT:
        raise NotImplementedError("chained GEMM shapes")
    chain = sorted(chain, key=lambda d: order[id(d)])
    return X, W1, W2, O, a0.name, chain, writes[0].values[0]


ROW_THREADS = 256
_LD_BATCH = 16


def emit_chained_rows(spec) -> str:
    """The chained GEMM ``out = g(f(x W1)) W2`` as one CTA per output row: x's row is staged
    in shared memory; thread j computes ``H[j] = f(x_row . W1[:, j])`` (W1 read along its
    rows, coalesced across the threads) with the IR's own statements for f (16-bit rounding,
    the activation) and writes it to shared memory; after one barrier thread n computes
    ``out[n] = H . W2[:, n]``.  Each H row is computed once instead of once per output
    element.  Products of 16-bit values are exact in f32 (the MMA's), sums in f32 in index
    order; loads issue 16 deep.  Contractions are unrolled in full, so K and J are capped
    (larger chains stay element maps)."""
    from ..ptx import Ptx, entry, module
    from ..stmts import ScalarCtx, Val, load_index_vars, lower_body, matmul_kernel
    from .common import arg_params, load_pointer
    X, W1, W2, O, a0, chain, hname = chained_parts(spec)
    M, K = X.shape
    J, N = W1.shape[1], W2.shape[1]
    if K > 1024 or J > 1024 or any(b.dtype not in _DT for b in (X, W1, W2)):
        raise NotImplementedError("chained GEMM: contraction above 1024 or operand type")
    T = ROW_THREADS
    p = Ptx()
    p.comment(f"chained GEMM {M}x{K} . {K}x{J} -> f -> . {J}x{N}, one CTA per row")
    ptr = {b.name: load_pointer(p, b.name) for b in (X, W1, W2, O)}
    row, tid = p.reg("u32"), p.reg("u32")
    xs, hs = p.reg("u32"), p.reg("u32")
    p.emit(f"mov.u32 {row}, %ctaid.x\nmov.u32 {tid}, %tid.x\nmov.u32 {xs}, chain_xs\nmov.u32 {hs}, chain_hs")

    def load(buf, addr, dst):
        if buf.dtype == "f32":
            p.emit(f"ld.global.nc.f32 {dst}, [{addr}]")
        else:
            h = p.reg("b16")
            p.emit(f"ld.global.nc.b16 {h}, [{addr}]\ncvt.f32.{buf.dtype} {dst}, {h}")

    def eb(buf):
        return 4 if buf.dtype == "f32" else 2

    # x's row -> shared (f32)
    for it in range(-(-K // T)):
        k, pk, a = p.reg("u32"), p.reg("pred"), p.reg("b64")
        v = p.reg("f32")
        skip = p.label("xs_skip")
        p.emit(f"add.u32 {k}, {tid}, {it * T}\nsetp.ge.u32 {pk}, {k}, {K}\n@{pk} bra {skip}")
        p.emit(f"mad.lo.u32 {k}, {row}, {K}, {k}\nmul.wide.u32 {a}, {k}, {eb(X)}\nadd.s64 {a}, {ptr[X.name]}, {a}")
        load(X, a, v)
        sa = p.reg("u32")
        p.emit(f"add.u32 {sa}, {tid}, {it * T}\nshl.b32 {sa}, {sa}, 2\nadd.u32 {sa}, {sa}, {xs}\nst.shared.f32 [{sa}], {v}")
        p.place(skip)
    p.emit("bar.sync 0")

    def dot(n_terms, lhs_smem, col_reg, buf, ncols):
        """sum_t lhs[t] * buf[t, col] over t < n_terms, loads 16 deep; returns the f32 sum."""
        acc = p.reg("f32")
        p.emit(f"mov.f32 {acc}, 0f00000000")
        base = p.reg("b64")
        p.emit(f"mul.wide.u32 {base}, {col_reg}, {eb(buf)}\nadd.s64 {base}, {ptr[buf.name]}, {base}")
        for t0 in range(0, n_terms, _LD_BATCH):
            ts = range(t0, min(n_terms, t0 + _LD_BATCH))
            vals = {}
            for t in ts:
                vals[t] = p.reg("f32")
                load(buf, f"{base}+{t * ncols * eb(buf)}", vals[t])
            for t in ts:
                lv = p.reg("f32")
                p.emit(f"ld.shared.f32 {lv}, [{lhs_smem}+{4 * t}]\nfma.rn.f32 {acc}, {lv}, {vals[t]}, {acc}")
        return acc

    ctx = ScalarCtx(p, constants=dict(spec.constants), half_results=True,
                    exact_products=matmul_kernel(spec.name), index_vars=load_index_vars(spec.body),
                    const_dtypes={q.name: q.dtype for q in spec.params})
    for it in range(-(-J // T)):
        j, pj = p.reg("u32"), p.reg("pred")
        skip = p.label("h_skip")
        p.emit(f"add.u32 {j}, {tid}, {it * T}\nsetp.ge.u32 {pj}, {j}, {J}\n@{pj} bra {skip}")
        acc = dot(K, xs, j, W1, J)
        saved = dict(ctx.env)
        ctx.env[a0] = Val(acc, "f32")
        try:
            lower_body(ctx, chain)
            h = ctx.f32(hname)
        except ValueError as err:      # H's statements read something other than the dot product
            raise NotImplementedError(f"chained GEMM: {err}") from None
        ctx.env = saved
        sa = p.reg("u32")
        p.emit(f"shl.b32 {sa}, {j}, 2\nadd.u32 {sa}, {sa}, {hs}\nst.shared.f32 [{sa}], {h}")
        p.place(skip)
    p.emit("bar.sync 0")
    for it in range(-(-N // T)):
        n, pn = p.reg("u32"), p.reg("pred")
        skip = p.label("o_skip")
        p.emit(f"add.u32 {n}, {tid}, {it * T}\nsetp.ge.u32 {pn}, {n}, {N}\n@{pn} bra {skip}")
        acc = dot(J, hs, n, W2, N)
        a, off = p.reg("b64"), p.reg("u32")
        p.emit(f"mad.lo.u32 {off}, {row}, {N}, {n}\nmul.wide.u32 {a}, {off}, {eb(O)}\nadd.s64 {a}, {ptr[O.name]}, {a}")
        if O.dtype == "f32":
            p.emit(f"st.global.f32 [{a}], {acc}")
        else:
            h = p.reg("b16")
            p.emit(f"cvt.rn.{O.dtype}.f32 {h}, {acc}\nst.global.b16 [{a}], {h}")
        p.place(skip)
    p.emit("ret")
    launch = {"kind": "chained_rows", "grid": [M, 1, 1], "block": [T, 1, 1], "cluster": [1, 1, 1],
              "smem": 0, "extra_params": [], "flops": 2 * M * J * (K + N)}
    return module([entry(spec.name, arg_params(spec), p, maxntid=T)], launch,
                  globals_=[f".shared .align 16 .f32 chain_xs[{K}];", f".shared .align 16 .f32 chain_hs[{J}];"])
