"""Element-map kernels: one output element per thread, short serial loops unrolled.

Emmy lowers the second half of a split-K matmul (``tests/problems/x_h_mm_rect``,
``x_h_bmm``, ``x_h_mm_bias``: ``k_matmul`` / ``k_add``) as a tile over the output
elements whose body sums the ``S`` partial slices in a serial ``Loop`` and applies the
rest of the graph (a rounding to the output dtype, a bias add) before the ``Write``.
The same shape covers elementwise kernels in general.  There is no cooperative axis,
no combine and no tensor-core work: the template maps the tile's elements onto a
grid-stride loop of threads, evaluates each ``Load`` index as an affine function of
the tile axes (serial loop variables are unrolled to constants), and lowers the IR's
scalar statements with per-op f16 / bf16 rounding where the IR types a result so.
"""

from __future__ import annotations

import math

from ..ptx import Ptx, entry, f32_hex, f64_hex, module
from ..stmts import ScalarCtx, Val, load_index_vars, lower_body, matmul_kernel
from .common import affine_offset, arg_params, load_pointer

ELEM = {"f32": 4, "f16": 2, "bf16": 2, "i32": 4, "i64": 8, "f64": 8}
KIND = {"i32": "s32", "i64": "s64", "f64": "f64"}        # value kinds of the wider buffer types
UNROLL = 8               # serial loops up to this many iterations are unrolled, longer ones loop
CTA = 256


class MapKernel:
    def __init__(self, spec):
        self.spec = spec
        if len(spec.body) != 1 or type(spec.body[0]).__name__ != "Tile":
            raise NotImplementedError("element map: body is not one Tile")
        tile = spec.body[0]
        if any(a.name.endswith("_co") for a in tile.axes):
            raise NotImplementedError("element map: cooperative axis")
        self.tile = tile
        self.axes = list(tile.axes)
        self.ext = {a.name: int(a.extent.value) for a in self.axes}   # + serial loop axes in scope
        self.n = math.prod(self.ext.values())
        self.writes = 0
        self._check(tile.body)
        if not self.writes:
            raise NotImplementedError("element map: the kernel writes nothing")

    def _check(self, body):
        for s in body:
            k = type(s).__name__
            if k == "Loop":
                self._check(s.body)
            elif k == "Cond":
                self._check(s.body)
                self._check(s.else_body or ())
            elif k == "Write":
                if s.atomic:
                    raise NotImplementedError("element map: atomic Write")
                self._buffer(s.output)
                self.writes += 1
            elif k == "Load":
                if s.input not in self.spec.constants:
                    self._buffer(s.input)
                elif len(s.names) != 1:
                    raise NotImplementedError("element map: multi-value constant Load")
            elif k not in ("Assign", "Let", "Init", "Accum", "Select"):
                raise NotImplementedError(f"element map: statement {k}")

    def _buffer(self, name):
        dt = self.spec.param(name).dtype
        if dt not in ELEM:
            raise NotImplementedError(f"element map: buffer {name} is {dt}")
        return dt

    # -- emission --------------------------------------------------------------
    def emit(self) -> str:
        spec = self.spec
        p = Ptx()
        p.comment(f"element map: {self.n} elements over {[a.name for a in self.axes]}")
        self.ptrs = {q.name: load_pointer(p, q.name) for q in spec.params if not q.scalar}
        # small maps (emmy's register tiles of a few hundred threads, long serial loops in
        # each) spread over every SM in CTAs of down to one warp; large ones 256 per CTA
        cta = CTA if self.n >= CTA * 148 else max(32, -(-self.n // (148 * 32)) * 32)
        self.cta = cta
        i, step = p.reg("u32"), p.reg("u32")
        p.emit(f"""
            mov.u32 {i}, %ctaid.x
            mov.u32 {step}, %tid.x
            mad.lo.u32 {i}, {i}, {cta}, {step}
            mov.u32 {step}, %nctaid.x
            mul.lo.u32 {step}, {step}, {cta}
        """)
        top, done = p.label("elem"), p.label("elem_done")
        p.place(top)
        pe = p.reg("pred")
        p.emit(f"setp.ge.u32 {pe}, {i}, {self.n}\n@{pe} bra {done}")
        # the tile axes of element i, row-major
        self.axis_reg = {}
        rem = i
        for a in reversed(self.axes):
            r = p.reg("u32")
            if a is self.axes[0]:
                p.emit(f"mov.u32 {r}, {rem}")
            else:
                q = p.reg("u32")
                p.emit(f"rem.u32 {r}, {rem}, {self.ext[a.name]}\ndiv.u32 {q}, {rem}, {self.ext[a.name]}")
                rem = q
            self.axis_reg[a.name] = r
        ctx = ScalarCtx(p, constants=dict(spec.constants), half_results=True,
                        exact_products=matmul_kernel(spec.name), index_vars=load_index_vars(spec.body),
                        const_dtypes={q.name: q.dtype for q in spec.params})
        ctx.on_load = self._load
        ctx.on_write = self._write
        self.fixed = {}
        self._lower(ctx, self.tile.body)
        p.emit(f"add.u32 {i}, {i}, {step}\nbra {top}")
        p.place(done)
        p.emit("ret")
        blocks = max(1, min(-(-self.n // cta), 148 * 8))
        launch = {"kind": "map", "grid": [blocks, 1, 1], "block": [cta, 1, 1], "cluster": [1, 1, 1],
                  "smem": 0, "extra_params": []}
        return module([entry(spec.name, arg_params(spec), p, maxntid=cta)], launch)

    def _lower(self, ctx, body):
        p = ctx.ptx
        for s in body:
            k = type(s).__name__
            if k == "Cond":
                # a guard over the element's indices (emmy's bounds checks on partial tiles):
                # each branch in its own scope, accumulators updated in place
                c, pc = self._index(p, s.cond), p.reg("pred")
                l_else, l_end = p.label("cond_else"), p.label("cond_end")
                p.emit(f"setp.ne.s32 {pc}, {c}, 0\n@!{pc} bra {l_else}")
                self._body_scope(ctx, s.body)
                p.emit(f"bra {l_end}")
                p.place(l_else)
                self._body_scope(ctx, s.else_body or ())
                p.place(l_end)
                continue
            if k == "Select":
                self._select(ctx, s)
                continue
            if k != "Loop":
                lower_body(ctx, [s])
                continue
            # a seeding loop starts the accumulators it folds into at their op's identity
            # every time it runs (the reference's _seed_accumulators, stmts.py:131-139)
            if s.seed:
                for st in s.body:
                    if type(st).__name__ == "Accum":
                        kind = KIND.get(getattr(st.dtype, "name", None), "f32")
                        if st.name in ctx.env and st.name in ctx.mutable:
                            r = ctx.env[st.name].text
                        else:
                            r = p.reg(kind)
                            ctx.env[st.name] = Val(r, kind)
                            ctx.mutable.add(st.name)
                        p.emit(f"mov.{'b64' if kind in ('s64', 'f64') else 'b32'} {r}, "
                               f"{_identity(kind, float(st.op.identity))}")
            ext, name = int(s.axis.extent.value), s.axis.name
            if ext <= UNROLL:
                for v in range(ext):
                    self.fixed[name] = v
                    self._body_scope(ctx, s.body)
                del self.fixed[name]
                continue
            # an innermost loop runs UNROLL copies of its body per trip (their loads issue
            # back to back instead of one load latency per element; accumulators still
            # update in the loop's order), then the remainder
            u = UNROLL if not _has_loop(s.body) else 1
            main = ext // u * u
            r, pl = p.reg("u32"), p.reg("pred")
            top = p.label("serial")
            p.emit(f"mov.u32 {r}, 0")
            self.ext[name] = ext

            def copies(n):
                for c in range(n):
                    rc = r
                    if c:
                        rc = p.reg("u32")
                        p.emit(f"add.u32 {rc}, {r}, {c}")
                    self.axis_reg[name] = rc
                    self._body_scope(ctx, s.body)
            if main:
                p.place(top)
                copies(u)
                p.emit(f"add.u32 {r}, {r}, {u}\nsetp.lt.u32 {pl}, {r}, {main}\n@{pl} bra {top}")
            copies(ext - main)
            del self.axis_reg[name], self.ext[name]

    def _select(self, ctx, s):
        """``v = a when c1, b when c2, ..., z when True``: the first branch whose index
        condition holds (emmy's concatenations, slices and triangular masks).  The values
        are computed before the Select, as the reference computes them; the conditions are
        over the element's indices and the serial loop variables."""
        p = ctx.ptx
        brs = list(s.branches)
        last = brs[-1].select
        if not (type(last).__name__ == "Literal" and bool(last.value)):
            raise NotImplementedError("element map: Select without a final default branch")
        kinds = {ctx.get(br.value).kind for br in brs}
        kind = next((k for k in ("f64", "f32", "s64", "s32") if k in kinds), "f32")
        b = "b64" if kind in ("f64", "s64") else "b32"
        out = p.reg(kind)
        p.emit(f"mov.{b} {out}, {ctx.as_kind(brs[-1].value, kind)}")
        for br in reversed(brs[:-1]):
            c, pc = self._index(p, br.select), p.reg("pred")
            p.emit(f"setp.ne.s32 {pc}, {c}, 0\nselp.{b} {out}, {ctx.as_kind(br.value, kind)}, {out}, {pc}")
        if s.name in ctx.mutable and s.name in ctx.env:
            p.emit(f"mov.{b} {ctx.env[s.name].text}, {out}")
        else:
            ctx.env[s.name] = Val(out, kind)

    def _body_scope(self, ctx, body):
        """Lower a loop body once; its element-local names do not outlive it, the
        accumulators it updates do."""
        saved = dict(ctx.env)
        self._lower(ctx, body)
        keep = {n: ctx.env[n] for n in ctx.mutable if n in ctx.env}
        ctx.env = saved
        ctx.env.update(keep)

    def _address(self, buffer: str, index) -> str:
        shape = self.spec.param(buffer).shape
        ptx = self._ptx
        off = ptx.reg("b64")
        try:
            aff = affine_offset(tuple(index), shape, dict(self.ext), fixed=dict(self.fixed))
        except NotImplementedError:
            aff = None
        if aff is not None:
            ptx.emit(f"mov.u64 {off}, {aff.const}")
            for var, c in aff.coef:
                w = ptx.reg("b64")
                ptx.emit(f"cvt.u64.u32 {w}, {self.axis_reg[var]}\nmad.lo.s64 {off}, {w}, {c}, {off}")
        else:
            # not affine (a grouped head a0 / 4, a clamp): each coordinate evaluated as
            # written, then the row-major offset
            if len(index) != len(shape):
                raise NotImplementedError("element map: index rank differs from the buffer's")
            ptx.emit(f"mov.u64 {off}, 0")
            for e, extent in zip(index, shape):
                v, w = self._index(ptx, e), ptx.reg("b64")
                ptx.emit(f"mul.lo.s64 {off}, {off}, {int(extent)}\ncvt.s64.s32 {w}, {v}\nadd.s64 {off}, {off}, {w}")
        addr = ptx.reg("b64")
        ptx.emit(f"mad.lo.s64 {addr}, {off}, {ELEM[self._buffer(buffer)]}, {self.ptrs[buffer]}")
        return addr

    _CMP = {"<": "lt", "<=": "le", ">": "gt", ">=": "ge", "==": "eq", "!=": "ne"}

    def _index(self, ptx, e) -> str:
        """An s32 index expression (C semantics for / and %, floor for //)."""
        k = type(e).__name__
        if k == "Literal":
            r = ptx.reg("s32")
            ptx.emit(f"mov.s32 {r}, {int(e.value)}")
            return r
        if k == "Var":
            if e.name in self.fixed:
                r = ptx.reg("s32")
                ptx.emit(f"mov.s32 {r}, {int(self.fixed[e.name])}")
                return r
            return self.axis_reg[e.name]
        if k == "TernaryExpr":
            c, a, b = self._index(ptx, e.cond), self._index(ptx, e.if_true), self._index(ptx, e.if_false)
            pc, r = ptx.reg("pred"), ptx.reg("s32")
            ptx.emit(f"setp.ne.s32 {pc}, {c}, 0\nselp.b32 {r}, {a}, {b}, {pc}")
            return r
        if k != "BinaryExpr":
            raise NotImplementedError(f"element map: index expression {k}")
        a, b, r = self._index(ptx, e.left), self._index(ptx, e.right), ptx.reg("s32")
        op = e.op
        if op in ("+", "-", "*"):
            ptx.emit(f"{ {'+': 'add', '-': 'sub', '*': 'mul.lo'}[op]}.s32 {r}, {a}, {b}")
        elif op == "/":
            ptx.emit(f"div.s32 {r}, {a}, {b}")
        elif op == "%":
            ptx.emit(f"rem.s32 {r}, {a}, {b}")
        elif op == "//":
            # floor: the truncated quotient, one less when the signs differ and it is inexact
            q, m, pn = ptx.reg("s32"), ptx.reg("s32"), ptx.reg("pred")
            ptx.emit(f"div.s32 {q}, {a}, {b}\nmul.lo.s32 {m}, {q}, {b}\nxor.b32 {r}, {a}, {b}\n"
                     f"setp.lt.s32 {pn}, {r}, 0\nsetp.ne.and.s32 {pn}, {m}, {a}, {pn}\n"
                     f"selp.s32 {r}, 1, 0, {pn}\nsub.s32 {r}, {q}, {r}")
        elif op in self._CMP:
            pc = ptx.reg("pred")
            ptx.emit(f"setp.{self._CMP[op]}.s32 {pc}, {a}, {b}\nselp.s32 {r}, 1, 0, {pc}")
        elif op in ("&&", "||"):
            pa, pb = ptx.reg("pred"), ptx.reg("pred")
            ptx.emit(f"setp.ne.s32 {pa}, {a}, 0\nsetp.ne.s32 {pb}, {b}, 0\n"
                     f"{'and' if op == '&&' else 'or'}.pred {pa}, {pa}, {pb}\nselp.s32 {r}, 1, 0, {pa}")
        else:
            raise NotImplementedError(f"element map: index operator {op}")
        return r

    def _load(self, ctx: ScalarCtx, s):
        """``names[k]`` of a multi-value Load is the element k after the index."""
        self._ptx = ctx.ptx
        dt = self._buffer(s.input)
        addr = self._address(s.input, s.index)
        for k, name in enumerate(s.names):
            off = k * ELEM[dt]
            if dt in KIND:
                r = ctx.ptx.reg(KIND[dt])
                ctx.ptx.emit(f"ld.global.{KIND[dt]} {r}, [{addr}+{off}]")
                ctx.env[name] = Val(r, KIND[dt])
                continue
            r = ctx.ptx.reg("f32")
            if dt == "f32":
                ctx.ptx.emit(f"ld.global.f32 {r}, [{addr}+{off}]")
            else:
                h = ctx.ptx.reg("b16")
                ctx.ptx.emit(f"ld.global.b16 {h}, [{addr}+{off}]\ncvt.f32.{dt} {r}, {h}")
            ctx.env[name] = Val(r, "f32")

    def _write(self, ctx: ScalarCtx, w):
        """``values[k]`` of a multi-value Write goes to the element k after the index."""
        self._ptx = ctx.ptx
        dt = self._buffer(w.output)
        addr = self._address(w.output, w.index)
        for k, name in enumerate(w.values):
            off = k * ELEM[dt]
            if dt in KIND:
                ctx.ptx.emit(f"st.global.{KIND[dt]} [{addr}+{off}], {ctx.as_kind(name, KIND[dt])}")
                continue
            v = ctx.f32(name)
            if dt == "f32":
                ctx.ptx.emit(f"st.global.f32 [{addr}+{off}], {v}")
            else:
                h = ctx.ptx.reg("b16")
                ctx.ptx.emit(f"cvt.rn.{dt}.f32 {h}, {v}\nst.global.b16 [{addr}+{off}], {h}")


def _has_loop(body) -> bool:
    for x in body:
        if type(x).__name__ in ("Loop", "StridedLoop"):
            return True
        for attr in ("body", "else_body"):
            sub = getattr(x, attr, None)
            if isinstance(sub, tuple) and _has_loop(sub):
                return True
    return False


def _identity(kind: str, v: float) -> str:
    """An accumulator's starting value in its register kind (the IR's f32 identities:
    0, 1, -1e30 for max, +1e30 for min; integers clamp them to their range)."""
    if kind == "f64":
        return f64_hex(v)
    if kind in ("s32", "s64"):
        lo, hi = (-(1 << 31), (1 << 31) - 1) if kind == "s32" else (-(1 << 63), (1 << 63) - 1)
        return str(int(min(max(v, lo), hi)))
    return f32_hex(v)


def serialize_cooperative(spec):
    """One thread per output instead of a cooperative tile: emmy's warp- and CTA-wide
    reductions (``Tile[.., a_co]`` with ``for a in a_co..N:W`` strided loops, a
    WarpShuffle / TreeHalve combine through shared memory and the result written by lane
    ``a_co == 0``) become serial loops over the whole axis, the combine statements go and
    the write guard opens.  Only the simple form is taken (every strided loop starts at
    the cooperative variable and steps by its width; nothing else reads it).  Used for
    the buffer types the streaming reduction template does not read (i32 / i64 / f64),
    whose kernels are small."""
    from dataclasses import replace
    from ..ir import IR_CLASSES
    from ..stmts import expr_vars
    if len(spec.body) != 1 or type(spec.body[0]).__name__ != "Tile":
        raise NotImplementedError("not a single-tile kernel")
    tile = spec.body[0]
    co = [a for a in tile.axes if a.name.endswith("_co")]
    if len(co) != 1:
        raise NotImplementedError("not one cooperative axis")
    cname, width = co[0].name, int(co[0].extent.value)

    def mentions(obj) -> bool:
        if type(obj).__name__ == "Var":
            return obj.name == cname
        if isinstance(obj, (tuple, list)):
            return any(mentions(x) for x in obj)
        if hasattr(obj, "__dataclass_fields__"):
            return any(mentions(getattr(obj, f)) for f in obj.__dataclass_fields__)
        return False

    def writes_global(stmts) -> bool:
        for x in stmts:
            if type(x).__name__ == "Write" and x.output in spec.buffers:
                return True
            for attr in ("body", "else_body"):
                sub = getattr(x, attr, None)
                if isinstance(sub, tuple) and writes_global(sub):
                    return True
        return False

    def conv(stmts) -> tuple:
        out = []
        for x in stmts:
            k = type(x).__name__
            if k in ("WarpShuffle", "TreeHalve", "Sync", "Smem"):
                continue
            if k == "Cond":
                cv = expr_vars(x.cond)
                if cv <= {"lane", "warp"} and not writes_global(x.body) and not writes_global(x.else_body or ()):
                    continue            # the shared-memory leg of the combine
                c = x.cond
                if type(c).__name__ == "BinaryExpr" and c.op == "==" and cv == {cname} and \
                        type(c.right).__name__ == "Literal" and int(c.right.value) == 0 and not x.else_body:
                    out.extend(conv(x.body))
                    continue
                if mentions(x.cond):
                    raise NotImplementedError("a condition on the cooperative lane")
                out.append(replace(x, body=conv(x.body), else_body=conv(x.else_body or ())))
                continue
            if k == "StridedLoop":
                st, sp = x.start, x.step
                if not (type(st).__name__ == "Var" and st.name == cname and type(sp).__name__ == "Literal"
                        and int(sp.value) == width) or mentions(x.body):
                    raise NotImplementedError("a strided loop other than the cooperative stride")
                out.append(IR_CLASSES["Loop"](axis=x.axis, body=conv(x.body), unroll=False, seed=x.seed))
                continue
            if k == "Loop":
                out.append(replace(x, body=conv(x.body)))
                continue
            if mentions(x):
                raise NotImplementedError(f"{k} reads the cooperative lane")
            out.append(x)
        return tuple(out)

    new_tile = replace(tile, axes=tuple(a for a in tile.axes if a.name != cname), body=conv(tile.body))
    return replace(spec, body=(new_tile,))


def emit_map(spec) -> str:
    return MapKernel(spec).emit()
