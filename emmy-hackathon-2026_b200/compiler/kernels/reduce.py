"""Row and global reductions as 128-bit HBM streams (no tensor cores).

Covers the reference's cooperative-reduction family (TASK.md categories 2 and 4):
row sums / means / max, RMSNorm, L2 norm, row softmax (``problems/f01_rmsnorm``,
``f02_row_softmax``, ``f03_l2norm``, ``r04_row_sum``, ``tests/problems/x_l_rmsnorm_w``,
``x_r_rowmax`` ...) and whole-array sums / means (``r01``-``r03``,
``tests/problems/x_r_unpinned_sum``).

Emmy's IR for these is one ``Tile`` over the rows plus a cooperative ``*_co`` axis of
``block_threads`` lanes; ``StridedLoop``\\ s stride that axis through a row, a
``WarpShuffle`` / ``Smem`` / ``Sync`` / ``TreeHalve`` group combines the per-lane
accumulators, a scalar tail finishes the row (``rsqrt``, ``reciprocal`` ...), and a
second ``StridedLoop`` (or a ``Cond(co == 0)`` leader section) writes the result.
Under emmy's schedule each thread makes scalar loads 128 threads apart, and the
second pass re-reads the row from memory.

The sm_100a schedule here keeps the IR's arithmetic and changes the movement:

* each thread owns ``VEC``-wide (128-bit) column chunks ``TPR * VEC`` apart, so a
  warp issues fully coalesced ``ld.global.v4.f32``; every load of a pass is issued
  before any arithmetic (``NCH`` loads in flight per thread);
* values a later pass loads again at the same address stay in registers, so the
  row crosses HBM once (RMSNorm and softmax read ``x`` once, write ``y`` once);
* the per-thread accumulators are combined with the IR's own ``combine_states``
  first by a ``shfl.sync.bfly`` butterfly and then, for rows wider than a warp,
  through shared memory in a fixed order (every thread ends with the row result);
* whole-array reductions stream with a grid-stride loop, fold 8-element f32 groups
  into an f64 per-thread accumulator, write one f64 partial per CTA to scratch,
  and the last CTA to arrive (an ``atom.add`` ticket) sums the partials with all its
  threads in a fixed order (each thread its strided share in CTA order, then the warp
  butterfly and the warp fold), runs the IR's leader section (e.g. ``/ count``) and
  stores the result -- deterministic, with 64-bit addressing for 2^31 elements.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

from ..ptx import Ptx, entry, f32_hex, f64_hex, module
from ..stmts import (ScalarCtx, Val, emit_exp_nonpos, expr_vars, load_index_vars,
                     lower_body, matmul_kernel)
from .common import Affine, affine_offset, arg_params, load_pointer

SMS = 148          # B200 multiprocessors (grid sizing for the streaming reduction)


class NotThisTemplate(Exception):
    """The kernel is not in this template's family (try the next template)."""


# ---------------------------------------------------------------------------
# structure parsing


@dataclass
class Combine:
    state: tuple
    state_b: tuple
    combine_states: tuple


@dataclass
class Phase:
    kind: str                 # "stream" | "combine" | "scalar" | "leader"
    stmt: object = None
    combine: Combine | None = None


def _is_var(e, name):
    return type(e).__name__ == "Var" and e.name == name


def _is_eq_zero(cond, name):
    return (type(cond).__name__ == "BinaryExpr" and cond.op == "==" and _is_var(cond.left, name)
            and type(cond.right).__name__ == "Literal" and int(cond.right.value) == 0)


def parse_cooperative(spec):
    """Split a cooperative-reduction Tile into phases; NotThisTemplate otherwise."""
    if len(spec.body) != 1 or type(spec.body[0]).__name__ != "Tile":
        raise NotThisTemplate("body is not one Tile")
    tile = spec.body[0]
    co = [a for a in tile.axes if a.name.endswith("_co")]
    if len(co) != 1:
        raise NotThisTemplate("no cooperative axis")
    co = co[0]
    kinds = {type(s).__name__ for s in tile.body}
    if "WarpShuffle" not in kinds or kinds & {"RegFragment", "MmaSyncPtx"}:
        raise NotThisTemplate("no cross-thread combine")
    row_len = {int(s.axis.extent.value) for s in tile.body if type(s).__name__ == "StridedLoop"}
    others = [a for a in tile.axes if a is not co]
    phases: list[Phase] = []
    body = list(tile.body)
    i = 0
    while i < len(body):
        s = body[i]
        k = type(s).__name__
        if k == "StridedLoop":
            if not _is_var(s.start, co.name):
                raise NotImplementedError("StridedLoop does not start at the cooperative lane")
            if int(s.step.value) != int(co.extent.value):
                raise NotImplementedError("StridedLoop step differs from the cooperative width")
            if s.end is not None:
                raise NotImplementedError("StridedLoop with an explicit end")
            phases.append(Phase("stream", s))
            i += 1
        elif k == "WarpShuffle":
            comb = Combine(tuple(s.state), tuple(s.state_b), tuple(s.combine_states))
            j = i + 1
            # emmy's cross-warp tail: Smem..., Cond(lane==0){smem[warp] = state}, Sync, TreeHalve
            while j < len(body) and type(body[j]).__name__ in ("Smem", "Sync", "Cond", "TreeHalve"):
                t = body[j]
                tk = type(t).__name__
                if tk == "Cond":
                    if not _is_eq_zero(t.cond, "lane"):
                        break
                    if any(type(w).__name__ != "Write" for w in t.body) or t.else_body:
                        raise NotImplementedError("unexpected statements in the lane-0 smem store")
                elif tk == "TreeHalve":
                    if tuple(t.state) != comb.state:
                        raise NotImplementedError("TreeHalve combines other states than the WarpShuffle")
                    j += 1
                    break
                j += 1
            phases.append(Phase("combine", combine=comb))
            i = j
        elif k == "Cond":
            if not _is_eq_zero(s.cond, co.name) or s.else_body:
                raise NotImplementedError("Cond other than the cooperative leader section")
            phases.append(Phase("leader", s))
            i += 1
        elif k in ("Assign", "Let", "Load", "Init"):
            phases.append(Phase("scalar", s))
            i += 1
        elif k == "Loop" and int(s.axis.extent.value) in row_len:
            # a reduction every lane runs over the whole row (emmy's serial variance
            # loop in LayerNorm): the same sum as a strided stream plus a combine
            phases.extend(_serial_to_stream(s, co))
            i += 1
        else:
            raise NotImplementedError(f"statement {k} in a cooperative reduction")
    return tile, co, others, phases


def _serial_to_stream(loop, co) -> list:
    """``for c in 0..L: acc <- op(acc, f(row[c]))`` run by every lane ->
    ``for c in co..L:W`` per lane + a cross-lane combine of the accumulators with
    the same op.  Only Load / Assign / Let / Accum (add, maximum, minimum) bodies."""
    from ..ir import IR_CLASSES as C
    accs = []
    for st in loop.body:
        k = type(st).__name__
        if k == "Accum":
            if st.op.name not in ("add", "maximum", "minimum") or st.base is not None:
                raise NotImplementedError(f"serial row loop accumulating with {st.op.name}")
            accs.append(st)
        elif k not in ("Load", "Assign", "Let"):
            raise NotImplementedError(f"{k} inside a serial row loop")
    if not accs:
        raise NotImplementedError("serial row loop without an accumulator")
    width = int(co.extent.value)
    stream = C["StridedLoop"](axis=loop.axis, start=C["Var"](name=co.name),
                              step=C["Literal"](value=width, dtype="int"), body=loop.body,
                              unroll=False, end=None, seed=True)
    names = tuple(a.name for a in accs)
    others = tuple(f"{n}__o" for n in names)
    comb = tuple(C["Assign"](name=a.name, op=a.op, args=(a.name, f"{a.name}__o"), dtype=a.dtype)
                 for a in accs)
    return [Phase("stream", stream), Phase("combine", combine=Combine(names, others, comb))]


def _zero_var(expr, name: str):
    """Substitute Literal(0) for Var(name) in an index expression."""
    from ..ir import IR_CLASSES as C
    k = type(expr).__name__
    if k == "Var":
        return C["Literal"](value=0, dtype="int") if expr.name == name else expr
    if k == "BinaryExpr":
        return type(expr)(op=expr.op, left=_zero_var(expr.left, name), right=_zero_var(expr.right, name))
    if k == "TernaryExpr":
        return type(expr)(cond=_zero_var(expr.cond, name), if_true=_zero_var(expr.if_true, name),
                          if_false=_zero_var(expr.if_false, name))
    return expr


def _mentions(obj, name: str) -> bool:
    """Does any index expression inside ``obj`` (a statement or expression) use Var(name)?"""
    if type(obj).__name__ == "Var":
        return obj.name == name
    if isinstance(obj, (tuple, list)):
        return any(_mentions(x, name) for x in obj)
    if hasattr(obj, "__dataclass_fields__"):
        return any(_mentions(getattr(obj, f), name) for f in obj.__dataclass_fields__)
    return False


def fold_ksplit(spec, others, phases):
    """Emmy's split rows (``Tile[_ksplit, rows.., co]``: each of S CTAs sums a C-wide
    slice ``x[row, c + _ksplit * C]`` and adds it to the output atomically) as whole
    rows: one stream over c in [0, S * C) with the same per-row combine and one
    atomic add per row.  Checked on every access: the split offset must be exactly
    C times the column stride."""
    from ..ir import IR_CLASSES as C, Dim
    ks = next(a for a in others if a.name == "_ksplit")
    S = int(ks.extent.value)
    rows = [a for a in others if a is not ks]
    if not rows:
        raise NotThisTemplate("split whole-array reduction")
    ranges = {a.name: int(a.extent.value) for a in others}
    out = []
    for ph in phases:
        if ph.kind != "stream":
            if _mentions(ph.stmt, "_ksplit") or (ph.combine and _mentions(ph.combine, "_ksplit")):
                raise NotImplementedError("_ksplit used outside the row streams")
            out.append(ph)
            continue
        loop = ph.stmt
        L = int(loop.axis.extent.value)
        body = []
        for st in loop.body:
            k = type(st).__name__
            if k in ("Load", "Write") and _mentions(st.index, "_ksplit"):
                buf = st.input if k == "Load" else st.output
                aff = affine_offset(tuple(st.index), spec.param(buf).shape,
                                    {**ranges, loop.axis.name: L})
                cf = dict(aff.coef)
                if cf.get("_ksplit", 0) != L * cf.get(loop.axis.name, 0) or not cf.get(loop.axis.name):
                    raise NotImplementedError("split offset is not a whole slice of the row")
                st = type(st)(**{fn: (tuple(_zero_var(e, "_ksplit") for e in st.index)
                                      if fn == "index" else getattr(st, fn))
                                 for fn in st.__dataclass_fields__})
            elif _mentions(st, "_ksplit"):
                raise NotImplementedError("_ksplit used in a stream statement other than an access")
            body.append(st)
        axis = C["Axis"](name=loop.axis.name, extent=Dim(value=S * L), window=loop.axis.window)
        out.append(Phase("stream", type(loop)(axis=axis, start=loop.start, step=loop.step, body=tuple(body),
                                              unroll=loop.unroll, end=loop.end, seed=loop.seed)))
    return rows, out


def _stream_loads(stmts):
    return [s for s in stmts if type(s).__name__ == "Load"]


def _accums(stmts):
    out = []
    for s in stmts:
        if type(s).__name__ == "Accum":
            out.append(s)
    return out


ESZ = {"f32": 4, "f16": 2, "bf16": 2}


def _check_buffer(spec, name):
    """The buffer's IR dtype: f32, or f16 / bf16 (widened to f32 on load, rounded on
    store; the arithmetic stays f32 with the IR's per-op 16-bit roundings)."""
    p = spec.param(name)
    if p.dtype not in ESZ:
        raise NotImplementedError(f"buffer {name} is {p.dtype}; reductions read f32, f16 or bf16")
    return p.dtype


def ld_vec(p, dt: str, regs: list, addr: str, guard: str = "", cache: str = "") -> None:
    """Load len(regs) consecutive elements of type ``dt`` at [addr] into f32 registers."""
    n = len(regs)
    if dt == "f32":
        if n == 1:
            p.emit(f"{guard}ld.global{cache}.f32 {regs[0]}, [{addr}]")
        else:
            p.emit(f"{guard}ld.global{cache}.v{n}.f32 {{{', '.join(regs)}}}, [{addr}]")
        return
    if n == 1:
        h = p.reg("b16")
        p.emit(f"{guard}ld.global{cache}.b16 {h}, [{addr}]\ncvt.f32.{dt} {regs[0]}, {h}")
        return
    words = [p.reg("b32") for _ in range(n // 2)]
    vec = f".v{len(words)}" if len(words) > 1 else ""
    p.emit(f"{guard}ld.global{cache}{vec}.b32 {{{', '.join(words)}}}, [{addr}]" if vec else
           f"{guard}ld.global{cache}.b32 {words[0]}, [{addr}]")
    for i, w in enumerate(words):
        lo, hi = p.reg("b16"), p.reg("b16")
        # the lower address holds the first element
        p.emit(f"mov.b32 {{{lo}, {hi}}}, {w}\ncvt.f32.{dt} {regs[2 * i]}, {lo}\n"
               f"cvt.f32.{dt} {regs[2 * i + 1]}, {hi}")


def st_vec(p, dt: str, vals: list, addr: str, guard: str = "") -> None:
    """Store len(vals) f32 values as consecutive elements of type ``dt`` at [addr]."""
    n = len(vals)
    if dt == "f32":
        if n == 1:
            p.emit(f"{guard}st.global.f32 [{addr}], {vals[0]}")
        else:
            p.emit(f"{guard}st.global.v{n}.f32 [{addr}], {{{', '.join(vals)}}}")
        return
    if n == 1:
        h = p.reg("b16")
        p.emit(f"cvt.rn.{dt}.f32 {h}, {vals[0]}\n{guard}st.global.b16 [{addr}], {h}")
        return
    words = [p.reg("b32") for _ in range(n // 2)]
    for i, w in enumerate(words):
        p.emit(f"cvt.rn.{dt}x2.f32 {w}, {vals[2 * i + 1]}, {vals[2 * i]}")
    if len(words) == 1:
        p.emit(f"{guard}st.global.b32 [{addr}], {words[0]}")
    else:
        p.emit(f"{guard}st.global.v{len(words)}.b32 [{addr}], {{{', '.join(words)}}}")


# ---------------------------------------------------------------------------
# row-wise reductions


@dataclass
class _Access:
    buffer: str
    aff: Affine           # over row axes + the column variable "__col"
    col_coef: int


class RowReduce:
    """One row (all tile axes but the cooperative one) per ``TPR`` threads."""

    COL = "__col"
    CHUNKS_PER_THREAD = 8    # VEC-wide column chunks each thread loads (loads in flight)

    def __init__(self, spec):
        self.spec = spec
        tile, co, others, phases = parse_cooperative(spec)
        if not others:
            raise NotThisTemplate("no row axes: whole-array reduction")
        if any(a.name == "_ksplit" for a in others):
            others, phases = fold_ksplit(spec, others, phases)
        self.tile, self.co, self.row_axes, self.phases = tile, co, others, phases
        self.row_ext = {a.name: int(a.extent.value) for a in others}
        self.rows = math.prod(self.row_ext.values())
        streams = [ph.stmt for ph in phases if ph.kind == "stream"]
        if not streams:
            raise NotImplementedError("cooperative reduction without a streaming loop")
        lens = {int(s.axis.extent.value) for s in streams}
        if len(lens) != 1:
            raise NotImplementedError("streaming loops of different lengths")
        self.L = lens.pop()
        self.ranges = dict(self.row_ext)
        self.ranges[self.COL] = self.L
        self._plan_accesses(streams)
        self._plan_schedule()

    # -- analysis --------------------------------------------------------------
    def _access(self, stmt, axis_name, buffer, index):
        shape = self.spec.param(buffer).shape
        idx = tuple(_rename(e, axis_name, self.COL) for e in index) if axis_name else tuple(index)
        aff = affine_offset(idx, shape, self.ranges)
        return _Access(buffer, aff, aff.get(self.COL))

    def _plan_accesses(self, streams):
        self.accesses = {}    # id(stmt) -> _Access
        for loop in streams:
            ax = loop.axis.name
            for s in loop.body:
                k = type(s).__name__
                if k == "Load" and s.input not in self.spec.constants:
                    _check_buffer(self.spec, s.input)
                    if len(s.names) != 1:
                        raise NotImplementedError("multi-value Load inside a reduction stream")
                    self.accesses[id(s)] = self._access(s, ax, s.input, s.index)
                elif k == "Write":
                    _check_buffer(self.spec, s.output)
                    if len(s.values) != 1 or s.atomic:
                        raise NotImplementedError("vector or atomic Write inside a reduction stream")
                    self.accesses[id(s)] = self._access(s, ax, s.output, s.index)
                elif k in ("Cond", "Loop", "StridedLoop"):
                    raise NotImplementedError(f"{k} inside a reduction stream")

    def _plan_schedule(self):
        col_accesses = [a for a in self.accesses.values() if a.col_coef]
        vec_ok = (self.L % 4 == 0 and all(a.col_coef == 1 for a in col_accesses)
                  and all(c % 4 == 0 for a in col_accesses for v, c in a.aff.coef if v != self.COL)
                  and all(a.aff.const % 4 == 0 for a in col_accesses))
        self.VEC = 4 if vec_ok else 1
        chunks = -(-self.L // self.VEC)
        tpr = 1 << max(0, math.ceil(math.log2(max(1, chunks / self.CHUNKS_PER_THREAD))))
        self.TPR = max(32, min(1024, tpr))
        self.NCH = -(-chunks // self.TPR)
        if self.NCH * self.VEC > 64:
            raise NotImplementedError(f"rows of {self.L} elements exceed the register-resident limit")
        self.CTA = max(self.TPR, 128)
        self.RPC = self.CTA // self.TPR
        self.grid = -(-self.rows // self.RPC)
        self.W = max(1, self.TPR // 32)      # warps per row

    # -- emission --------------------------------------------------------------
    def emit(self) -> str:
        spec = self.spec
        p = Ptx()
        self._ctx_ptx = p
        p.comment(f"row reduction: {self.rows} rows x {self.L} cols, {self.TPR} threads/row, "
                  f"{self.NCH} chunks of {self.VEC}")
        ptrs = {q.name: load_pointer(p, q.name) for q in spec.params if not q.scalar}

        tid, row, lane_r, rowc = p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32")
        pvalid, plead = p.reg("pred"), p.reg("pred")
        log_tpr = int(math.log2(self.TPR))
        p.emit(f"""
            mov.u32 {tid}, %tid.x
            mov.u32 {row}, %ctaid.x
            shr.u32 {rowc}, {tid}, {log_tpr}
            mad.lo.u32 {row}, {row}, {self.RPC}, {rowc}
            and.b32 {lane_r}, {tid}, {self.TPR - 1}
            setp.lt.u32 {pvalid}, {row}, {self.rows}
            min.u32 {rowc}, {row}, {self.rows - 1}
            setp.eq.and.u32 {plead}, {lane_r}, 0, {pvalid}
        """)
        # decompose the (clamped) row into the row axes, row-major
        axis_reg = {}
        rem = rowc
        for a in reversed(self.row_axes):
            ext = self.row_ext[a.name]
            r = p.reg("u32")
            if a is self.row_axes[0]:
                p.emit(f"mov.u32 {r}, {rem}")
            else:
                q = p.reg("u32")
                p.emit(f"rem.u32 {r}, {rem}, {ext}\ndiv.u32 {q}, {rem}, {ext}")
                rem = q
            axis_reg[a.name] = r
        col0 = p.reg("u32")
        p.emit(f"mul.lo.u32 {col0}, {lane_r}, {self.VEC}")
        self.axis_reg, self.col0, self.ptrs = axis_reg, col0, ptrs
        self.pvalid, self.plead, self.lane_r, self.tid = pvalid, plead, lane_r, tid
        self.base_cache = {}    # (buffer, aff) -> u64 address of chunk 0, lane 0
        self.val_cache = {}     # (buffer, aff, chunk) -> [regs]

        ctx = ScalarCtx(p, constants=dict(spec.constants), half_results=True,
                        exact_products=matmul_kernel(spec.name), index_vars=load_index_vars(spec.body))
        ctx.on_load = self._scalar_load
        ctx.on_write = self._leader_write
        # exp(x - M) in a later pass, for an element x whose exp(x - m_t) the online
        # rewrite already holds: e * exp(m_t - M), one exponential per thread, not per element
        self.exp_cache, self.exp_base, self.exp_corr = {}, {}, {}

        def exp_reuse(x_reg, state):
            e = self.exp_cache.get(x_reg)
            if e is None or state not in self.exp_base:
                return None
            corr = self.exp_corr.get(state)
            if corr is None:
                d, corr = p.reg("f32"), p.reg("f32")
                p.emit(f"sub.rn.f32 {d}, {self.exp_base[state]}, {ctx.f32(state)}")
                emit_exp_nonpos(p, corr, d)
                self.exp_corr[state] = corr
            r = p.reg("f32")
            p.emit(f"mul.rn.f32 {r}, {e}, {corr}")
            return r
        ctx.exp_reuse = exp_reuse if self.L % (self.TPR * self.VEC) == 0 else None
        # every accumulator starts at its op's identity before the first pass
        for ph in self.phases:
            if ph.kind == "stream":
                for acc in _accums(ph.stmt.body):
                    if acc.name not in ctx.env:
                        r = p.reg("f32")
                        p.emit(f"mov.f32 {r}, {f32_hex(float(acc.op.identity))}")
                        ctx.env[acc.name] = Val(r, "f32")
                        ctx.mutable.add(acc.name)
        # programmatic dependent launch: every CTA of this grid is on an SM once all have
        # passed here, so the stream's next kernel may launch and set up while this one
        # finishes; this grid waits for the previous kernel (complete, writes visible)
        # before its first global load
        p.emit("griddepcontrol.launch_dependents\ngriddepcontrol.wait")
        # every pass's column loads are independent of the row results: issue them all up
        # front so the second pass's operands (e.g. RMSNorm's weight) are in flight with x
        for ph in self.phases:
            if ph.kind == "stream":
                self._issue_loads(p, ph.stmt)
        smem_decls = []
        for n, ph in enumerate(self.phases):
            if ph.kind == "stream":
                self._emit_stream(ctx, ph.stmt)
            elif ph.kind == "combine":
                smem_decls.append(self._emit_combine(ctx, ph.combine, n))
            elif ph.kind == "scalar":
                lower_body(ctx, [ph.stmt])
            elif ph.kind == "leader":
                skip = p.label("leader")
                p.emit(f"@!{plead} bra {skip}")
                lower_body(ctx, ph.stmt.body)
                p.place(skip)
        p.emit("ret")
        launch = {"kind": "row_reduce", "grid": [self.grid, 1, 1], "block": [self.CTA, 1, 1],
                  "cluster": [1, 1, 1], "smem": 0, "extra_params": [], "pdl": True,
                  "rows": self.rows, "cols": self.L}
        text = entry(spec.name, arg_params(spec), p, maxntid=self.CTA)
        # shared arrays are declared inside the entry body
        if smem_decls:
            text = text.replace("{\n", "{\n" + "\n".join(d for d in smem_decls if d) + "\n", 1)
        return module([text], launch)

    # -- addressing --------------------------------------------------------------
    def _row_base(self, buffer: str, aff: Affine) -> str:
        """u64 address of element (this row, column col0) of ``buffer``."""
        key = (buffer, aff)
        if key in self.base_cache:
            return self.base_cache[key]
        p = self.p
        off = p.reg("b64")
        p.emit(f"mov.u64 {off}, {aff.const}")
        for var, c in aff.coef:
            src = self.col0 if var == self.COL else self.axis_reg[var]
            w = p.reg("b64")
            p.emit(f"cvt.u64.u32 {w}, {src}\nmad.lo.s64 {off}, {w}, {c}, {off}")
        addr = p.reg("b64")
        p.emit(f"mad.lo.s64 {addr}, {off}, {ESZ[_check_buffer(self.spec, buffer)]}, {self.ptrs[buffer]}")
        self.base_cache[key] = addr
        return addr

    @property
    def p(self):
        return self._ctx_ptx

    def _chunk_pred(self, c: int) -> str | None:
        """Predicate 'chunk c of this thread is inside the row', None when always."""
        span = self.TPR * self.VEC
        if (c + 1) * span <= self.L:
            return None
        key = ("chunk", c)
        if key in self.base_cache:
            return self.base_cache[key]
        p = self.p
        pc, col = p.reg("pred"), p.reg("u32")
        p.emit(f"add.u32 {col}, {self.col0}, {c * span}\nsetp.lt.u32 {pc}, {col}, {self.L}")
        self.base_cache[key] = pc
        return pc

    # -- phases ------------------------------------------------------------------
    def _match_online_softmax(self, loop):
        """The online-softmax accumulator pair of one pass, if that is what it is:
        ``m <- max(m, X)`` and ``l <- l * exp(m - G) + exp(X - G) [* 1]`` with
        ``G = max(m, X)``.  Returns (X, m, l) or None."""
        accs = _accums(loop.body)
        if len(accs) != 2:
            return None
        am = [a for a in accs if a.op.name == "maximum" and a.base is None]
        al = [a for a in accs if a.op.name == "add" and a.base is not None]
        if len(am) != 1 or len(al) != 1:
            return None
        am, al = am[0], al[0]
        X, m, l = am.value, am.name, al.name
        defs, ones = {}, set()
        for s in loop.body:
            k = type(s).__name__
            if k == "Assign":
                defs[s.name] = (s.op.name, tuple(s.args))
            elif k == "Let" and type(s.value).__name__ == "Literal" and float(s.value.value) == 1.0:
                ones.add(s.name)

        def is_op(name, op, args=None):
            d = defs.get(name)
            if d is None or d[0] != op:
                return False
            if args is None:
                return True
            if op in ("maximum", "multiply"):
                return sorted(d[1]) == sorted(args)
            return d[1] == tuple(args)

        def strip_one(name):
            d = defs.get(name)
            if d and d[0] == "multiply":
                a, b = d[1]
                if b in ones:
                    return a
                if a in ones:
                    return b
            return name
        gs = [n for n, d in defs.items() if d[0] == "maximum" and sorted(d[1]) == sorted((m, X))]
        if len(gs) != 1:
            return None
        G = gs[0]
        v = strip_one(al.value)
        if not (is_op(v, "exp") and is_op(defs[v][1][0], "subtract", (X, G))):
            return None
        base = defs.get(al.base)
        if base is None or base[0] != "multiply" or l not in base[1]:
            return None
        alpha = [a for a in base[1] if a != l][0]
        if not (is_op(alpha, "exp") and is_op(defs[alpha][1][0], "subtract", (m, G))):
            return None
        return X, m, l

    def _emit_online_softmax(self, ctx: ScalarCtx, loop, match, loads):
        """Register-resident rewrite of the online pair: each thread takes the max of
        its elements, then sums exp(X - max) -- one exp per element and no serial
        dependency -- and folds that into (m, l) with the same online rule."""
        p = ctx.ptx
        X, m, l = match
        # only the statements X depends on (the online update itself is replaced)
        need, deps = {X}, {}
        for s in loop.body:
            k = type(s).__name__
            if k == "Assign":
                deps[s.name] = set(s.args)
            elif k in ("Let", "Load"):
                for n in (s.names if k == "Load" else (s.name,)):
                    deps[n] = set()
        changed = True
        while changed:
            changed = False
            for n in list(need):
                for d in deps.get(n, ()):
                    if d not in need:
                        need.add(d)
                        changed = True
        keep_stmts = [s for s in loop.body if type(s).__name__ in ("Assign", "Let") and
                      s.name in need]
        xs = []
        for c in range(self.NCH):
            for v in range(self.VEC):
                saved = dict(ctx.env)
                for s in loads:
                    acc = self.accesses[id(s)]
                    regs = self.val_cache[(acc.buffer, acc.aff, c if acc.col_coef else "row")]
                    ctx.env[s.names[0]] = Val(regs[v] if acc.col_coef else regs[0], "f32")
                lower_body(ctx, keep_stmts)
                xs.append(ctx.f32(X))
                keep = {n: ctx.env[n] for n in ctx.mutable if n in ctx.env}
                ctx.env = saved
                ctx.env.update(keep)

        def tree(vals, op):
            while len(vals) > 1:
                nxt = []
                for i in range(0, len(vals) - 1, 2):
                    r = p.reg("f32")
                    p.emit(f"{op} {r}, {vals[i]}, {vals[i + 1]}")
                    nxt.append(r)
                if len(vals) % 2:
                    nxt.append(vals[-1])
                vals = nxt
            return vals[0]
        mt = tree(list(xs), "max.f32")
        es = []
        for x in xs:
            d, e = p.reg("f32"), p.reg("f32")
            p.emit(f"sub.rn.f32 {d}, {x}, {mt}")
            emit_exp_nonpos(p, e, d)
            es.append(e)
            self.exp_cache[x] = e
        self.exp_base[m] = mt
        lt = tree(es, "add.rn.f32")
        mr, lr = ctx.f32(m), ctx.f32(l)
        mn, d0, d1, a0, a1 = p.regs("f32", 5)
        p.emit(f"max.f32 {mn}, {mr}, {mt}\nsub.rn.f32 {d0}, {mr}, {mn}\nsub.rn.f32 {d1}, {mt}, {mn}")
        emit_exp_nonpos(p, a0, d0)
        emit_exp_nonpos(p, a1, d1)
        p.emit(f"mul.rn.f32 {a0}, {lr}, {a0}\nfma.rn.f32 {lr}, {lt}, {a1}, {a0}\nmov.f32 {mr}, {mn}")
        ctx.max_states.add(m)

    def _issue_loads(self, p, loop):
        """Issue the pass's column loads (values already cached are not reloaded)."""
        span = self.TPR * self.VEC
        loads = [s for s in loop.body if type(s).__name__ == "Load" and id(s) in self.accesses]
        for s in loads:
            acc = self.accesses[id(s)]
            if not acc.col_coef:
                continue
            for c in range(self.NCH):
                key = (acc.buffer, acc.aff, c)
                if key in self.val_cache:
                    continue
                regs = p.regs("f32", self.VEC)
                addr = self._row_base(acc.buffer, acc.aff)
                pc = self._chunk_pred(c)
                guard = f"@{pc} " if pc else ""
                dt = _check_buffer(self.spec, acc.buffer)
                off = c * span * acc.col_coef * ESZ[dt]      # chunk c: span columns further on
                ld_vec(p, dt, regs, f"{addr}+{off}", guard)
                self.val_cache[key] = regs

    def _emit_stream(self, ctx: ScalarCtx, loop):
        p = ctx.ptx
        span = self.TPR * self.VEC
        loads = [s for s in loop.body if type(s).__name__ == "Load" and id(s) in self.accesses]
        # 1. every column load of the pass was issued up front (_issue_loads)
        self._issue_loads(p, loop)
        # row-constant loads inside the loop: one scalar load per row
        for s in loads:
            acc = self.accesses[id(s)]
            if acc.col_coef:
                continue
            key = (acc.buffer, acc.aff, "row")
            if key not in self.val_cache:
                r = p.reg("f32")
                ld_vec(p, _check_buffer(self.spec, acc.buffer), [r], self._row_base(acc.buffer, acc.aff))
                self.val_cache[key] = [r]
        # 2a. the online-softmax accumulator pair over full chunks: register-resident rewrite
        writes = [s for s in loop.body if type(s).__name__ == "Write"]
        match = self._match_online_softmax(loop)
        if match and not writes and self.L % span == 0:
            self._emit_online_softmax(ctx, loop, match, loads)
            return
        # 2b. the IR's per-element statements, chunk by chunk, lane by lane
        for c in range(self.NCH):
            pc = self._chunk_pred(c)
            skip = None
            if pc:
                skip = p.label("tail")
                p.emit(f"@!{pc} bra {skip}")
            outvals = {id(w): [] for w in writes}
            for v in range(self.VEC):
                saved = dict(ctx.env)
                for s in loads:
                    acc = self.accesses[id(s)]
                    regs = self.val_cache[(acc.buffer, acc.aff, c if acc.col_coef else "row")]
                    ctx.env[s.names[0]] = Val(regs[v] if acc.col_coef else regs[0], "f32")

                def on_write(cx, w, _out=outvals):
                    _out[id(w)].append(cx.f32(w.values[0]))
                ctx.on_write = on_write
                lower_body(ctx, [s for s in loop.body if type(s).__name__ != "Load" or id(s) not in self.accesses])
                # element-local names do not leak into the next element; accumulators persist
                keep = {n: ctx.env[n] for n in ctx.mutable if n in ctx.env}
                ctx.env = saved
                ctx.env.update(keep)
            ctx.on_write = self._leader_write
            for w in writes:
                acc = self.accesses[id(w)]
                addr = self._row_base(acc.buffer, acc.aff)
                vals = outvals[id(w)]
                dt = _check_buffer(self.spec, acc.buffer)
                off = c * span * acc.col_coef * ESZ[dt]
                st_vec(p, dt, vals, f"{addr}+{off}", f"@{self.pvalid} ")
            if skip:
                p.place(skip)

    def _combine_into(self, ctx: ScalarCtx, comb: Combine, others: list[str]):
        for b, o in zip(comb.state_b, others):
            ctx.env[b] = Val(o, "f32")
        lower_body(ctx, comb.combine_states)

    def _emit_combine(self, ctx: ScalarCtx, comb: Combine, n: int) -> str:
        p = ctx.ptx
        for s in comb.state:
            if s not in ctx.mutable:
                ctx.mutable.add(s)
        lanes = min(32, self.TPR)
        xor = lanes // 2
        while xor >= 1:
            others = []
            for s in comb.state:
                o = p.reg("f32")
                p.emit(f"shfl.sync.bfly.b32 {o}, {ctx.f32(s)}, {xor}, 31, -1")
                others.append(o)
            self._combine_into(ctx, comb, others)
            xor //= 2
        if self.W == 1:
            return ""
        # across the warps of a row: lane 0 of each warp publishes, every thread folds
        # the row's W partials in warp order (deterministic, result in every thread)
        ns = len(comb.state)
        arr = f"comb{n}"
        warp, lane, addr, slot = p.reg("u32"), p.reg("u32"), p.reg("u32"), p.reg("u32")
        pl0 = p.reg("pred")
        p.emit(f"""
            shr.u32 {warp}, {self.tid}, 5
            and.b32 {lane}, {self.tid}, 31
            setp.eq.u32 {pl0}, {lane}, 0
            mov.u32 {addr}, {arr}
            mad.lo.u32 {slot}, {warp}, {ns * 4}, {addr}
        """)
        for i, s in enumerate(comb.state):
            p.emit(f"@{pl0} st.shared.f32 [{slot}+{i * 4}], {ctx.f32(s)}")
        p.emit("bar.sync 0")
        rowbase = p.reg("u32")
        # first warp of this thread's row within the CTA
        p.emit(f"shr.u32 {rowbase}, {self.tid}, {int(math.log2(self.TPR))}\n"
               f"mad.lo.u32 {rowbase}, {rowbase}, {self.W * ns * 4}, {addr}")
        for i, s in enumerate(comb.state):
            p.emit(f"ld.shared.f32 {ctx.f32(s)}, [{rowbase}+{i * 4}]")
        for w in range(1, self.W):
            others = []
            for i, s in enumerate(comb.state):
                o = p.reg("f32")
                p.emit(f"ld.shared.f32 {o}, [{rowbase}+{(w * ns + i) * 4}]")
                others.append(o)
            self._combine_into(ctx, comb, others)
        return f"\t.shared .align 16 .f32 {arr}[{self.CTA // 32 * ns}];"

    def _scalar_load(self, ctx: ScalarCtx, s):
        """A Load outside the streams: a row-constant value (e.g. a per-row bias)."""
        dt = _check_buffer(self.spec, s.input)
        if len(s.names) != 1:
            raise NotImplementedError("multi-value scalar Load")
        shape = self.spec.param(s.input).shape
        aff = affine_offset(tuple(s.index), shape, self.row_ext)
        r = ctx.ptx.reg("f32")
        ld_vec(ctx.ptx, dt, [r], self._row_base(s.input, aff))
        ctx.env[s.names[0]] = Val(r, "f32")

    def _leader_write(self, ctx: ScalarCtx, w):
        """A Write in the leader section: one value per row."""
        dt = _check_buffer(self.spec, w.output)
        if len(w.values) != 1:
            raise NotImplementedError("vector leader Write")
        shape = self.spec.param(w.output).shape
        aff = affine_offset(tuple(w.index), shape, self.row_ext)
        addr = self._row_base(w.output, aff)
        if w.atomic:
            # an atomic (+=) output gets one add per row: the whole row is summed here
            if dt != "f32":
                raise NotImplementedError("atomic 16-bit row result")
            ctx.ptx.emit(f"red.global.add.f32 [{addr}], {ctx.f32(w.values[0])}")
        else:
            st_vec(ctx.ptx, dt, [ctx.f32(w.values[0])], addr)


def _rename(expr, old: str, new: str):
    """Substitute Var(old) -> Var(new) in an index expression."""
    k = type(expr).__name__
    if k == "Var":
        return type(expr)(name=new) if expr.name == old else expr
    if k == "BinaryExpr":
        return type(expr)(op=expr.op, left=_rename(expr.left, old, new),
                          right=_rename(expr.right, old, new))
    if k == "TernaryExpr":
        return type(expr)(cond=_rename(expr.cond, old, new), if_true=_rename(expr.if_true, old, new),
                          if_false=_rename(expr.if_false, old, new))
    return expr


# ---------------------------------------------------------------------------
# whole-array reductions


class FullReduce:
    """Every element of the tile's index space folds into one scalar per kernel."""

    UNROLL = 8          # 128-bit loads in flight per thread per iteration
    CTA = 256
    CTAS_PER_SM = 8     # one wave: 8 x 256 threads fit at the kernel's 32 registers

    def __init__(self, spec):
        self.spec = spec
        tile, co, others, phases = parse_cooperative(spec)
        if any(a.name != "_ksplit" for a in others):
            raise NotThisTemplate("has row axes")
        self.tile, self.co, self.others, self.phases = tile, co, others, phases
        streams = [ph for ph in phases if ph.kind == "stream"]
        combines = [ph for ph in phases if ph.kind == "combine"]
        if len(streams) != 1 or len(combines) != 1:
            raise NotImplementedError("whole-array reduction with several passes")
        if phases.index(streams[0]) > phases.index(combines[0]):
            raise NotImplementedError("stream after the combine")
        self.loop = streams[0].stmt
        self.comb = combines[0].combine
        self.tail = phases[phases.index(combines[0]) + 1:]
        accs = _accums(self.loop.body)
        if len(accs) != 1 or accs[0].base is not None:
            raise NotImplementedError("whole-array reduction with coupled accumulators")
        self.acc = accs[0]
        self.op = self.acc.op.name
        if self.op not in ("add", "maximum", "minimum"):
            raise NotImplementedError(f"whole-array {self.op} reduction")
        if self.comb.state != (self.acc.name,):
            raise NotImplementedError("combine of other states than the accumulator")
        # the element index space: ksplit (outer) x loop axis (inner) must be one
        # contiguous run of the input buffer
        self.L = int(self.loop.axis.extent.value)
        ks = int(others[0].extent.value) if others else 1
        self.count = ks * self.L
        loads = [s for s in self.loop.body if type(s).__name__ == "Load"
                 and s.input not in spec.constants]
        if len(loads) != 1 or len(loads[0].names) != 1:
            raise NotImplementedError("whole-array reduction must stream exactly one buffer")
        self.load = loads[0]
        self.dt = _check_buffer(spec, self.load.input)
        self.esz = ESZ[self.dt]
        ranges = {"__i": self.L}
        if others:
            ranges["_ksplit"] = ks
        idx = tuple(_rename(e, self.loop.axis.name, "__i") for e in self.load.index)
        aff = affine_offset(idx, spec.param(self.load.input).shape, ranges)
        if aff.get("__i") != 1 or aff.get("_ksplit") not in (0, self.L) or aff.const != 0:
            raise NotImplementedError("reduced elements are not one contiguous run")
        if ks > 1 and aff.get("_ksplit") != self.L:
            raise NotImplementedError("split axis is not the outer block of the run")
        vw = 16 // self.esz                      # elements in one 128-bit load
        self.VEC = vw if self.count % vw == 0 else 1
        per_iter = self.CTA * self.VEC * self.UNROLL
        self.grid = max(1, min(SMS * self.CTAS_PER_SM, -(-self.count // per_iter)))
        self.scratch_bytes = 16 + 8 * self.grid

    def emit(self) -> str:
        spec = self.spec
        p = Ptx()
        p.comment(f"whole-array {self.op}: {self.count} elements, grid {self.grid} x {self.CTA}")
        ptrs = {q.name: load_pointer(p, q.name) for q in spec.params if not q.scalar}
        scratch = p.reg("b64")
        p.emit(f"ld.param.u64 {scratch}, [param__scratch]\ncvta.to.global.u64 {scratch}, {scratch}")
        x = ptrs[self.load.input]
        is_add = self.op == "add"
        ident = float(self.acc.op.identity)

        tid, gtid, nthr = p.reg("u32"), p.reg("b64"), p.reg("b64")
        p.emit(f"""
            mov.u32 {tid}, %tid.x
            mov.u32 %r_cta, %ctaid.x
            mad.wide.u32 {gtid}, %r_cta, {self.CTA}, {0}
        """.replace("%r_cta", p.named_reg("%cta", "u32")))
        p.emit(f"cvt.u64.u32 {nthr}, {tid}\nadd.s64 {gtid}, {gtid}, {nthr}")
        total_thr = self.grid * self.CTA
        ctx = ScalarCtx(p, constants=dict(spec.constants), half_results=True,
                        exact_products=matmul_kernel(spec.name), index_vars=load_index_vars(spec.body))

        # per-thread accumulators: f64 for sums (f32 groups of VEC*UNROLL folded in),
        # f32 for max/min (exact)
        if is_add:
            accd = p.reg("f64")
            p.emit(f"mov.f64 {accd}, 0d0000000000000000")
        else:
            accf = p.reg("f32")
            p.emit(f"mov.f32 {accf}, {f32_hex(ident)}")

        body_wo_acc = [s for s in self.loop.body if s is not self.load and s is not self.acc]
        combine_op = {"add": "add.rn.f32", "maximum": "max.f32", "minimum": "min.f32"}[self.op]

        def fold_elements(vals: list[str]):
            """Map each loaded value through the IR's per-element statements (the
            Accum's operand), then fold the group as a balanced tree; sums return the
            f32 group partial, max/min fold straight into ``accf``."""
            mapped = []
            for v in vals:
                saved = dict(ctx.env)
                ctx.env[self.load.names[0]] = Val(v, "f32")
                lower_body(ctx, body_wo_acc)
                mapped.append(ctx.f32(self.acc.value))
                ctx.env = saved
            while len(mapped) > 1:
                nxt = []
                for i in range(0, len(mapped) - 1, 2):
                    r = p.reg("f32")
                    p.emit(f"{combine_op} {r}, {mapped[i]}, {mapped[i + 1]}")
                    nxt.append(r)
                if len(mapped) % 2:
                    nxt.append(mapped[-1])
                mapped = nxt
            if is_add:
                return mapped[0]
            p.emit(f"{combine_op} {accf}, {accf}, {mapped[0]}")
            return None

        # ---- main grid-stride loop over warp spans of 32 x UNROLL x VEC elements
        # (64-bit offsets): load u of a warp reads 32 consecutive vectors, so every
        # load instruction is one fully coalesced 512-byte (VEC=4) access
        group = self.VEC * self.UNROLL
        span = 32 * group                        # elements per warp per iteration
        nspans = self.count // span
        nwarps = total_thr // 32
        wi, pg = p.reg("b64"), p.reg("pred")
        loop, done = p.label("grp"), p.label("grp_done")
        lane0, wid = p.reg("u32"), p.reg("b64")
        p.emit(f"and.b32 {lane0}, {tid}, 31\nshr.u64 {wid}, {gtid}, 5\nmov.u64 {wi}, {wid}")
        lane_off = p.reg("b64")
        p.emit(f"mul.wide.u32 {lane_off}, {lane0}, {self.VEC * self.esz}")
        p.place(loop)
        p.emit(f"setp.ge.u64 {pg}, {wi}, {nspans}\n@{pg} bra {done}")
        addr = p.reg("b64")
        p.emit(f"mad.lo.s64 {addr}, {wi}, {span * self.esz}, {x}\nadd.s64 {addr}, {addr}, {lane_off}")
        vals = []
        for u in range(self.UNROLL):
            regs = p.regs("f32", self.VEC)
            ld_vec(p, self.dt, regs, f"{addr}+{u * 32 * self.VEC * self.esz}",
                   cache=".nc.L1::no_allocate" if self.VEC > 1 else ".nc")
            vals += regs
        grp = fold_elements(vals)
        if is_add:
            gd = p.reg("f64")
            p.emit(f"cvt.f64.f32 {gd}, {grp}\nadd.rn.f64 {accd}, {accd}, {gd}")
        p.emit(f"add.s64 {wi}, {wi}, {nwarps}\nbra.uni {loop}")
        p.place(done)
        # ---- tail elements (count not a multiple of a warp span): one per thread
        tail0 = nspans * span
        if tail0 < self.count:
            ti, pt = p.reg("b64"), p.reg("pred")
            tl, td = p.label("tail"), p.label("tail_done")
            p.emit(f"add.s64 {ti}, {gtid}, {tail0}")
            p.place(tl)
            p.emit(f"setp.ge.u64 {pt}, {ti}, {self.count}\n@{pt} bra {td}")
            v, a2 = p.reg("f32"), p.reg("b64")
            p.emit(f"mad.lo.s64 {a2}, {ti}, {self.esz}, {x}")
            ld_vec(p, self.dt, [v], a2, cache=".nc")
            grp = fold_elements([v])
            if is_add:
                gd = p.reg("f64")
                p.emit(f"cvt.f64.f32 {gd}, {grp}\nadd.rn.f64 {accd}, {accd}, {gd}")
            p.emit(f"add.s64 {ti}, {ti}, {total_thr}\nbra.uni {tl}")
            p.place(td)

        # ---- CTA combine (fixed order): warp butterfly, then warp partials via smem
        if is_add:
            for xor in (16, 8, 4, 2, 1):
                lo, hi, o = p.reg("b32"), p.reg("b32"), p.reg("f64")
                p.emit(f"""
                    mov.b64 {{{lo}, {hi}}}, {accd}
                    shfl.sync.bfly.b32 {lo}, {lo}, {xor}, 31, -1
                    shfl.sync.bfly.b32 {hi}, {hi}, {xor}, 31, -1
                    mov.b64 {o}, {{{lo}, {hi}}}
                    add.rn.f64 {accd}, {accd}, {o}
                """)
            part = accd
        else:
            mm = "max" if self.op == "maximum" else "min"
            for xor in (16, 8, 4, 2, 1):
                o = p.reg("f32")
                p.emit(f"shfl.sync.bfly.b32 {o}, {accf}, {xor}, 31, -1\n{mm}.f32 {accf}, {accf}, {o}")
            part = p.reg("f64")
            p.emit(f"cvt.f64.f32 {part}, {accf}")
        nw = self.CTA // 32
        lane, warp, sa = p.reg("u32"), p.reg("u32"), p.reg("u32")
        pl0, pt0 = p.reg("pred"), p.reg("pred")
        p.emit(f"""
            and.b32 {lane}, {tid}, 31
            shr.u32 {warp}, {tid}, 5
            setp.eq.u32 {pl0}, {lane}, 0
            setp.eq.u32 {pt0}, {tid}, 0
            mov.u32 {sa}, wpart
            mad.lo.u32 {sa}, {warp}, 8, {sa}
            @{pl0} st.shared.f64 [{sa}], {part}
            bar.sync 0
        """)
        done2 = p.label("cta_done")
        l_t0 = p.label("t0_done")
        flag = p.reg("u32")
        p.emit(f"@!{pt0} bra {l_t0}")
        ctot, t = p.reg("f64"), p.reg("f64")
        p.emit(f"ld.shared.f64 {ctot}, [wpart]")
        for w in range(1, nw):
            p.emit(f"ld.shared.f64 {t}, [wpart+{w * 8}]")
            p.emit(self._combine_f64(ctot, t))
        # publish the CTA partial, then take a ticket; the CTA that takes the last one
        # finishes (thread 0 tells the others through shared memory)
        paddr, ticket, pl = p.reg("b64"), p.reg("u32"), p.reg("pred")
        p.emit(f"""
            mad.wide.u32 {paddr}, %cta, 8, {scratch}
            st.global.f64 [{paddr}+16], {ctot}
            fence.acq_rel.gpu
            atom.global.acq_rel.gpu.add.u32 {ticket}, [{scratch}], 1
            setp.eq.u32 {pl}, {ticket}, {self.grid - 1}
            selp.u32 {flag}, 1, 0, {pl}
            st.shared.u32 [wlast], {flag}
        """)
        p.place(l_t0)
        plast = p.reg("pred")
        p.emit(f"bar.sync 0\nld.shared.u32 {flag}, [wlast]\nsetp.eq.u32 {plast}, {flag}, 0\n"
               f"@{plast} bra {done2}")
        # last CTA, every thread: the CTA partials strided over the threads (all loads of a
        # thread in flight together, folded in CTA order), then the same fixed-order warp
        # butterfly and warp fold as above.  (A single thread walking the partials one
        # dependent L2 load at a time cost tens of microseconds per launch.)
        ident64 = f64_hex(0.0 if is_add else (-math.inf if self.op == "maximum" else math.inf))
        p.emit("fence.acq_rel.gpu")
        per = -(-self.grid // self.CTA)
        vals = []
        for j in range(per):
            idx, a, v, pj = p.reg("u32"), p.reg("b64"), p.reg("f64"), p.reg("pred")
            p.emit(f"""
                mov.f64 {v}, {ident64}
                add.u32 {idx}, {tid}, {j * self.CTA}
                setp.lt.u32 {pj}, {idx}, {self.grid}
                mad.wide.u32 {a}, {idx}, 8, {scratch}
                @{pj} ld.global.cg.f64 {v}, [{a}+16]
            """)
            vals.append(v)
        tot = vals[0]
        for v in vals[1:]:
            p.emit(self._combine_f64(tot, v))
        for xor in (16, 8, 4, 2, 1):
            lo, hi, o = p.reg("b32"), p.reg("b32"), p.reg("f64")
            p.emit(f"""
                mov.b64 {{{lo}, {hi}}}, {tot}
                shfl.sync.bfly.b32 {lo}, {lo}, {xor}, 31, -1
                shfl.sync.bfly.b32 {hi}, {hi}, {xor}, 31, -1
                mov.b64 {o}, {{{lo}, {hi}}}
            """)
            p.emit(self._combine_f64(tot, o))
        p.emit(f"@{pl0} st.shared.f64 [{sa}], {tot}\nbar.sync 0\n@!{pt0} bra {done2}")
        p.emit(f"ld.shared.f64 {tot}, [wpart]")
        for w in range(1, nw):
            p.emit(f"ld.shared.f64 {t}, [wpart+{w * 8}]")
            p.emit(self._combine_f64(tot, t))
        # keep the f64 total beside the ticket (scratch bytes 8..16): a sharded reduction
        # all-reduces these per-GPU totals in f64; then reset the ticket for the next launch
        p.emit(f"st.global.f64 [{scratch}+8], {tot}")
        p.emit(f"st.global.u32 [{scratch}], 0")
        fin = p.reg("f32")
        p.emit(f"cvt.rn.f32.f64 {fin}, {tot}")
        lctx = ScalarCtx(p, constants=dict(spec.constants), half_results=True)
        lctx.env[self.acc.name] = Val(fin, "f32")
        lctx.on_write = self._final_write(ptrs)
        for ph in self.tail:
            if ph.kind == "scalar":
                lower_body(lctx, [ph.stmt])
            elif ph.kind == "leader":
                lower_body(lctx, ph.stmt.body)
            else:
                raise NotImplementedError(f"{ph.kind} after the whole-array combine")
        p.place(done2)
        p.emit("ret")
        params = arg_params(spec) + [".param .u64 param__scratch"]
        text = entry(spec.name, params, p, maxntid=self.CTA)
        text = text.replace("{\n", "{\n" + f"\t.shared .align 8 .f64 wpart[{nw}];\n"
                            "\t.shared .align 4 .u32 wlast;\n", 1)
        launch = {"kind": "full_reduce", "grid": [self.grid, 1, 1], "block": [self.CTA, 1, 1],
                  "cluster": [1, 1, 1], "smem": 0, "count": self.count,
                  "extra_params": [{"kind": "scratch", "bytes": self.scratch_bytes, "zero_once": True,
                                    "f64_total_offset": 8}]}
        return module([text], launch)

    def _combine_f64(self, a: str, b: str) -> str:
        if self.op == "add":
            return f"add.rn.f64 {a}, {a}, {b}"
        return f"{'max' if self.op == 'maximum' else 'min'}.f64 {a}, {a}, {b}"

    def _final_write(self, ptrs):
        def on_write(ctx, w):
            dt = _check_buffer(self.spec, w.output)
            if len(w.values) != 1:
                raise NotImplementedError("vector result write")
            shape = self.spec.param(w.output).shape
            if any(expr_vars(e) for e in w.index):
                raise NotImplementedError("whole-array result indexed by an axis")
            from ..stmts import flat_offset
            off = flat_offset(tuple(w.index), shape, {})
            # the IR's atomic add into a zeroed scalar and this single store of the
            # full sum leave the same value (the runner re-zeroes atomic outputs)
            st_vec(ctx.ptx, dt, [ctx.f32(w.values[0])], f"{ptrs[w.output]}+{off * ESZ[dt]}")
        return on_write


def emit_reduction(spec):
    """Row-wise or whole-array template for a cooperative reduction kernel."""
    try:
        k = RowReduce(spec)
    except NotThisTemplate:
        try:
            k = FullReduce(spec)
        except NotThisTemplate as e:
            raise NotImplementedError(f"cooperative reduction outside both templates: {e}") from None
    return k.emit()
