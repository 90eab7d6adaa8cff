"""emmy's f32 attention ``softmax(q @ kt * c) @ v`` as one warp-per-query-row SIMT kernel.

The reference lowers f32 attention (problems/a01_attention, problems/a02_attention_128,
tests/problems/x_a_*) to a register-tiled Tile over the OUTPUT elements: every thread owns
a few (row, column) outputs and, for each of them, walks all keys with an online softmax,
recomputing the full ``q . k`` dot product per key and per output column
(compiler/codegen.py's tiled lowering; the IR: ``Loop(key) { Loop(d) { Accum(q*kt) } ;
max / exp / rescale ; Accum(p * v) }``).  Run as written, that is Sk x D x Dv FMAs per row
on a few hundred threads.

Here the same arithmetic is reorganised around the query row:

* one CTA of W warps per block of W x R query rows of one batch entry; a warp owns R rows;
* keys stream through shared memory in chunks of KC (32 or 64) keys: the chunk of kt
  (``[D][KC]``, staged along the key axis, which is contiguous in kt) -- or of a
  key-major k (sdpa's ``[.., Sk, D]``: one contiguous span, rows stored with the odd
  stride D + 1 so the lanes' key rows fall in different banks) -- and of v (``[KC][Dv]``,
  one contiguous span), zero-filled past Sk so padding keys give p = 0 and never NaN;
* grouped-query heads (``k.repeat_interleave(G, dim=1)``, tests/problems/x_l_gqa): query
  entry y reads k / v entry y // G, checked over every entry from the loads' indices;
* scores: lane j owns keys j and j + 32 of the chunk, ``s = sum_d q[d] kt[d][j]`` with q
  broadcast from shared memory (128-bit loads) -- each kt element read once per warp
  serves R rows;
* online softmax per row: chunk max by warp butterfly, ``alpha = 2^((m - m') log2 e)``,
  ``p = 2^((s c - m') log2 e)``; the row sum stays a per-lane partial until the end;
* ``o += p v``: p goes through a per-warp shared row (128-bit broadcast loads), lane c
  owns output columns c, c + 32, ...;
* epilogue: the row sum by butterfly, ``o / l`` (IEEE division), predicated stores.

The same kernel takes the score-input form (the online softmax over a score buffer that the
reference's split attention runs after its Q K^T kernel, tests/problems/x_h_attn_odd): the
scores are read from the buffer instead of computed, the IR's per-key transform (its f16
rounding and f16 scale) and its loop-invariant statements are lowered with the element-map
statement lowering, and v / the output may be 16-bit (widened to f32 in shared memory,
rounded on the store).

Everything is f32; the exponentials use ``ex2.approx`` (relative error ~2^-22), inside the
fixtures' rtol 1e-3.  No global synchronisation, no atomics: deterministic.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

from ..ptx import Ptx, entry, f32_hex, module
from ..stmts import Val, expr_vars, lower_body
from .common import arg_params, load_pointer

LOG2E = 1.4426950408889634
WARPS = 4


@dataclass
class F32AttnConfig:
    name: str
    B: int
    Sq: int
    Sk: int
    D: int
    Dv: int
    q: str
    k: str
    v: str
    o: str
    scale_param: str | None        # 1-element buffer holding the multiplier (or its inverse)
    scale_recip: bool              # multiplier = 1 / param[0]
    scale_const: float             # used when scale_param is None
    kt: bool = True                # k stored [.., D, Sk] (kt); False: [.., Sk, D] (sdpa's k)
    group: int = 1                 # query batch entries per k / v entry (grouped-query heads)
    R: int = 1                     # query rows per warp
    KC: int = 64                   # keys per staged chunk
    scores: str | None = None      # score-input form: this [.., Sq, Sk] buffer instead of q kt
    s_name: str = ""               # the name its Load binds
    s_out: str = ""                # the transformed score the softmax takes
    s_chain: tuple = ()            # the IR's statements from s_name to s_out, per key
    prelude: tuple = ()            # the loop-invariant statements before the key loop
    dtypes: tuple = ()             # (buffer, dtype) of 16-bit buffers (all others f32)

    def dt(self, name: str) -> str:
        return dict(self.dtypes).get(name, "f32")

    @property
    def KPL(self) -> int:          # keys per lane per chunk
        return self.KC // 32

    @property
    def NC(self) -> int:           # output columns per lane
        return -(-self.Dv // 32)

    @property
    def DP(self) -> int:           # q row stride in shared memory (16-byte rows)
        return -(-self.D // 4) * 4

    @property
    def DK(self) -> int:           # shared row stride of a key-major k chunk (odd: no conflicts)
        return self.D + 1

    @property
    def vec(self) -> bool:         # 128-bit staging: key and value rows in whole float4s
        return ((self.Sk % 4 == 0 if self.kt else self.D % 4 == 0) and self.Dv % 4 == 0
                and self.dt(self.v) == "f32")


def _walk_loops(body, loops=()):
    """(statement, enclosing loop axes outermost first) over a statement tree."""
    for s in body:
        yield s, loops
        k = type(s).__name__
        inner = loops + ((s.axis.name,) if k == "Loop" else ())
        for attr in ("body", "else_body"):
            sub = getattr(s, attr, None)
            if isinstance(sub, tuple):
                yield from _walk_loops(sub, inner)


_ALLOWED = {"Tile", "Load", "Assign", "Accum", "Loop", "Let", "Write", "Cond"}


def analyze(spec) -> F32AttnConfig:
    """Recognise ``softmax(q @ kt * c, -1) @ v`` in f32 from the statements.

    Raises NotImplementedError for anything else (masks, 16-bit operands, batch maps
    other than y -> y // G, ...), which then lowers as an element map."""
    if len(spec.body) != 1 or type(spec.body[0]).__name__ != "Tile":
        raise NotImplementedError("not a single Tile")
    walk = list(_walk_loops(spec.body))
    kinds = {type(s).__name__ for s, _ in walk}
    if not kinds <= _ALLOWED:
        raise NotImplementedError(f"statements {sorted(kinds - _ALLOWED)}")
    defs = {}
    for s, _ in walk:
        k = type(s).__name__
        if k == "Load":
            for n in s.names:
                defs[n] = s
        elif k in ("Assign", "Let"):
            defs[s.name] = s
    # the contraction: Accum(add) of a product of two loads, in a loop nested in the key loop
    dots = []
    for s, loops in walk:
        if type(s).__name__ == "Accum" and s.op.name == "add" and len(loops) >= 2:
            prod = defs.get(s.value)
            if prod is not None and type(prod).__name__ == "Assign" and prod.op.name == "multiply" \
                    and all(type(defs.get(a)).__name__ == "Load" for a in prod.args):
                dots.append((s, loops, [defs[a] for a in prod.args]))
    if not dots:
        return _analyze_scores(spec, walk, defs)
    key, red = dots[0][1][-2], dots[0][1][-1]
    q_in = k_in = None
    q_ld = k_ld = None
    kt_layout = set()
    for acc, loops, lds in dots:
        if loops[-2:] != (key, red) or tuple(acc.axes or ()) != (red,):
            raise NotImplementedError("dot products over different loops")
        for ld in lds:
            last = expr_vars(ld.index[-1])
            prev = expr_vars(ld.index[-2]) if len(ld.index) >= 2 else set()
            if last == {red} and not any(key in expr_vars(i) for i in ld.index):
                q_in, q_ld = q_in or ld.input, q_ld or ld
                if ld.input != q_in:
                    raise NotImplementedError("two q buffers")
                continue
            if last == {key} and prev == {red}:
                kt_layout.add(True)
            elif last == {red} and prev == {key}:
                kt_layout.add(False)
            else:
                raise NotImplementedError("dot product operands not (q row, k row / kt column)")
            k_in, k_ld = k_in or ld.input, k_ld or ld
            if ld.input != k_in:
                raise NotImplementedError("two k buffers")
    if q_in is None or k_in is None or len(kt_layout) != 1:
        raise NotImplementedError("q / k not identified")
    # v: read in the key loop (outside the dot product), key index on its rows
    v_in = v_ld = None
    for s, loops in walk:
        if type(s).__name__ == "Load" and s.input not in (q_in, k_in):
            if len(s.index) >= 2 and key in loops and red not in loops and \
                    expr_vars(s.index[-2]) == {key} and key not in expr_vars(s.index[-1]):
                v_in, v_ld = v_in or s.input, v_ld or s
                if s.input != v_in:
                    raise NotImplementedError("two v buffers")
    if v_in is None:
        raise NotImplementedError("no v operand")
    # the softmax: an exp and a running max over the key axis; the score times a scale
    if not any(type(s).__name__ == "Assign" and s.op.name == "exp" for s, _ in walk):
        raise NotImplementedError("no exp")
    if not any(type(s).__name__ == "Accum" and s.op.name == "maximum" and key in (s.axes or ())
               for s, _ in walk):
        raise NotImplementedError("no running max over the keys")
    dot_names = {d[0].name for d in dots}
    scale_param, recip, const = None, False, 1.0
    scaled = [s for s, _ in walk if type(s).__name__ == "Assign" and set(s.args) & dot_names]
    if not scaled or any(s.op.name != "multiply" or len(s.args) != 2 for s in scaled):
        raise NotImplementedError("score not scaled by a multiply")
    others = {a for s in scaled for a in s.args if a not in dot_names}
    if len(others) != 1:
        raise NotImplementedError("scores scaled by different values")
    sd = defs.get(next(iter(others)))

    def scalar_param(ld):
        if ld is None or type(ld).__name__ != "Load":
            return None
        p = spec.param(ld.input)
        if p.dtype != "f32" or p.scalar or math.prod(p.shape) != 1:
            return None
        return p.name
    if type(sd).__name__ == "Load" and scalar_param(sd):
        scale_param = scalar_param(sd)
    elif type(sd).__name__ == "Assign" and sd.op.name == "reciprocal" and len(sd.args) == 1 \
            and scalar_param(defs.get(sd.args[0])):
        scale_param, recip = scalar_param(defs.get(sd.args[0])), True
    elif type(sd).__name__ == "Let" and type(sd.value).__name__ == "Literal":
        const = float(sd.value.value)
    else:
        raise NotImplementedError("scale is not a constant or a 1-element buffer")
    # the scaled score feeds the online softmax and nothing else: the running maximum and
    # the differences taken against it (a softcap, a bias or a mask in between would sit
    # here, and this template does not compute them)
    _check_softmax_use(walk, {s.name for s in scaled})
    _check_normalised(walk, defs, key)
    _check_pv(walk, defs, key, v_in)
    _check_guards(walk, {key, red})
    loaded = {s.input for s, _ in walk if type(s).__name__ == "Load"}
    if loaded - {q_in, k_in, v_in, scale_param}:
        raise NotImplementedError(f"extra inputs {sorted(loaded - {q_in, k_in, v_in})}")
    writes = [s for s, _ in walk if type(s).__name__ == "Write"]
    if len({w.output for w in writes}) != 1:
        raise NotImplementedError("not one output")
    Q, K, V, O = (spec.param(n) for n in (q_in, k_in, v_in, writes[0].output))
    if any(p.dtype != "f32" or p.scalar for p in (Q, K, V, O)):
        raise NotImplementedError("f32 buffers only")
    if len(Q.shape) < 2 or not (len(Q.shape) == len(K.shape) == len(V.shape) == len(O.shape)):
        raise NotImplementedError("operand ranks")
    kt = kt_layout.pop()
    Sq, D = Q.shape[-2:]
    Sk, Dv = V.shape[-2:]
    if tuple(K.shape[-2:]) != ((D, Sk) if kt else (Sk, D)) or tuple(O.shape[-2:]) != (Sq, Dv) \
            or tuple(O.shape) != tuple(Q.shape[:-1]) + (Dv,):
        raise NotImplementedError("operand shapes")
    B = math.prod(Q.shape[:-2])
    group = _lead_group(spec, q_ld, [w.index for w in writes], k_ld, v_ld)
    if D > 256 or Dv > 256 or B > 65535 or min(Sq, Sk, D, Dv) < 1:
        raise NotImplementedError("head dims above 256")
    cfg = F32AttnConfig(spec.name, B, Sq, Sk, D, Dv, Q.name, K.name, V.name, O.name,
                        scale_param, recip, const, kt=kt, group=group)
    cfg.KC = 32 if Sk <= 32 else 64
    # rows per warp: reuse each staged key across rows once the grid covers the SMs
    for R in (4, 2):
        if B * -(-Sq // (WARPS * R)) >= 148:
            cfg.R = R
            break
    return cfg


def _check_softmax_use(walk, scaled_names: set) -> None:
    """The scaled score feeds the online softmax and nothing else: the running maximum and
    the differences taken against it (a softcap, a bias or a mask in between would sit
    here, and this template does not compute them)."""
    for s, _ in walk:
        k = type(s).__name__
        uses = set(s.args) if k == "Assign" else {s.value} if k == "Accum" else set()
        if uses & scaled_names:
            if not ((k == "Assign" and s.op.name in ("maximum", "subtract")) or
                    (k == "Accum" and s.op.name == "maximum")):
                raise NotImplementedError(f"the scaled score also feeds {s.op.name}")


def _check_normalised(walk, defs, key: str) -> None:
    """Every written value is (sum of p v) * 1 / (sum of p), both accumulated over the keys."""
    key_sums = {s.name for s, _ in walk if type(s).__name__ == "Accum" and s.op.name == "add"
                and key in (s.axes or ())}
    for w, _ in ((s, l) for s, l in walk if type(s).__name__ == "Write"):
        for val in w.values:
            d = defs.get(val)
            if type(d).__name__ != "Assign" or d.op.name != "multiply" or len(d.args) != 2:
                raise NotImplementedError("output is not a normalised sum")
            a, b = (defs.get(x) for x in d.args)
            if type(b).__name__ == "Assign" and b.op.name == "reciprocal":
                num, den = d.args[0], b.args[0]
            elif type(a).__name__ == "Assign" and a.op.name == "reciprocal":
                num, den = d.args[1], a.args[0]
            else:
                raise NotImplementedError("output is not a normalised sum")
            if num not in key_sums or den not in key_sums:
                raise NotImplementedError("output is not a normalised sum")


def _check_pv(walk, defs, key: str, v_input: str) -> None:
    """Every sum over the keys adds exp(..) times a v element (o) or times 1 (l): the
    template multiplies the f32 probabilities straight into v, so a p rounded to 16 bits
    first (or any other step between the exponential and the product) is handed back."""
    for acc, _ in walk:
        if type(acc).__name__ != "Accum" or acc.op.name != "add" or key not in (acc.axes or ()):
            continue
        d = defs.get(acc.value)
        if type(d).__name__ != "Assign" or d.op.name != "multiply" or len(d.args) != 2:
            raise NotImplementedError("a key sum that is not a product")
        kinds = []
        for a in d.args:
            x = defs.get(a)
            k = type(x).__name__
            if k == "Assign" and x.op.name == "exp":
                kinds.append("exp")
            elif k == "Load" and x.input == v_input:
                kinds.append("v")
            elif k == "Let" and type(x.value).__name__ == "Literal" and float(x.value.value) == 1.0:
                kinds.append("one")
            else:
                kinds.append("other")
        if sorted(kinds) not in (["exp", "v"], ["exp", "one"]):
            raise NotImplementedError("a key sum other than exp * v or exp * 1")


def _check_guards(walk, axes: set) -> None:
    """Guards only: no condition may look at the key or reduction axis (a mask would)."""
    for s, _ in walk:
        if type(s).__name__ == "Cond" and expr_vars(s.cond) & axes:
            raise NotImplementedError("a condition on the key axis (mask)")


_HALF = ("f16", "bf16")


def _analyze_scores(spec, walk, defs) -> F32AttnConfig:
    """``softmax(f(s), -1) @ v`` over a score buffer s: the second kernel of the reference's
    split attention (tests/problems/x_h_attn_odd, after a Q K^T kernel wrote s), an online
    softmax over the key loop whose per-key transform f (the 16-bit rounding and scale the
    IR states) is lowered from the IR's own statements; the loop-invariant statements before
    the key loop (a scale read from a 1-element buffer, its reciprocal) run once."""
    tile = spec.body[0]
    maxes = [(s, l) for s, l in walk if type(s).__name__ == "Accum" and s.op.name == "maximum"]
    if not maxes or any(len(s.axes or ()) != 1 for s, _ in maxes):
        raise NotImplementedError("no running max over one axis")
    key = maxes[0][0].axes[0]
    if any(s.axes[0] != key or key not in l for s, l in maxes):
        raise NotImplementedError("running maxima over different loops")
    if any(key in l and len(l) > 1 for _, l in walk):
        raise NotImplementedError("loops nested in the key loop")
    in_loop = {id(s) for s, l in walk if key in l}
    s_ld, chain, seen = None, [], set()

    def trace(name):
        nonlocal s_ld
        d = defs.get(name)
        if d is None:
            raise NotImplementedError(f"{name} not defined")
        if id(d) not in in_loop or id(d) in seen:
            return
        seen.add(id(d))
        k = type(d).__name__
        if k == "Load":
            if s_ld is not None or len(d.names) != 1 or expr_vars(d.index[-1]) != {key} \
                    or any(key in expr_vars(i) for i in d.index[:-1]):
                raise NotImplementedError("score not one load of a [.., Sq, Sk] buffer")
            s_ld = d
        elif k == "Assign":
            for a in d.args:
                trace(a)
            chain.append(d)
        elif k == "Let":
            chain.append(d)
        else:
            raise NotImplementedError(f"{k} in the score transform")
    s_out = maxes[0][0].value
    trace(s_out)
    if s_ld is None:
        raise NotImplementedError("no score load")
    prelude = []
    for st in tile.body:
        k = type(st).__name__
        if k == "Loop":
            break
        if k == "Load" and not any(expr_vars(i) for i in st.index) and len(st.names) == 1:
            prelude.append(st)
        elif k in ("Assign", "Let"):
            prelude.append(st)
        else:
            raise NotImplementedError(f"{k} before the key loop")
    v_ld = None
    for st, loops in walk:
        if type(st).__name__ == "Load" and st.input != s_ld.input and key in loops:
            if len(st.index) < 2 or expr_vars(st.index[-2]) != {key} or key in expr_vars(st.index[-1]):
                raise NotImplementedError("a load in the key loop that is not s or v")
            if v_ld is not None and st.input != v_ld.input:
                raise NotImplementedError("two v buffers")
            v_ld = v_ld or st
    if v_ld is None:
        raise NotImplementedError("no v operand")
    if not any(type(st).__name__ == "Assign" and st.op.name == "exp" for st, _ in walk):
        raise NotImplementedError("no exp")
    _check_softmax_use(walk, {s.value for s, _ in maxes})
    _check_normalised(walk, defs, key)
    _check_pv(walk, defs, key, v_ld.input)
    _check_guards(walk, {key})
    _check_copies(tile, walk, defs, in_loop, maxes, chain, s_ld, v_ld.input)
    writes = [st for st, _ in walk if type(st).__name__ == "Write"]
    if len({w.output for w in writes}) != 1:
        raise NotImplementedError("not one output")
    S, V, O = (spec.param(n) for n in (s_ld.input, v_ld.input, writes[0].output))
    pre_in = {st.input for st in prelude if type(st).__name__ == "Load"}
    loaded = {st.input for st, _ in walk if type(st).__name__ == "Load"}
    if loaded - {S.name, V.name} - pre_in:
        raise NotImplementedError("extra inputs")
    for n in pre_in:
        q = spec.param(n)
        if q.scalar or q.dtype not in ("f32",) + _HALF:
            raise NotImplementedError("a prelude load that is not a float buffer")
    if any(q.scalar or q.dtype not in ("f32",) + _HALF for q in (S, V, O)) or len(S.shape) < 2 \
            or not (len(S.shape) == len(V.shape) == len(O.shape)):
        raise NotImplementedError("operand types or ranks")
    Sq, Sk = S.shape[-2:]
    Dv = V.shape[-1]
    if V.shape[-2] != Sk or tuple(O.shape) != tuple(S.shape[:-1]) + (Dv,):
        raise NotImplementedError("operand shapes")
    B = math.prod(S.shape[:-2])
    group = _lead_group(spec, s_ld, [w.index for w in writes], v_ld, v_ld)
    if Dv > 256 or B > 65535 or min(Sq, Sk, Dv) < 1:
        raise NotImplementedError("value dims above 256")
    cfg = F32AttnConfig(spec.name, B, Sq, Sk, 0, Dv, "", "", V.name, O.name, None, False, 1.0,
                        group=group, scores=S.name, s_name=s_ld.names[0], s_out=s_out,
                        s_chain=tuple(chain), prelude=tuple(prelude),
                        dtypes=tuple((q.name, q.dtype) for q in (S, V, O) if q.dtype in _HALF))
    cfg.KC = 32 if Sk <= 32 else 64
    for R in (4, 2):
        if B * -(-Sq // (WARPS * R)) >= 148:
            cfg.R = R
            break
    return cfg


def _chain_signature(root: str, defs, in_loop: set, s_input: str):
    """(the score load, a name-free signature of the per-key statements from that load
    to ``root``): every statement's kind, op, type and where each argument comes from
    (an earlier statement of the chain, the score load, or a named loop-invariant)."""
    order, seen, s_lds = [], {}, []

    def visit(name):
        d = defs.get(name)
        if d is None or id(d) not in in_loop:
            return ("outer", name)
        if id(d) in seen:
            return ("step", seen[id(d)])
        k = type(d).__name__
        if k == "Load":
            if d.input != s_input:
                raise NotImplementedError("a load other than the score in the score transform")
            s_lds.append(d)
            return ("score",)
        if k == "Assign":
            args = tuple(visit(a) for a in d.args)
            sig = ("Assign", d.op.name, getattr(d.dtype, "name", None), args)
        elif k == "Let":
            sig = ("Let", repr(d.value), getattr(d.dtype, "name", None))
        else:
            raise NotImplementedError(f"{k} in the score transform")
        seen[id(d)] = len(order)
        order.append(sig)
        return ("step", seen[id(d)])
    visit(root)
    if len({id(x) for x in s_lds}) != 1:
        raise NotImplementedError("a score transform that is not fed by one score load")
    return s_lds[0], tuple(order)


def _tile_points(tile, limit: int = 1 << 14):
    """Values of the tile's axes to evaluate index expressions at: every combination
    when there are at most ``limit``, else a seeded sample of them."""
    import itertools
    import random
    names = [a.name for a in tile.axes]
    ext = [int(a.extent.value) for a in tile.axes]
    if math.prod(ext) <= limit:
        return [dict(zip(names, c)) for c in itertools.product(*(range(e) for e in ext))]
    rng = random.Random(0)
    return [{n: rng.randrange(e) for n, e in zip(names, ext)} for _ in range(limit)]


def _check_copies(tile, walk, defs, in_loop, maxes, chain, s_ld, v_input: str) -> None:
    """The IR unrolls rows and value columns into register copies (c<row>_<col>); the
    template lowers the first copy's score transform for every row and writes o[row, c]
    from s[row, :] and v[:, c].  So every copy must apply the same transform to its score
    load, and every Write must put row r's result, from v column c, at [r, c]: the Write's
    row index equals its score load's row index and its column index its v element's
    column, at every point of the tile."""
    from ..stmts import eval_index
    first = _chain_signature(maxes[0][0].value, defs, in_loop, s_ld.input)
    for acc, _ in maxes[1:]:
        _, sig = _chain_signature(acc.value, defs, in_loop, s_ld.input)
        if sig != first[1]:
            raise NotImplementedError("register copies with different score transforms")
    accums = {st.name: st for st, _ in walk if type(st).__name__ == "Accum"}
    points = _tile_points(tile)
    for w, _ in walk:
        if type(w).__name__ != "Write":
            continue
        s_loads, v_elems, todo, seen = set(), set(), list(w.values), set()
        while todo:
            n = todo.pop()
            if n in seen:
                continue
            seen.add(n)
            d = defs.get(n)
            if d is None and n in accums:
                todo.append(accums[n].value)
                continue
            k = type(d).__name__
            if k == "Load":
                if d.input == s_ld.input:
                    s_loads.add(id(d))
                    s_row = d.index[-2]
                elif d.input == v_input:
                    v_elems.add((id(d), d.names.index(n)))
                    v_col, v_pos = d.index[-1], d.names.index(n)
            elif k == "Assign":
                todo.extend(d.args)
        if len(s_loads) != 1 or len(v_elems) != 1:
            raise NotImplementedError("an output element not fed by one score row and one v column")
        for env in points:
            if eval_index(w.index[-2], env) != eval_index(s_row, env) or \
                    eval_index(w.index[-1], env) != eval_index(v_col, env) + v_pos:
                raise NotImplementedError("an output element written away from its score row "
                                          "or value column")


def _lead_group(spec, q_ld, out_indices, k_ld, v_ld) -> int:
    """The batch map between q / o entries and k / v entries, from the loads' leading
    coordinates: every query entry y (row-major over q's leading dims) must read k and v
    entry ``y // G`` for one G (1 for plain attention; the head group of grouped-query
    attention, ``k.repeat_interleave(G, dim=1)``, which the IR indexes as ``h / G``)."""
    from ..stmts import eval_index
    Q, K, V = (spec.param(ld.input) for ld in (q_ld, k_ld, v_ld))
    ql, nl = tuple(Q.shape[:-2]), len(Q.shape) - 2
    if tuple(K.shape[:-2]) != tuple(V.shape[:-2]) or len(K.shape) - 2 != nl:
        raise NotImplementedError("k / v batch dims differ")
    qe = q_ld.index[:nl]
    if any(repr(tuple(ix[:nl])) != repr(tuple(qe)) for ix in out_indices):
        raise NotImplementedError("output rows not q's rows")
    nq, nk = math.prod(ql), math.prod(K.shape[:-2])
    if nq % nk:
        raise NotImplementedError("query entries not a multiple of key entries")
    G = nq // nk
    for y in range(nq):
        coords, r = [], y
        for d in reversed(ql):
            coords.append(r % d)
            r //= d
        coords.reverse()
        env = {}
        for e, c in zip(qe, coords):
            k = type(e).__name__
            if k == "Var":
                if env.get(e.name, c) != c:
                    raise NotImplementedError("q's leading index repeats a variable")
                env[e.name] = c
            elif not (k == "Literal" and int(e.value) == c):
                raise NotImplementedError("q's leading index is not one variable per dim")
        for ld in (k_ld, v_ld):
            try:
                kc = [eval_index(e, env) for e in ld.index[:nl]]
            except KeyError:
                raise NotImplementedError("k / v leading index uses other variables") from None
            flat = 0
            for c, d in zip(kc, K.shape[:-2]):
                if not 0 <= c < d:
                    raise NotImplementedError("k / v leading index out of range")
                flat = flat * d + c
            if flat != y // G:
                raise NotImplementedError("k / v entries not y // G")
    return G


def _esz(dtype: str) -> int:
    return 2 if dtype in _HALF else 4


def _emit_ld(p: Ptx, dtype: str, addr: str, dst: str, pred: str) -> None:
    """dst = buffer element at addr widened to f32, 0 where pred is false."""
    if dtype == "f32":
        p.emit(f"mov.f32 {dst}, 0f00000000\n@{pred} ld.global.nc.f32 {dst}, [{addr}]")
    else:
        h = p.reg("b16")
        p.emit(f"mov.b16 {h}, 0\n@{pred} ld.global.nc.b16 {h}, [{addr}]\ncvt.f32.{dtype} {dst}, {h}")


def _score_ctx(p: Ptx, spec):
    """The element-map statement lowering for the score transform: 16-bit results rounded
    per op as the IR states; loads are the prelude's 1-element reads."""
    from ..stmts import ScalarCtx, eval_index, flat_offset

    def on_load(ctx, ld):
        q = spec.param(ld.input)
        off = flat_offset(tuple(ld.index), q.shape, {})
        a, r = p.reg("b64"), p.reg("f32")
        p.emit(f"add.s64 {a}, {load_pointer(p, q.name)}, {off * _esz(q.dtype)}")
        t = p.reg("pred")
        p.emit(f"setp.eq.u32 {t}, 0, 0")
        _emit_ld(p, q.dtype, a, r, t)
        ctx.env[ld.names[0]] = Val(r, "f32")
    ctx = ScalarCtx(p, constants=dict(spec.constants), half_results=True,
                    const_dtypes={q.name: q.dtype for q in spec.params})
    ctx.on_load = on_load
    return ctx


def smem_layout(cfg: F32AttnConfig) -> dict:
    """Byte offsets in dynamic shared memory (each region 16-byte aligned)."""
    ks = 0
    vs = ks + (cfg.D * cfg.KC if cfg.kt else cfg.KC * cfg.DK) * 4
    vs = -(-vs // 16) * 16
    qs = vs + cfg.KC * cfg.Dv * 4
    qs = -(-qs // 16) * 16
    ps = qs + WARPS * cfg.R * cfg.DP * 4
    end = ps + WARPS * cfg.R * cfg.KC * 4
    return {"ks": ks, "vs": vs, "qs": qs, "ps": ps, "bytes": end}


def emit_attention_f32(spec) -> str:
    return emit_module(spec, analyze(spec))


def emit_module(spec, cfg: F32AttnConfig) -> str:
    p = Ptx()
    T, R, KC, KPL, NC, D, Dv, DP = WARPS * 32, cfg.R, cfg.KC, cfg.KPL, cfg.NC, cfg.D, cfg.Dv, cfg.DP
    lay = smem_layout(cfg)
    NEG_INF = "0fFF800000"

    tid, lane, warp = p.reg("u32"), p.reg("u32"), p.reg("u32")
    bidx, row0 = p.reg("u32"), p.reg("u32")
    p.emit(f"""
        mov.u32 {tid}, %tid.x
        and.b32 {lane}, {tid}, 31
        shr.u32 {warp}, {tid}, 5
        mov.u32 {bidx}, %ctaid.y
        mov.u32 {row0}, %ctaid.x
        mad.lo.u32 {row0}, {row0}, {WARPS}, {warp}
        mul.lo.u32 {row0}, {row0}, {R}
    """)
    score = cfg.scores is not None
    ptr = {n: load_pointer(p, n) for n in ((cfg.scores,) if score else (cfg.q, cfg.k)) + (cfg.v, cfg.o)}

    def batch_base(name, per):
        off = p.reg("u64")
        p.emit(f"mul.wide.u32 {off}, {bidx}, {per * _esz(cfg.dt(name))}\n"
               f"add.s64 {ptr[name]}, {ptr[name]}, {off}")
    batch_base(cfg.scores if score else cfg.q, cfg.Sq * (cfg.Sk if score else D))
    batch_base(cfg.o, cfg.Sq * Dv)
    if cfg.group > 1:
        p.emit(f"div.u32 {bidx}, {bidx}, {cfg.group}")
    if not score:
        batch_base(cfg.k, D * cfg.Sk)
    batch_base(cfg.v, cfg.Sk * Dv)

    # the score multiplier c; or (score input) the IR's loop-invariant statements, run once
    sc = p.reg("f32")
    ctx = None
    if score:
        ctx = _score_ctx(p, spec)
        lower_body(ctx, cfg.prelude)
    elif cfg.scale_param is not None:
        sp = load_pointer(p, cfg.scale_param)
        p.emit(f"ld.global.nc.f32 {sc}, [{sp}]")
        if cfg.scale_recip:
            p.emit(f"rcp.rn.f32 {sc}, {sc}")
    else:
        p.emit(f"mov.f32 {sc}, {f32_hex(cfg.scale_const)}")

    # shared-memory bases (32-bit shared addresses)
    sbase = p.reg("u32")
    p.emit(f"mov.u32 {sbase}, dsmem")
    ks_lane, vs_lane, qw, pw, pwl = (p.reg("u32") for _ in range(5))
    t0 = p.reg("u32")
    # a lane's key column: kt chunk [D][KC] -> 4 lane; key-major chunk [KC][DK] -> 4 DK lane
    p.emit(f"""
        mul.lo.u32 {t0}, {lane}, {4 if cfg.kt else 4 * cfg.DK}
        add.u32 {ks_lane}, {sbase}, {lay['ks']}
        add.u32 {ks_lane}, {ks_lane}, {t0}
        shl.b32 {t0}, {lane}, 2
        add.u32 {vs_lane}, {sbase}, {lay['vs']}
        add.u32 {vs_lane}, {vs_lane}, {t0}
        mad.lo.u32 {qw}, {warp}, {R * DP * 4}, {sbase}
        add.u32 {qw}, {qw}, {lay['qs']}
        mad.lo.u32 {pw}, {warp}, {R * KC * 4}, {sbase}
        add.u32 {pw}, {pw}, {lay['ps']}
        add.u32 {pwl}, {pw}, {t0}
    """)

    # ---- the warp's q rows into shared memory (zero past Sq and past D)
    for r in range(R if not score else 0):
        row, prow = p.reg("u32"), p.reg("pred")
        p.emit(f"add.u32 {row}, {row0}, {r}\nsetp.lt.u32 {prow}, {row}, {cfg.Sq}")
        for i in range(-(-DP // 32)):
            d = p.reg("u32")
            val, pd, pst, a64 = p.reg("f32"), p.reg("pred"), p.reg("pred"), p.reg("u64")
            p.emit(f"""
                add.u32 {d}, {lane}, {32 * i}
                setp.lt.and.u32 {pd}, {d}, {D}, {prow}
                setp.lt.u32 {pst}, {d}, {DP}
                mov.f32 {val}, 0f00000000
                mad.lo.u32 {t0}, {row}, {D}, {d}
                mul.wide.u32 {a64}, {t0}, 4
                add.s64 {a64}, {ptr[cfg.q]}, {a64}
                @{pd} ld.global.nc.f32 {val}, [{a64}]
                shl.b32 {t0}, {d}, 2
                add.u32 {t0}, {t0}, {qw}
                @{pst} st.shared.f32 [{t0}+{r * DP * 4}], {val}
            """)

    # running state
    m = [p.reg("f32") for _ in range(R)]
    l = [p.reg("f32") for _ in range(R)]
    o = [[p.reg("f32") for _ in range(NC)] for _ in range(R)]
    for r in range(R):
        p.emit(f"mov.f32 {m[r]}, {NEG_INF}\nmov.f32 {l[r]}, 0f00000000")
        for i in range(NC):
            p.emit(f"mov.f32 {o[r][i]}, 0f00000000")
    pcol = []
    for i in range(NC):
        pc = p.reg("pred")
        p.emit(f"add.u32 {t0}, {lane}, {32 * i}\nsetp.lt.u32 {pc}, {t0}, {Dv}")
        pcol.append(pc)
    vv = [p.reg("f32") for _ in range(NC)]
    for i in range(NC):
        p.emit(f"mov.f32 {vv[i]}, 0f00000000")

    # staging geometry: kt chunk [D][KC] and v chunk [KC][Dv]
    key0 = p.reg("u32")
    p.emit(f"mov.u32 {key0}, 0")
    top = p.label("chunk")
    p.place(top)
    p.emit("bar.sync 0")
    _stage(p, cfg, ptr, tid, key0, sbase, lay, T)
    p.emit("bar.sync 0")

    # ---- scores for the chunk: acc[r][k] = q_r . kt[:, key0 + lane + 32k] (or read from s)
    acc = [[p.reg("f32") for _ in range(KPL)] for _ in range(R)]
    for r in range(R):
        for k in range(KPL):
            p.emit(f"mov.f32 {acc[r][k]}, 0f00000000")
    if score:
        sdt = cfg.dt(cfg.scores)
        for r in range(R):
            for k in range(KPL):
                pk, a64 = p.reg("pred"), p.reg("u64")
                p.emit(f"""
                    add.u32 {t0}, {row0}, {r}
                    setp.lt.u32 {pk}, {t0}, {cfg.Sq}
                    mad.lo.u32 {t0}, {t0}, {cfg.Sk}, {key0}
                    add.u32 {t0}, {t0}, {lane}
                    add.u32 {t0}, {t0}, {32 * k}
                    mul.wide.u32 {a64}, {t0}, {_esz(sdt)}
                    add.s64 {a64}, {ptr[cfg.scores]}, {a64}
                """)
                # the key index: lane + 32 k past key0 (predicated on the row and the key)
                pkk = p.reg("pred")
                p.emit(f"add.u32 {t0}, {key0}, {lane}\nadd.u32 {t0}, {t0}, {32 * k}\n"
                       f"setp.lt.and.u32 {pkk}, {t0}, {cfg.Sk}, {pk}")
                _emit_ld(p, sdt, a64, acc[r][k], pkk)
    kv = [p.reg("f32") for _ in range(KPL)]
    qv = [[p.reg("f32") for _ in range(4)] for _ in range(R)]
    for d0 in range(0, D if not score else 0, 4):
        for r in range(R):
            p.emit(f"ld.shared.v4.f32 {{{', '.join(qv[r])}}}, [{qw}+{(r * DP + d0) * 4}]")
        for dd in range(min(4, D - d0)):
            d = d0 + dd
            for k in range(KPL):
                off = d * KC + 32 * k if cfg.kt else 32 * k * cfg.DK + d
                p.emit(f"ld.shared.f32 {kv[k]}, [{ks_lane}+{off * 4}]")
            for r in range(R):
                for k in range(KPL):
                    p.emit(f"fma.rn.f32 {acc[r][k]}, {qv[r][dd]}, {kv[k]}, {acc[r][k]}")

    # ---- online softmax per row; p to the warp's shared row
    kvalid = []
    for k in range(KPL):
        pk = p.reg("pred")
        p.emit(f"add.u32 {t0}, {key0}, {lane}\nadd.u32 {t0}, {t0}, {32 * k}\nsetp.lt.u32 {pk}, {t0}, {cfg.Sk}")
        kvalid.append(pk)
    l2e = f32_hex(LOG2E)
    for r in range(R):
        t = [p.reg("f32") for _ in range(KPL)]
        cm, sh, mn, alpha, ps_sum = p.reg("f32"), p.reg("f32"), p.reg("f32"), p.reg("f32"), p.reg("f32")
        for k in range(KPL):
            if score:
                saved = dict(ctx.env)
                ctx.env[cfg.s_name] = Val(acc[r][k], "f32")
                lower_body(ctx, cfg.s_chain)
                p.emit(f"mov.f32 {t[k]}, {ctx.f32(cfg.s_out)}")
                ctx.env = saved
            else:
                p.emit(f"mul.rn.f32 {t[k]}, {acc[r][k]}, {sc}")
            p.emit(f"selp.f32 {t[k]}, {t[k]}, {NEG_INF}, {kvalid[k]}")
        p.emit(f"mov.f32 {cm}, {t[0]}")
        for k in range(1, KPL):
            p.emit(f"max.f32 {cm}, {cm}, {t[k]}")
        for off in (16, 8, 4, 2, 1):
            p.emit(f"shfl.sync.bfly.b32 {sh}, {cm}, {off}, 31, 0xffffffff\nmax.f32 {cm}, {cm}, {sh}")
        p.emit(f"""
            max.f32 {mn}, {m[r]}, {cm}
            sub.f32 {alpha}, {m[r]}, {mn}
            mul.rn.f32 {alpha}, {alpha}, {l2e}
            ex2.approx.f32 {alpha}, {alpha}
            mov.f32 {m[r]}, {mn}
            mov.f32 {ps_sum}, 0f00000000
        """)
        for k in range(KPL):
            p.emit(f"""
                sub.f32 {t[k]}, {t[k]}, {mn}
                mul.rn.f32 {t[k]}, {t[k]}, {l2e}
                ex2.approx.f32 {t[k]}, {t[k]}
                add.f32 {ps_sum}, {ps_sum}, {t[k]}
                st.shared.f32 [{pwl}+{(r * KC + 32 * k) * 4}], {t[k]}
            """)
        p.emit(f"fma.rn.f32 {l[r]}, {l[r]}, {alpha}, {ps_sum}")
        for i in range(NC):
            p.emit(f"mul.rn.f32 {o[r][i]}, {o[r][i]}, {alpha}")
    p.emit("bar.warp.sync 0xffffffff")

    # ---- o += p v over the chunk's keys
    pv = [[p.reg("f32") for _ in range(4)] for _ in range(R)]
    for j0 in range(0, KC, 4):
        for r in range(R):
            p.emit(f"ld.shared.v4.f32 {{{', '.join(pv[r])}}}, [{pw}+{(r * KC + j0) * 4}]")
        for jj in range(4):
            j = j0 + jj
            for i in range(NC):
                p.emit(f"@{pcol[i]} ld.shared.f32 {vv[i]}, [{vs_lane}+{(j * Dv + 32 * i) * 4}]")
            for r in range(R):
                for i in range(NC):
                    p.emit(f"fma.rn.f32 {o[r][i]}, {pv[r][jj]}, {vv[i]}, {o[r][i]}")
    pl = p.reg("pred")
    p.emit(f"add.u32 {key0}, {key0}, {KC}\nsetp.lt.u32 {pl}, {key0}, {cfg.Sk}\n@{pl} bra {top}")

    # ---- epilogue: o / l
    for r in range(R):
        sh, row, prow = p.reg("f32"), p.reg("u32"), p.reg("pred")
        for off in (16, 8, 4, 2, 1):
            p.emit(f"shfl.sync.bfly.b32 {sh}, {l[r]}, {off}, 31, 0xffffffff\nadd.f32 {l[r]}, {l[r]}, {sh}")
        p.emit(f"add.u32 {row}, {row0}, {r}\nsetp.lt.u32 {prow}, {row}, {cfg.Sq}")
        for i in range(NC):
            ps_, a64, res = p.reg("pred"), p.reg("u64"), p.reg("f32")
            p.emit(f"""
                and.pred {ps_}, {prow}, {pcol[i]}
                div.rn.f32 {res}, {o[r][i]}, {l[r]}
                mad.lo.u32 {t0}, {row}, {Dv}, {lane}
                add.u32 {t0}, {t0}, {32 * i}
                mul.wide.u32 {a64}, {t0}, {_esz(cfg.dt(cfg.o))}
                add.s64 {a64}, {ptr[cfg.o]}, {a64}
            """)
            if cfg.dt(cfg.o) == "f32":
                p.emit(f"@{ps_} st.global.f32 [{a64}], {res}")
            else:
                h = p.reg("b16")
                p.emit(f"cvt.rn.{cfg.dt(cfg.o)}.f32 {h}, {res}\n@{ps_} st.global.b16 [{a64}], {h}")
    p.emit("ret")

    grid = [-(-cfg.Sq // (WARPS * R)), cfg.B, 1]
    flops = 2 * cfg.B * cfg.Sq * cfg.Sk * (D + Dv)
    launch = {"kind": "attention_f32", "grid": grid, "block": [T, 1, 1], "cluster": [1, 1, 1],
              "smem": lay["bytes"], "extra_params": [], "flops": flops}
    return module([entry(spec.name, arg_params(spec), p, maxntid=T)], launch,
                  globals_=[".extern .shared .align 16 .b8 dsmem[];"])


def _stage(p: Ptx, cfg: F32AttnConfig, ptr: dict, tid: str, key0: str, sbase: str, lay: dict,
           T: int) -> None:
    """Copy the chunk's keys [key0, key0 + KC) of k and v into shared memory, zero past
    Sk.  128-bit global loads when rows are whole float4s; loads batched 16 deep."""
    KC, D, Sk = cfg.KC, cfg.D, cfg.Sk
    w = 4 if cfg.vec else 1
    nk = p.reg("u32")
    p.emit(f"sub.u32 {nk}, {Sk}, {key0}")
    ops = []        # (load predicate, store predicate, global address, [shared addresses])
    if cfg.scores is not None:
        pass                  # scores come from the score buffer, not from k
    elif cfg.kt:
        # kt [D][Sk]: unit e = tid + T it over [D][KC / w]; T is a multiple of KC / w
        per_row = KC // w
        rows_per_pass = T // per_row
        dt, jt = p.reg("u32"), p.reg("u32")
        p.emit(f"""
            shr.u32 {dt}, {tid}, {per_row.bit_length() - 1}
            and.b32 {jt}, {tid}, {per_row - 1}
            mul.lo.u32 {jt}, {jt}, {w}
        """)
        pkey, gk = p.reg("pred"), p.reg("u32")
        p.emit(f"setp.lt.u32 {pkey}, {jt}, {nk}\nadd.u32 {gk}, {key0}, {jt}")
        for it in range(-(-D // rows_per_pass)):
            d, pr, pst = p.reg("u32"), p.reg("pred"), p.reg("pred")
            ga, sa, t = p.reg("u64"), p.reg("u32"), p.reg("u32")
            p.emit(f"""
                add.u32 {d}, {dt}, {it * rows_per_pass}
                setp.lt.and.u32 {pr}, {d}, {D}, {pkey}
                setp.lt.u32 {pst}, {d}, {D}
                mad.lo.u32 {t}, {d}, {Sk}, {gk}
                mul.wide.u32 {ga}, {t}, 4
                add.s64 {ga}, {ptr[cfg.k]}, {ga}
                mad.lo.u32 {sa}, {d}, {KC}, {jt}
                shl.b32 {sa}, {sa}, 2
                add.u32 {sa}, {sa}, {sbase}
            """)
            ops.append((pr, pst, ga, [f"{sa}+{lay['ks']}"]))
    else:
        # key-major k: rows of D floats, stored with the odd stride DK
        ops += _span(p, cfg, ptr[cfg.k], tid, key0, nk, sbase, lay["ks"], D, cfg.DK, T, w)
    vops = _span(p, cfg, ptr[cfg.v], tid, key0, nk, sbase, lay["vs"], cfg.Dv, cfg.Dv, T, w,
                 _esz(cfg.dt(cfg.v)))
    if cfg.dt(cfg.v) != "f32":      # 16-bit v: element loads widened to f32 in shared memory
        for pr, pst, ga, sas in vops:
            x = p.reg("f32")
            _emit_ld(p, cfg.dt(cfg.v), ga, x, pr)
            p.emit(f"@{pst} st.shared.f32 [{sas[0]}], {x}")
        vops = []
    ops += vops
    sfx = ".v4.f32" if w == 4 else ".f32"
    for b0 in range(0, len(ops), 16):
        batch = ops[b0:b0 + 16]
        vals = []
        for pr, _, ga, _ in batch:
            v = [p.reg("f32") for _ in range(w)]
            p.emit("\n".join(f"mov.f32 {x}, 0f00000000" for x in v))
            p.emit(f"@{pr} ld.global.nc{sfx} {'{' + ', '.join(v) + '}' if w == 4 else v[0]}, [{ga}]")
            vals.append(v)
        for (_, pst, _, sas), v in zip(batch, vals):
            if len(sas) == 1 and w == 4:
                p.emit(f"@{pst} st.shared.v4.f32 [{sas[0]}], {{{', '.join(v)}}}")
            else:
                for sa, x in zip(sas, v):
                    p.emit(f"@{pst} st.shared.f32 [{sa}], {x}")


def _span(p: Ptx, cfg: F32AttnConfig, gptr: str, tid: str, key0: str, nk: str, sbase: str,
          soff: int, width: int, sstride: int, T: int, w: int, esz: int = 4) -> list:
    """Staging ops for rows [key0, key0 + KC) of a [.., Sk, width] buffer: one contiguous
    span of global memory; in shared memory row j starts at j * sstride (floats)."""
    KC = cfg.KC
    nv = p.reg("u32")
    p.emit(f"min.u32 {nv}, {nk}, {KC}\nmul.lo.u32 {nv}, {nv}, {width}")
    base = p.reg("u64")
    p.emit(f"mul.wide.u32 {base}, {key0}, {width * esz}\nadd.s64 {base}, {gptr}, {base}")
    ops = []
    for it in range(-(-(KC * width // w) // T)):
        e, pr, pst = p.reg("u32"), p.reg("pred"), p.reg("pred")
        ga, sa = p.reg("u64"), p.reg("u32")
        p.emit(f"""
            add.u32 {e}, {tid}, {it * T}
            mul.lo.u32 {e}, {e}, {w}
            setp.lt.u32 {pr}, {e}, {nv}
            setp.lt.u32 {pst}, {e}, {KC * width}
            mul.wide.u32 {ga}, {e}, {esz}
            add.s64 {ga}, {base}, {ga}
        """)
        if sstride == width:
            p.emit(f"shl.b32 {sa}, {e}, 2\nadd.u32 {sa}, {sa}, {sbase}")
            ops.append((pr, pst, ga, [f"{sa}+{soff}"]))
        else:
            # element e sits in row e / width: shift it by that many pad floats (a float4
            # never straddles rows: width is a multiple of w)
            j = p.reg("u32")
            p.emit(f"div.u32 {j}, {e}, {width}\nmad.lo.u32 {sa}, {j}, {sstride - width}, {e}\n"
                   f"shl.b32 {sa}, {sa}, 2\nadd.u32 {sa}, {sa}, {sbase}")
            ops.append((pr, pst, ga, [f"{sa}+{soff + 4 * c}" for c in range(w)]))
    return ops
