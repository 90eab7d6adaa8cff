"""Statement registry and scalar lowering.

Keeps the reference's dispatch surface (``compiler/stmts.py:23-41``): a module-level
``HANDLERS`` table filled by the ``@handles("Kind")`` decorator, dispatched on
``type(stmt).__name__``, with unknown kinds raising
``NotImplementedError(f"statement {kind}")``.

What differs is who owns the schedule.  The reference lowers every statement in
emmy's sm_89 schedule.  Here a kernel template (``compiler/kernels``) owns the
launch, the memory movement and the cross-thread combines, and calls
:func:`lower_body` only for the IR's *scalar* statements -- the per-element map
before an accumulation, the accumulator updates, the per-row tail and the
per-element output expression.  Those statements are lowered exactly as the IR
states them, so the template computes the IR's own arithmetic.

Loads and writes are routed through hooks the template installs on the context,
because the template decides how an element's address maps to registers (a
vector lane of a 128-bit load, a value cached from an earlier pass, a constant
folded to an immediate).
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Callable

from .ptx import Ptx, f32_hex, f64_hex

HANDLERS: dict[str, Callable] = {}


def handles(*kinds: str):
    """Register ``fn(ctx, stmt)`` as the lowering of statement kind(s)."""
    def deco(fn):
        for k in kinds:
            HANDLERS[k] = fn
        return fn
    return deco


def lower_body(ctx, body) -> None:
    for s in body:
        kind = type(s).__name__
        fn = HANDLERS.get(kind)
        if fn is None:
            raise NotImplementedError(f"statement {kind}")
        fn(ctx, s)


def dtype_name(dt) -> str | None:
    if dt is None:
        return None
    return getattr(dt, "name", dt)


# --------------------------------------------------------------------------
# values and the scalar context


@dataclass
class Val:
    text: str          # register name or immediate
    kind: str          # "f32" | "s32" | "pred"
    const: float | None = None
    nonpos: bool = False   # known <= 0 (an element minus the row maximum)
    diff: tuple | None = None   # (element register, max state) when the value is their difference


@dataclass
class ScalarCtx:
    ptx: Ptx
    env: dict = field(default_factory=dict)          # SSA name -> Val
    mutable: set = field(default_factory=set)        # names updated in place (accumulators)
    constants: dict = field(default_factory=dict)    # ConstantOp buffer -> value
    on_load: Callable | None = None                  # fn(ctx, Load) -> None (binds names)
    on_write: Callable | None = None                 # fn(ctx, Write) -> None
    axis_regs: dict = field(default_factory=dict)    # axis name -> s32 register / immediate
    max_states: set = field(default_factory=set)     # accumulators holding a row maximum
    exp_reuse: Callable | None = None                # fn(element register, max state) -> register
    half_results: bool = False                       # f16 / bf16 results rounded per op (else rejected)
    exact_products: bool = False                     # a matmul kernel: 16-bit products stay exact
    index_vars: dict = field(default_factory=dict)   # loaded name -> index variables of its Load
    const_dtypes: dict = field(default_factory=dict) # constant buffer -> IR dtype (i32 / i64 / f64 ...)

    def bind(self, name: str, val: Val) -> None:
        if name in self.mutable and name in self.env:
            dst = self.env[name]
            if dst.text != val.text:
                self.ptx.emit(f"mov.f32 {dst.text}, {val.text}" if dst.kind == "f32"
                              else f"mov.b32 {dst.text}, {val.text}")
            return
        self.env[name] = val

    def get(self, name: str) -> Val:
        try:
            return self.env[name]
        except KeyError:
            raise ValueError(f"IR name {name!r} is used before it is defined") from None

    def f32(self, name: str) -> str:
        v = self.get(name)
        if v.kind == "pred":
            # a bool in arithmetic is 1.0 / 0.0 (torch promotes bool to the float type)
            r = self.ptx.reg("f32")
            self.ptx.emit(f"selp.f32 {r}, 0f3F800000, 0f00000000, {v.text}")
            return r
        if v.kind in ("s32", "s64", "f64"):
            return self.as_kind(name, "f32")
        if v.kind != "f32":
            raise NotImplementedError(f"{name!r} is {v.kind}, expected f32")
        return v.text

    def as_kind(self, name: str, kind: str) -> str:
        """``name``'s value as a ``kind`` register (f32 / f64 / s32 / s64): integers and
        bools promote to floats exactly where they can (nearest otherwise), floats to
        integers truncate toward zero (torch's ``.to(int)``), wide integers narrow by
        dropping high bits."""
        v, p = self.get(name), self.ptx
        if v.kind == kind:
            return v.text
        r = p.reg(kind)
        if v.kind == "pred":
            one, zero = {"f32": ("0f3F800000", "0f00000000"), "f64": ("0d3FF0000000000000", "0d0000000000000000"),
                         "s32": ("1", "0"), "s64": ("1", "0")}[kind]
            p.emit(f"selp.{'b32' if kind in ('f32', 's32') else 'b64'} {r}, {one}, {zero}, {v.text}")
            return r
        if v.const is not None and kind in ("f32", "f64"):
            return f32_hex(v.const) if kind == "f32" else f64_hex(v.const)
        if v.const is not None and kind in ("s32", "s64"):
            return str(int(v.const))
        src = {"f32": "f32", "f64": "f64", "s32": "s32", "s64": "s64"}[v.kind]
        if kind in ("f32", "f64"):
            rnd = "" if (src == "f32" and kind == "f64") else ".rn"
            p.emit(f"cvt{rnd}.{kind}.{src} {r}, {v.text}")
        elif src in ("f32", "f64"):
            p.emit(f"cvt.rzi.{kind}.{src} {r}, {v.text}")
        else:
            p.emit(f"cvt.{kind}.{src} {r}, {v.text}")
        return r

    def pred(self, name: str) -> str:
        v = self.get(name)
        if v.kind != "pred":
            raise NotImplementedError(f"{name!r} is {v.kind}, expected bool")
        return v.text


# --------------------------------------------------------------------------
# f32 elementwise op table (the subset the hot-path kernels use: arithmetic,
# max/min, exp, sqrt, rsqrt, reciprocal).  The reference's table is
# compiler/ops.py:254-414.

_LOG2E_HI = 1.4426950216293335       # float32(log2 e)
_LOG2E_LO = 1.925963033500011e-08    # log2 e - _LOG2E_HI
_LN2 = 0.6931471805599453


def emit_exp_nonpos(p: Ptx, dst: str, x: str) -> None:
    """exp(x) for x <= 0 (an element minus its row maximum): ``ex2.approx`` of the
    rounded product x*log2(e).  The product's rounding adds at most |x| * 2^-24
    relative error to the argument, so for x in [-20, 0] the result is within
    ~1.5e-6 relative (plus ex2.approx's 2 ulp); arguments below -126 flush to 0."""
    t = p.reg("f32")
    p.emit(f"mul.rn.f32 {t}, {x}, {f32_hex(_LOG2E_HI)}\nex2.approx.ftz.f32 {dst}, {t}")


def emit_exp(p: Ptx, dst: str, x: str) -> None:
    """exp(x) = 2^(x log2 e) on the MUFU ``ex2.approx`` unit.

    The product x*log2(e) is formed in two pieces (Cody-Waite style): ``t`` is the
    rounded product with the f32 constant, ``e`` the exact residual of that product
    plus x times the constant's own rounding error.  2^(t+e) = 2^t (1 + e ln 2) to
    first order in e (|e| < 2^-23 |t|), so the result keeps ex2.approx's ~2 ulp
    instead of losing |x log2 e| ulp to the rounding of the product."""
    t, e, lo, r = p.reg("f32"), p.reg("f32"), p.reg("f32"), p.reg("f32")
    p.emit(f"""
        mul.rn.f32 {t}, {x}, {f32_hex(_LOG2E_HI)}
        neg.f32 {e}, {t}
        fma.rn.f32 {e}, {x}, {f32_hex(_LOG2E_HI)}, {e}
        fma.rn.f32 {e}, {x}, {f32_hex(_LOG2E_LO)}, {e}
        ex2.approx.f32 {r}, {t}
        mul.rn.f32 {lo}, {e}, {f32_hex(_LN2)}
        fma.rn.f32 {dst}, {r}, {lo}, {r}
    """)


# erf by Abramowitz & Stegun, Handbook of Mathematical Functions, 7.1.26:
# erf(x) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-x^2), t = 1 / (1 + p x),
# x >= 0, |error| <= 1.5e-7; odd extension for x < 0
_AS_P = 0.3275911
_AS_A = (0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)


def emit_erf(p: Ptx, dst: str, x: str) -> None:
    ax, t, q, e, x2, r = (p.reg("f32") for _ in range(6))
    p.emit(f"""
        abs.f32 {ax}, {x}
        fma.rn.f32 {t}, {ax}, {f32_hex(_AS_P)}, 0f3F800000
        rcp.rn.f32 {t}, {t}
        fma.rn.f32 {q}, {t}, {f32_hex(_AS_A[4])}, {f32_hex(_AS_A[3])}
        fma.rn.f32 {q}, {q}, {t}, {f32_hex(_AS_A[2])}
        fma.rn.f32 {q}, {q}, {t}, {f32_hex(_AS_A[1])}
        fma.rn.f32 {q}, {q}, {t}, {f32_hex(_AS_A[0])}
        mul.rn.f32 {q}, {q}, {t}
        mul.rn.f32 {x2}, {ax}, {ax}
        neg.f32 {x2}, {x2}
    """)
    emit_exp(p, e, x2)
    p.emit(f"""
        neg.f32 {q}, {q}
        fma.rn.f32 {r}, {q}, {e}, 0f3F800000
        copysign.f32 {dst}, {x}, {r}
    """)


# tanh x = x + c3 x^3 + ... + c17 x^17 + ...: its Taylor series, c(2n-1) =
# 2^(2n) (2^(2n) - 1) B(2n) / (2n)! with B the Bernoulli numbers (-1/3, 2/15, -17/315, ...)
_TANH_C = (-0.3333333333333333, 0.13333333333333333, -0.05396825396825397, 0.021869488536155203, -0.008863235529902197, 0.003592128036572481, -0.0014558343870513183, 0.000590027440945586)
_TANH_SERIES_MAX = 0.55      # below: the series (next term < 1e-8 relative); above: via exp


def emit_tanh(p: Ptx, dst: str, x: str) -> None:
    """tanh x: for |x| < 0.55 the odd Taylor series to x^17 (Horner in x^2, error a few
    ulp); above, 1 - 2 / (exp(2|x|) + 1) with this back end's exp (no cancellation:
    the subtracted term is at most 1/2 of the result); the sign restored last."""
    ax, x2, q, e, r, big = (p.reg("f32") for _ in range(6))
    ps = p.reg("pred")
    p.emit(f"abs.f32 {ax}, {x}\nmul.rn.f32 {x2}, {x}, {x}\nmov.f32 {q}, {f32_hex(_TANH_C[-1])}")
    for c in reversed(_TANH_C[:-1]):
        p.emit(f"fma.rn.f32 {q}, {q}, {x2}, {f32_hex(c)}")
    p.emit(f"mul.rn.f32 {q}, {q}, {x2}\nfma.rn.f32 {q}, {q}, {ax}, {ax}\nadd.rn.f32 {e}, {ax}, {ax}")
    emit_exp(p, e, e)
    p.emit(f"""
        add.rn.f32 {e}, {e}, 0f3F800000
        div.rn.f32 {big}, 0f40000000, {e}
        sub.rn.f32 {big}, 0f3F800000, {big}
        setp.lt.f32 {ps}, {ax}, {f32_hex(_TANH_SERIES_MAX)}
        selp.f32 {r}, {q}, {big}, {ps}
        copysign.f32 {dst}, {x}, {r}
    """)


def emit_sigmoid(p: Ptx, dst: str, x: str) -> None:
    """1 / (1 + exp(-x)): exp(-x) overflows to inf for x < -88, giving 0 as it should."""
    n = p.reg("f32")
    p.emit(f"neg.f32 {n}, {x}")
    emit_exp(p, n, n)
    p.emit(f"add.rn.f32 {n}, {n}, 0f3F800000\nrcp.rn.f32 {dst}, {n}")


# pi / 2 (from Machin's formula pi = 16 atan(1/5) - 4 atan(1/239)) in three parts; the first
# two keep 12 mantissa bits, so k * part is exact for |k| < 2^11 (|x| below ~3200)
_PIO2 = (1.570556640625, 0.0002396702766418457, 1.5893254712295857e-08)
_TWO_OVER_PI = 0.6366197723675814
# Taylor coefficients: sin r = r + r (r^2 S1 + r^4 S2 + ...), cos r = 1 + r^2 C1 + r^4 C2 + ...
_SIN_C = (-0.16666666666666666, 0.008333333333333333, -0.0001984126984126984, 2.7557319223985893e-06, -2.505210838544172e-08)          # (-1)^k / (2k+1)!, k = 1..5
_COS_C = (-0.5, 0.041666666666666664, -0.001388888888888889, 2.48015873015873e-05, -2.755731922398589e-07, 2.08767569878681e-09)          # (-1)^k / (2k)!,   k = 1..6


def emit_sincos(p: Ptx, dst: str, x: str, cos: bool) -> None:
    """sin x / cos x written here from the definitions: x = k pi/2 + r with |r| <= pi/4
    (Cody-Waite, pi/2 in three parts), then the Taylor series of sin r or cos r (to r^11 /
    r^12, truncation below 2e-9) picked and signed by the quadrant k mod 4 (cos x =
    sin(x + pi/2): the quadrant of k + 1)."""
    kf, r, r2, sp, cp, res = (p.reg("f32") for _ in range(6))
    k = p.reg("s32")
    p1, p2, p3 = p.reg("pred"), p.reg("pred"), p.reg("pred")
    q, qb = p.reg("b32"), p.reg("b32")
    p.emit(f"""
        mul.rn.f32 {kf}, {x}, {f32_hex(_TWO_OVER_PI)}
        cvt.rni.f32.f32 {kf}, {kf}
        cvt.rni.s32.f32 {k}, {kf}
        neg.f32 {r}, {kf}
        fma.rn.f32 {r}, {r}, {f32_hex(_PIO2[0])}, {x}
        neg.f32 {res}, {kf}
        fma.rn.f32 {r}, {res}, {f32_hex(_PIO2[1])}, {r}
        fma.rn.f32 {r}, {res}, {f32_hex(_PIO2[2])}, {r}
        mul.rn.f32 {r2}, {r}, {r}
        mov.f32 {sp}, {f32_hex(_SIN_C[-1])}
    """)
    for c in reversed(_SIN_C[:-1]):
        p.emit(f"fma.rn.f32 {sp}, {sp}, {r2}, {f32_hex(c)}")
    p.emit(f"mul.rn.f32 {sp}, {sp}, {r2}\nfma.rn.f32 {sp}, {sp}, {r}, {r}\nmov.f32 {cp}, {f32_hex(_COS_C[-1])}")
    for c in reversed(_COS_C[:-1]):
        p.emit(f"fma.rn.f32 {cp}, {cp}, {r2}, {f32_hex(c)}")
    p.emit(f"""
        fma.rn.f32 {cp}, {cp}, {r2}, 0f3F800000
        add.s32 {q}, {k}, {1 if cos else 0}
        and.b32 {q}, {q}, 3
        and.b32 {qb}, {q}, 1
        setp.ne.b32 {p1}, {qb}, 0
        selp.f32 {res}, {cp}, {sp}, {p1}
        and.b32 {q}, {q}, 2
        setp.ne.b32 {p2}, {q}, 0
        neg.f32 {dst}, {res}
        selp.f32 {dst}, {dst}, {res}, {p2}
        setp.nan.f32 {p3}, {x}, {x}
        @{p3} mov.f32 {dst}, {x}
    """)


def emit_pow(p: Ptx, dst: str, x: str, y: str) -> None:
    """x^y = 2^(y log2 |x|) on the MUFU units (error ~ |y log2 x| * 2^-22 relative), with
    torch's special cases: x^0 = 1 and 1^y = 1, a negative x only with an integral y
    (negative for an odd one), NaN otherwise."""
    ax, l, e, yi, hy, hi = (p.reg("f32") for _ in range(6))
    pint, podd, pneg, pz, p1, pnan = (p.reg("pred") for _ in range(6))
    p.emit(f"""
        abs.f32 {ax}, {x}
        lg2.approx.f32 {l}, {ax}
        mul.rn.f32 {l}, {l}, {y}
        ex2.approx.f32 {e}, {l}
        cvt.rzi.f32.f32 {yi}, {y}
        setp.eq.f32 {pint}, {yi}, {y}
        mul.rn.f32 {hy}, {y}, 0f3F000000
        cvt.rzi.f32.f32 {hi}, {hy}
        setp.ne.and.f32 {podd}, {hi}, {hy}, {pint}
        setp.lt.f32 {pneg}, {x}, 0f00000000
        mov.f32 {dst}, {e}
        and.pred {podd}, {podd}, {pneg}
        @{podd} neg.f32 {dst}, {e}
        not.pred {pnan}, {pint}
        and.pred {pnan}, {pnan}, {pneg}
        @{pnan} mov.f32 {dst}, 0f7FFFFFFF
        setp.eq.f32 {pz}, {y}, 0f00000000
        setp.eq.f32 {p1}, {x}, 0f3F800000
        or.pred {pz}, {pz}, {p1}
        @{pz} mov.f32 {dst}, 0f3F800000
    """)


def _unary(p: Ptx, op: str, dst: str, a: str) -> None:
    if op == "copy":
        p.emit(f"mov.f32 {dst}, {a}")
    elif op == "negative":
        p.emit(f"neg.f32 {dst}, {a}")
    elif op == "abs":
        p.emit(f"abs.f32 {dst}, {a}")
    elif op == "exp":
        emit_exp(p, dst, a)
    elif op == "sqrt":
        p.emit(f"sqrt.rn.f32 {dst}, {a}")
    elif op == "reciprocal":
        p.emit(f"rcp.rn.f32 {dst}, {a}")
    elif op == "rsqrt":
        # 1/sqrt(x) from the two IEEE-rounded instructions (both correctly rounded),
        # as the reference lowers it (compiler/ops.py:88-92).
        s = p.reg("f32")
        p.emit(f"sqrt.rn.f32 {s}, {a}\nrcp.rn.f32 {dst}, {s}")
    elif op == "relu":
        p.emit(f"max.f32 {dst}, {a}, 0f00000000")
    elif op == "square":
        p.emit(f"mul.rn.f32 {dst}, {a}, {a}")
    elif op == "erf":
        emit_erf(p, dst, a)
    elif op == "tanh":
        emit_tanh(p, dst, a)
    elif op in ("sin", "cos"):
        emit_sincos(p, dst, a, op == "cos")
    elif op == "sigmoid":
        emit_sigmoid(p, dst, a)
    elif op == "log":
        # ln x = log2(x) * ln 2 on the MUFU lg2 unit (about 2^-22 absolute error for
        # x in [1/2, 2], a few ulp relative elsewhere)
        l2 = p.reg("f32")
        p.emit(f"lg2.approx.f32 {l2}, {a}\nmul.rn.f32 {dst}, {l2}, {f32_hex(_LN2)}")
    else:
        raise NotImplementedError(f"elementwise op {op} (f32, unary)")


def _binary(p: Ptx, op: str, dst: str, a: str, b: str) -> None:
    if op == "add":
        p.emit(f"add.rn.f32 {dst}, {a}, {b}")
    elif op == "subtract":
        p.emit(f"sub.rn.f32 {dst}, {a}, {b}")
    elif op == "multiply":
        p.emit(f"mul.rn.f32 {dst}, {a}, {b}")
    elif op == "divide":
        p.emit(f"div.rn.f32 {dst}, {a}, {b}")
    elif op == "maximum":
        p.emit(f"max.f32 {dst}, {a}, {b}")
    elif op == "minimum":
        p.emit(f"min.f32 {dst}, {a}, {b}")
    elif op == "pow":
        emit_pow(p, dst, a, b)
    else:
        raise NotImplementedError(f"elementwise op {op} (f32, binary)")


def compute_f32(ctx: ScalarCtx, op: str, args: list[str], dst: str | None = None) -> Val:
    p = ctx.ptx
    vals = [ctx.f32(a) for a in args]
    out = dst or p.reg("f32")
    if op == "subtract" and len(args) == 2 and args[1] in ctx.max_states:
        _binary(p, op, out, vals[0], vals[1])
        return Val(out, "f32", nonpos=True, diff=(vals[0], args[1]))
    if op == "exp" and len(args) == 1 and ctx.get(args[0]).nonpos:
        v = ctx.get(args[0])
        if ctx.exp_reuse is not None and v.diff is not None:
            r = ctx.exp_reuse(*v.diff)
            if r is not None:
                return Val(r, "f32")
        emit_exp_nonpos(p, out, vals[0])
        return Val(out, "f32")
    if op == "pow" and len(args) == 2 and ctx.get(args[1]).const is not None:
        n = float(ctx.get(args[1]).const)
        if n.is_integer() and 1 <= abs(n) <= 16:
            # x^n by repeated squaring, 1 / x^|n| for a negative n (a few ulp)
            k, base, acc = int(abs(n)), vals[0], None
            while k:
                if k & 1:
                    if acc is None:
                        acc = base
                    else:
                        t = p.reg("f32")
                        p.emit(f"mul.rn.f32 {t}, {acc}, {base}")
                        acc = t
                k >>= 1
                if k:
                    t = p.reg("f32")
                    p.emit(f"mul.rn.f32 {t}, {base}, {base}")
                    base = t
            if n < 0:
                p.emit(f"rcp.rn.f32 {out}, {acc}")
            else:
                p.emit(f"mov.f32 {out}, {acc}")
            return Val(out, "f32")
        if n == 0.5:
            p.emit(f"sqrt.rn.f32 {out}, {vals[0]}")
            return Val(out, "f32")
    if len(vals) == 1:
        _unary(p, op, out, vals[0])
    elif len(vals) == 2:
        _binary(p, op, out, vals[0], vals[1])
    else:
        raise NotImplementedError(f"elementwise op {op} with {len(vals)} operands")
    return Val(out, "f32")


# --------------------------------------------------------------------------
# handlers


NARROW = ("f16", "bf16", "f8e4m3", "f8e5m2")     # result types rounded per op (values stay f32)


def _check_f32(dt, what: str, ctx: ScalarCtx | None = None) -> None:
    n = dtype_name(dt)
    if n in NARROW and ctx is not None and ctx.half_results:
        return
    if n not in (None, "f32"):
        raise NotImplementedError(f"{what} of dtype {n}: this back end computes reductions in f32")


def round_half(ctx: ScalarCtx, dt, reg: str) -> str:
    """A result of IR dtype f16 / bf16 / f8e4m3: the f32 value rounded to that type
    (nearest even; e4m3 saturating at +-448 like torch's float8_e4m3fn cast) and widened
    back, as the reference rounds every narrow op's result (``compiler/dtypes.py:148-227``)."""
    n = dtype_name(dt)
    if n not in NARROW:
        return reg
    p = ctx.ptx
    out = p.reg("f32")
    if n == "f8e5m2":
        # nearest even with torch's overflow to +-inf: the saturating convert (no other form
        # takes f32 to e5m2), then inf from the midpoint above the largest finite (61440)
        q, hh, lo, hi, big = p.reg("b16"), p.reg("b32"), p.reg("b16"), p.reg("b16"), p.reg("pred")
        ax, inf = p.reg("f32"), p.reg("f32")
        p.emit(f"cvt.rn.satfinite.e5m2x2.f32 {q}, 0f00000000, {reg}\n"
               f"cvt.rn.f16x2.e5m2x2 {hh}, {q}\nmov.b32 {{{lo}, {hi}}}, {hh}\ncvt.f32.f16 {out}, {lo}\n"
               f"abs.f32 {ax}, {reg}\nsetp.ge.f32 {big}, {ax}, 0f47700000\n"
               f"copysign.f32 {inf}, {reg}, 0f7F800000\n@{big} mov.f32 {out}, {inf}")
        return out
    if n == "f8e4m3":
        # e4m3 pair (value, 0) -> f16 pair -> the value's half -> f32; every e4m3 value is
        # exact in f16
        q, hh, lo, hi = p.reg("b16"), p.reg("b32"), p.reg("b16"), p.reg("b16")
        p.emit(f"cvt.rn.satfinite.e4m3x2.f32 {q}, 0f00000000, {reg}\n"
               f"cvt.rn.f16x2.e4m3x2 {hh}, {q}\nmov.b32 {{{lo}, {hi}}}, {hh}\ncvt.f32.f16 {out}, {lo}")
        return out
    h = p.reg("b16")
    p.emit(f"cvt.rn.{n}.f32 {h}, {reg}\ncvt.f32.{n} {out}, {h}")
    return out


# torch ops whose 16-bit products are summed exactly in f32 (cuBLAS, flash attention):
# the reference tells them from an elementwise product-sum by the kernel's name
# (``compiler/__init__.py:16-32``); the op list has to be the same to round alike
_MATMUL_OPS = re.compile(r"(?:^|_)(?:matmul|mm|bmm|addmm|baddbmm|addbmm|mv|addmv|dot|inner|"
                         r"tensordot|linear|bilinear|sdpa|einsum)(?:_|$)")


def matmul_kernel(name: str) -> bool:
    """Does the kernel compute a torch matmul (its 16-bit products are not rounded)?"""
    return bool(_MATMUL_OPS.search(name.removeprefix("k_")))


def load_index_vars(body) -> dict:
    """Loaded name -> the index variables of its Load, over a whole kernel body."""
    out = {}

    def walk(stmts):
        for s in stmts:
            if type(s).__name__ == "Load":
                vs = set()
                for e in s.index:
                    vs |= expr_vars(e)
                for n in s.names:
                    out[n] = vs
            for attr in ("body", "else_body"):
                sub = getattr(s, attr, None)
                if isinstance(sub, tuple):
                    walk(sub)
    walk(body)
    return out


def _contraction(ctx: ScalarCtx, args) -> bool:
    """``a * b`` as a matmul step by its indexing: each operand is indexed by a variable
    the other lacks (an outer product summed over the shared one), as the reference
    decides it (``compiler/stmts.py:421-430``)."""
    if len(args) != 2:
        return False
    a, b = (ctx.index_vars.get(n) for n in args)
    return bool(a and b and a - b and b - a)


# f64 exp: e^x = 2^k e^r with k = rint(x / ln 2), r = x - k ln 2 (ln 2 in two parts, so r is
# exact to f64), |r| <= ln2 / 2 and e^r by its Taylor series to r^13 (the next term is below
# 2^-60 relative): 1/n! for n = 2 .. 13
_EXP64_TAYLOR = (0.5, 0.16666666666666666, 0.041666666666666664, 0.008333333333333333, 0.001388888888888889, 0.0001984126984126984, 2.48015873015873e-05, 2.7557319223985893e-06, 2.755731922398589e-07, 2.505210838544172e-08, 2.08767569878681e-09, 1.6059043836821613e-10)
# ln 2 (from its series sum 1 / (k 2^k)) split at the low 32 mantissa bits: k * _LN2_HI is
# exact for the |k| < 1100 used here, _LN2_LO the rest to f64
_LN2_HI = 0.6931467056274414
_LN2_LO = 4.7493250390316726e-07


def emit_exp_f64(p: Ptx, dst: str, x: str) -> None:
    """e^x in f64, written here from the definition (not a library's exp).  2^k is built in
    the exponent field; where k is outside the normal exponents (results near the overflow
    threshold, or subnormal results) q is pre-scaled by 2 or 2^-54 and k moved back into
    range.  Above log(DBL_MAX) the result is inf, below -745.2 it is 0, NaN stays NaN."""
    xc, kf, r, q, sc = (p.reg("f64") for _ in range(5))
    k64, bits = p.reg("s64"), p.reg("b64")
    plo, phi, pnan, pbig, psmall = (p.reg("pred") for _ in range(5))
    p.emit(f"""
        setp.lt.f64 {plo}, {x}, {f64_hex(-745.2)}
        setp.gt.f64 {phi}, {x}, {f64_hex(709.782712893384)}
        setp.nan.f64 {pnan}, {x}, {x}
        max.f64 {xc}, {x}, {f64_hex(-745.2)}
        min.f64 {xc}, {xc}, {f64_hex(709.782712893384)}
        mul.rn.f64 {kf}, {xc}, {f64_hex(1.4426950408889634)}
        cvt.rni.f64.f64 {kf}, {kf}
        neg.f64 {r}, {kf}
        fma.rn.f64 {r}, {r}, {f64_hex(_LN2_HI)}, {xc}
        neg.f64 {q}, {kf}
        fma.rn.f64 {r}, {q}, {f64_hex(_LN2_LO)}, {r}
        mov.f64 {q}, {f64_hex(_EXP64_TAYLOR[-1])}
    """)
    for c in reversed(_EXP64_TAYLOR[:-1]):
        p.emit(f"fma.rn.f64 {q}, {q}, {r}, {f64_hex(c)}")
    p.emit(f"""
        fma.rn.f64 {q}, {q}, {r}, 0d3FF0000000000000
        fma.rn.f64 {q}, {q}, {r}, 0d3FF0000000000000
        cvt.rni.s64.f64 {k64}, {kf}
        setp.gt.s64 {pbig}, {k64}, 1023
        @{pbig} add.rn.f64 {q}, {q}, {q}
        @{pbig} sub.s64 {k64}, {k64}, 1
        setp.lt.s64 {psmall}, {k64}, -1022
        @{psmall} mul.rn.f64 {q}, {q}, 0d3C90000000000000
        @{psmall} add.s64 {k64}, {k64}, 54
        add.s64 {k64}, {k64}, 1023
        shl.b64 {bits}, {k64}, 52
        mov.b64 {sc}, {bits}
        mul.rn.f64 {dst}, {q}, {sc}
        @{plo} mov.f64 {dst}, 0d0000000000000000
        @{phi} mov.f64 {dst}, 0d7FF0000000000000
        @{pnan} mov.f64 {dst}, {x}
    """)


_KIND = {"i32": "s32", "i64": "s64", "f64": "f64", "f32": "f32"}


def _lower_typed(ctx: ScalarCtx, s) -> bool:
    """Assigns whose result is i32, i64 or f64: the IR's result dtype says the type, the
    operands promote to it (``ScalarCtx.as_kind``).  Integer ops follow torch: wrap-around
    arithmetic, floor division and a remainder with the divisor's sign, arithmetic right
    shift."""
    kind = _KIND.get(dtype_name(s.dtype))
    if kind not in ("s32", "s64", "f64"):
        return False
    op, p = s.op.name, ctx.ptx
    w = kind[1:]
    b = "b" + w
    r = p.reg(kind)
    if op == "where":
        c = ctx.pred(s.args[0])
        x, y = ctx.as_kind(s.args[1], kind), ctx.as_kind(s.args[2], kind)
        p.emit(f"selp.{b} {r}, {x}, {y}, {c}")
    elif op == "copy":
        r = ctx.as_kind(s.args[0], kind)
    elif kind == "f64":
        args = [ctx.as_kind(x, "f64") for x in s.args]
        binop = {"add": "add.rn.f64", "subtract": "sub.rn.f64", "multiply": "mul.rn.f64",
                 "divide": "div.rn.f64", "maximum": "max.f64", "minimum": "min.f64"}
        unop = {"negative": "neg.f64", "abs": "abs.f64", "sqrt": "sqrt.rn.f64", "reciprocal": "rcp.rn.f64"}
        if op in binop and len(args) == 2:
            p.emit(f"{binop[op]} {r}, {args[0]}, {args[1]}")
        elif op in unop and len(args) == 1:
            p.emit(f"{unop[op]} {r}, {args[0]}")
        elif op == "exp" and len(args) == 1:
            emit_exp_f64(p, r, args[0])
        else:
            raise NotImplementedError(f"elementwise op {op} (f64)")
    else:
        args = [ctx.as_kind(x, kind) for x in s.args]
        t = kind                       # s32 / s64
        if op in ("add", "subtract") and len(args) == 2:
            p.emit(f"{'add' if op == 'add' else 'sub'}.{t} {r}, {args[0]}, {args[1]}")
        elif op == "multiply" and len(args) == 2:
            p.emit(f"mul.lo.{t} {r}, {args[0]}, {args[1]}")
        elif op in ("maximum", "minimum") and len(args) == 2:
            p.emit(f"{'max' if op == 'maximum' else 'min'}.{t} {r}, {args[0]}, {args[1]}")
        elif op in ("bitwise_and", "bitwise_or", "bitwise_xor") and len(args) == 2:
            p.emit(f"{op.split('_')[1]}.{b} {r}, {args[0]}, {args[1]}")
        elif op == "bitwise_not" and len(args) == 1:
            p.emit(f"not.{b} {r}, {args[0]}")
        elif op == "negative" and len(args) == 1:
            p.emit(f"neg.{t} {r}, {args[0]}")
        elif op == "abs" and len(args) == 1:
            p.emit(f"abs.{t} {r}, {args[0]}")
        elif op in ("right_shift", "bitwise_right_shift", "left_shift", "bitwise_left_shift") and len(args) == 2:
            n = ctx.as_kind(s.args[1], "s32") if kind == "s64" else args[1]
            ins = f"shr.{t}" if "right" in op else f"shl.{b}"
            p.emit(f"{ins} {r}, {args[0]}, {n}")
        elif op in ("floor_divide", "remainder") and len(args) == 2:
            # C's truncating quotient / remainder, then moved toward -inf when the signs differ
            q, m, x, pn, pz = p.reg(kind), p.reg(kind), p.reg(kind), p.reg("pred"), p.reg("pred")
            p.emit(f"""
                div.{t} {q}, {args[0]}, {args[1]}
                rem.{t} {m}, {args[0]}, {args[1]}
                xor.{b} {x}, {m}, {args[1]}
                setp.lt.{t} {pn}, {x}, 0
                setp.ne.{t} {pz}, {m}, 0
                and.pred {pn}, {pn}, {pz}
            """)
            if op == "floor_divide":
                p.emit(f"mov.{b} {r}, {q}\n@{pn} sub.{t} {r}, {q}, 1")
            else:
                p.emit(f"mov.{b} {r}, {m}\n@{pn} add.{t} {r}, {m}, {args[1]}")
        else:
            raise NotImplementedError(f"elementwise op {op} ({dtype_name(s.dtype)})")
    target = ctx.env[s.name].text if (s.name in ctx.mutable and s.name in ctx.env) else None
    if target is not None:
        p.emit(f"mov.{b} {target}, {r}")
    else:
        ctx.env[s.name] = Val(r, kind)
    return True


# comparisons as ordered PTX compares (false with a NaN operand, as torch's), except
# not_equal (true with a NaN)
_CMP_OPS = {"greater": "gt", "greater_equal": "ge", "less": "lt", "less_equal": "le",
            "equal": "eq", "not_equal": "neu"}
_BOOL_OPS = {"bitwise_and": "and", "bitwise_or": "or", "bitwise_xor": "xor",
             "logical_and": "and", "logical_or": "or", "logical_xor": "xor"}


def _lower_bool(ctx: ScalarCtx, s) -> bool:
    """Comparisons, logic on bools and ``where``: the bool values live in predicates."""
    op, p = s.op.name, ctx.ptx
    if op in _CMP_OPS:
        # compared in the operands' common type (torch's promotion)
        kinds = {ctx.get(x).kind for x in s.args}
        kind = next((k for k in ("f64", "f32", "s64", "s32") if k in kinds), "f32")
        a, b = (ctx.as_kind(x, kind) for x in s.args)
        cmp = _CMP_OPS[op]
        if kind in ("s32", "s64") and cmp == "neu":
            cmp = "ne"
        r = p.reg("pred")
        p.emit(f"setp.{cmp}.{kind} {r}, {a}, {b}")
        ctx.env[s.name] = Val(r, "pred")
        return True
    if op in _BOOL_OPS and all(ctx.get(x).kind == "pred" for x in s.args):
        a, b = (ctx.pred(x) for x in s.args)
        r = p.reg("pred")
        p.emit(f"{_BOOL_OPS[op]}.pred {r}, {a}, {b}")
        ctx.env[s.name] = Val(r, "pred")
        return True
    if op in ("bitwise_not", "logical_not") and ctx.get(s.args[0]).kind == "pred":
        r = p.reg("pred")
        p.emit(f"not.pred {r}, {ctx.pred(s.args[0])}")
        ctx.env[s.name] = Val(r, "pred")
        return True
    if op == "where":
        c = ctx.pred(s.args[0])
        a, b = ctx.f32(s.args[1]), ctx.f32(s.args[2])
        r = p.reg("f32")
        p.emit(f"selp.f32 {r}, {a}, {b}, {c}")
        val = Val(r, "f32")
        if dtype_name(s.dtype) in NARROW:
            val = Val(round_half(ctx, s.dtype, r), "f32")
        target = ctx.env[s.name].text if (s.name in ctx.mutable and s.name in ctx.env) else None
        if target is not None:
            p.emit(f"mov.f32 {target}, {val.text}")
        else:
            ctx.env[s.name] = val
        return True
    if op == "copy" and dtype_name(s.dtype) == "bool" and ctx.get(s.args[0]).kind == "pred":
        ctx.env[s.name] = ctx.get(s.args[0])
        return True
    return False


@handles("Assign")
def lower_assign(ctx: ScalarCtx, s) -> None:
    if _lower_bool(ctx, s) or _lower_typed(ctx, s):
        return
    _check_f32(s.dtype, "Assign", ctx)
    target = ctx.env[s.name].text if (s.name in ctx.mutable and s.name in ctx.env) else None
    val = compute_f32(ctx, s.op.name, list(s.args), dst=None)
    if s.op.name == "copy" and len(s.args) == 1 and s.args[0] in ctx.index_vars:
        ctx.index_vars[s.name] = ctx.index_vars[s.args[0]]     # `f16 v0 = copy(in0)`
    exact = s.op.name == "multiply" and (ctx.exact_products or _contraction(ctx, s.args))
    if dtype_name(s.dtype) in NARROW and not exact:
        # (a product of two 16-bit values is exact in f32: kept as is in a matmul)
        val = Val(round_half(ctx, s.dtype, val.text), "f32")
    if target is not None:
        ctx.ptx.emit(f"mov.f32 {target}, {val.text}")
    else:
        ctx.env[s.name] = val


@handles("Let")
def lower_let(ctx: ScalarCtx, s) -> None:
    v = s.value
    if type(v).__name__ == "Literal":
        if dtype_name(s.dtype) in (None, "f32") and isinstance(v.value, (int, float)):
            ctx.env[s.name] = Val(f32_hex(float(v.value)), "f32", float(v.value))
            return
    raise NotImplementedError(f"Let of {type(v).__name__}")


@handles("Init")
def lower_init(ctx: ScalarCtx, s) -> None:
    _check_f32(s.dtype, "Init")
    r = ctx.ptx.reg("f32")
    ctx.ptx.emit(f"mov.f32 {r}, {f32_hex(float(s.identity))}")
    ctx.env[s.name] = Val(r, "f32")
    ctx.mutable.add(s.name)


@handles("Accum")
def lower_accum(ctx: ScalarCtx, s) -> None:
    """``acc = op(base or acc, value)`` into the accumulator's own register
    (the reference: ``compiler/stmts.py:441-467``).  The template seeds the
    accumulator register with the op's identity before the loop."""
    acc = ctx.get(s.name)
    left = s.base or s.name
    if acc.kind in ("s32", "s64", "f64"):
        # an accumulator of the IR's integer / f64 type (its register kind set when seeded)
        a, b = ctx.as_kind(left, acc.kind), ctx.as_kind(s.value, acc.kind)
        t, op = acc.kind, s.op.name
        ins = {"add": f"add.{t}" if t != "f64" else "add.rn.f64", "maximum": f"max.{t}",
               "minimum": f"min.{t}", "multiply": f"mul.lo.{t}" if t != "f64" else "mul.rn.f64"}.get(op)
        if ins is None:
            raise NotImplementedError(f"accumulation {op} ({t})")
        ctx.ptx.emit(f"{ins} {acc.text}, {a}, {b}")
        return
    _check_f32(s.dtype, "Accum", ctx)
    a, b = ctx.f32(left), ctx.f32(s.value)
    _binary(ctx.ptx, s.op.name, acc.text, a, b)
    if dtype_name(s.dtype) in NARROW:
        ctx.ptx.emit(f"mov.f32 {acc.text}, {round_half(ctx, s.dtype, acc.text)}")


@handles("Load")
def lower_load(ctx: ScalarCtx, s) -> None:
    if all(n in ctx.env for n in s.names):
        return   # bound by the template (vector lane or cached value)
    if len(s.names) == 1 and s.input in ctx.constants:
        cdt = ctx.const_dtypes.get(s.input)
        v = float(ctx.constants[s.input])
        if cdt in ("i32", "i64"):
            ctx.env[s.names[0]] = Val(str(int(v)), "s32" if cdt == "i32" else "s64", v)
            return
        if cdt == "f64":
            ctx.env[s.names[0]] = Val(f64_hex(v), "f64", v)
            return
        _check_f32(s.dtype, "constant Load", ctx)
        ctx.env[s.names[0]] = Val(f32_hex(v), "f32", v)
        return
    if ctx.on_load is None:
        raise NotImplementedError(f"Load of {s.input} outside a template stream")
    ctx.on_load(ctx, s)


@handles("Write")
def lower_write(ctx: ScalarCtx, s) -> None:
    if ctx.on_write is None:
        raise NotImplementedError(f"Write to {s.output} outside a template stream")
    ctx.on_write(ctx, s)


# Structural statements are consumed by the kernel templates; reaching one
# here means the IR nests it somewhere no template expects.
def _structural(ctx, s):
    raise NotImplementedError(f"statement {type(s).__name__} in an unsupported position")


for _k in ("Tile", "Loop", "StridedLoop", "Cond", "WarpShuffle", "TreeHalve", "Smem", "Sync",
           "CpAsyncCopy", "CpAsyncCommit", "CpAsyncWait", "RegFragment", "LdmatrixLoad",
           "MmaSyncPtx", "RegStore", "FragmentApply", "FragmentRowReduce", "FragmentRepack"):
    HANDLERS.setdefault(_k, _structural)


# --------------------------------------------------------------------------
# integer index expressions (Var / Literal / BinaryExpr / TernaryExpr)


def eval_index(expr, env: dict) -> int:
    """Evaluate an index expression with Python ints (C semantics for / and %)."""
    k = type(expr).__name__
    if k == "Var":
        return env[expr.name]
    if k == "Literal":
        return int(expr.value)
    if k == "BinaryExpr":
        a, b = eval_index(expr.left, env), eval_index(expr.right, env)
        op = expr.op
        if op == "+":
            return a + b
        if op == "-":
            return a - b
        if op == "*":
            return a * b
        if op == "/":
            q = abs(a) // abs(b)
            return q if (a >= 0) == (b >= 0) else -q
        if op == "//":
            return a // b
        if op == "%":
            return a - b * eval_index_div(a, b)
        if op == "<":
            return int(a < b)
        if op == "<=":
            return int(a <= b)
        if op == ">":
            return int(a > b)
        if op == ">=":
            return int(a >= b)
        if op == "==":
            return int(a == b)
        if op == "!=":
            return int(a != b)
        if op == "&&":
            return int(bool(a) and bool(b))
        if op == "||":
            return int(bool(a) or bool(b))
        raise NotImplementedError(f"index operator {op}")
    if k == "TernaryExpr":
        return eval_index(expr.if_true if eval_index(expr.cond, env) else expr.if_false, env)
    raise NotImplementedError(f"index expression {k}")


def eval_index_div(a: int, b: int) -> int:
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b >= 0) else -q


def expr_vars(expr) -> set:
    k = type(expr).__name__
    if k == "Var":
        return {expr.name}
    if k == "BinaryExpr":
        return expr_vars(expr.left) | expr_vars(expr.right)
    if k == "TernaryExpr":
        return expr_vars(expr.cond) | expr_vars(expr.if_true) | expr_vars(expr.if_false)
    return set()


def flat_offset(index: tuple, shape: tuple, env: dict) -> int:
    """Row-major element offset of ``buffer[index]`` (scalar buffers: ``()``)."""
    off = 0
    for e, d in zip(index, shape):
        off = off * int(d) + eval_index(e, env)
    return off
