"""Shared pieces of the sm_100a templates: parameter lists, affine index analysis."""

from __future__ import annotations

import random
import re
from dataclasses import dataclass

from ..stmts import flat_offset, eval_index

DTYPE_BYTES = {"f32": 4, "f16": 2, "bf16": 2, "f64": 8, "i32": 4, "i64": 8, "e4m3": 1, "u8": 1}


def param_symbol(name: str) -> str:
    """Buffer names are IR identifiers; prefix them so they never clash with PTX names
    (the reference does the same: compiler/prologue.py:21-23)."""
    return "param_" + re.sub(r"\W", "_", name)


def arg_params(spec) -> list[str]:
    """``.param`` declarations in meta.json arg_order: buffers as .u64 pointers,
    scalars by value (compiler/prologue.py:33-42 in the reference)."""
    out = []
    for p in spec.params:
        if p.scalar:
            t = {"f32": ".f32", "i32": ".s32", "i64": ".s64"}.get(p.dtype)
            if t is None:
                raise NotImplementedError(f"scalar parameter {p.name!r} of dtype {p.dtype}")
            out.append(f".param {t} {param_symbol(p.name)}")
        else:
            out.append(f".param .u64 {param_symbol(p.name)}")
    return out


def load_pointer(ptx, name: str) -> str:
    """ld.param + cvta.to.global of one buffer pointer."""
    raw, glob = ptx.reg("b64"), ptx.reg("b64")
    ptx.emit(f"ld.param.u64 {raw}, [{param_symbol(name)}]\ncvta.to.global.u64 {glob}, {raw}")
    return glob


@dataclass(frozen=True)
class Affine:
    """offset = sum(coef[v] * v) + const over the named integer variables."""
    coef: tuple            # ((var, coef), ...) sorted, zero coefficients dropped
    const: int

    def get(self, var: str) -> int:
        return dict(self.coef).get(var, 0)

    def eval(self, env: dict) -> int:
        return self.const + sum(c * env[v] for v, c in self.coef)


def affine_offset(index: tuple, shape: tuple, ranges: dict, fixed: dict | None = None,
                  trials: int = 24) -> Affine:
    """Fit the row-major flat offset of ``buf[index]`` as an affine function of the
    variables in ``ranges`` (name -> extent) and verify it on random points.

    Raises NotImplementedError when the index is not affine (div/mod of a
    variable that does not cancel, a ternary clamp that is active, ...)."""
    fixed = dict(fixed or {})
    names = sorted(ranges)
    zero = {n: 0 for n in names}
    zero.update(fixed)
    base = flat_offset(index, shape, zero)
    coef = []
    for n in names:
        if ranges[n] <= 1:
            continue
        env = dict(zero)
        env[n] = 1
        c = flat_offset(index, shape, env) - base
        if c:
            coef.append((n, c))
    aff = Affine(tuple(coef), base)
    rng = random.Random(1234)
    probes = [dict(zero)]
    probes.append({**zero, **{n: max(0, ranges[n] - 1) for n in names}})
    for _ in range(trials):
        probes.append({**zero, **{n: rng.randrange(max(1, ranges[n])) for n in names}})
    for env in probes:
        if flat_offset(index, shape, env) != aff.eval(env):
            raise NotImplementedError("buffer index is not affine in the loop/tile axes")
    return aff


def in_bounds(index: tuple, shape: tuple, env: dict) -> bool:
    for e, d in zip(index, shape):
        v = eval_index(e, env)
        if v < 0 or v >= int(d):
            return False
    return True
