"""The parity criterion of the BASELINE-size tests (test infrastructure).

BASELINE.json's bars are relative: fp32-accumulated bf16 within 1e-2, fp8 within 5e-2,
reductions within 1e-5.  A relative bar on the whole output is measured as
``||got - ref||_2 / ||ref||_2``; on its own it lets a few badly wrong elements through,
so the element-wise error is also bounded, by a few bf16 units in the last place of
the output's largest magnitude (the output is rounded to bf16 once, so a correct
kernel is within one of them) -- with no absolute floor.
"""

from __future__ import annotations

import math

import numpy as np


def bf16_ulp(x: float) -> float:
    """The spacing of bf16 values at |x| (8 significant bits)."""
    x = abs(float(x))
    if x == 0.0 or not math.isfinite(x):
        return 0.0
    return 2.0 ** (math.floor(math.log2(x)) - 7)


def parity(got, ref, rel: float, ulps: float = 4.0) -> dict:
    """Error statistics of ``got`` against ``ref`` and whether they meet the bars."""
    g = np.asarray(got, np.float64)
    r = np.asarray(ref, np.float64)
    if g.shape != r.shape:
        raise ValueError(f"shapes differ: {g.shape} vs {r.shape}")
    diff = g - r
    rn = float(np.linalg.norm(r.reshape(-1)))
    rel_norm = float(np.linalg.norm(diff.reshape(-1))) / rn if rn else float(np.abs(diff).max())
    max_abs = float(np.abs(diff).max()) if diff.size else 0.0
    bound = ulps * bf16_ulp(np.abs(r).max()) if r.size else 0.0
    ok = bool(np.isfinite(g).all() and rel_norm <= rel and max_abs <= bound)
    return {"ok": ok, "rel_norm": rel_norm, "max_abs": max_abs, "max_abs_bound": bound,
            "rel_bar": rel}


def assert_parity(got, ref, rel: float, ulps: float = 4.0, what: str = "") -> dict:
    s = parity(got, ref, rel, ulps)
    assert s["ok"], (f"{what}: rel_norm {s['rel_norm']:.3e} (bar {rel}), max |err| "
                     f"{s['max_abs']:.3e} (bar {s['max_abs_bound']:.3e})")
    return s


def sample_rows(n: int, count: int, seed: int = 0) -> np.ndarray:
    """First, last and random rows of an n-row output."""
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, count)]))
