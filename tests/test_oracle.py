"""The CPU oracle reproduces the reference's golden vectors (expected.npz)."""

import json

import numpy as np
import pytest

from oracle.refs import PROBLEM_REFS, problem_expected, e4m3_round, bf16_round

from conftest import GOLDEN

PROBLEMS = sorted(p.name for p in GOLDEN.iterdir())

# bf16 matmul results: torch adds the f32 products in its own order before rounding to
# bf16, so a sum that lands next to a bf16 rounding boundary may round the other way
# (1 of 4096 outputs of x_q_bf16_mm); these agree to one bf16 ulp
ONE_BF16_ULP = {"x_q_bf16_mm", "x_q_bf16_mm_t", "x_q_bf16_mm_odd"}
# f64 exp: the golden vectors came from another libm; differences in the last bits
TWO_F64_ULP = {"x_d_f64_exp", "x_d_f64_softmax"}


@pytest.mark.parametrize("pid", PROBLEMS)
def test_oracle_matches_golden(pid):
    d = GOLDEN / pid
    meta = json.loads((d / "meta.json").read_text())
    assert meta["id"] in PROBLEM_REFS, f"no oracle ref for {pid}"
    exp = dict(np.load(d / "expected.npz"))
    got = problem_expected(meta)
    for name, ref in exp.items():
        g = np.asarray(got[name]).reshape(ref.shape)
        if pid in TWO_F64_ULP:
            assert np.allclose(g, ref, rtol=2.0 ** -48, atol=0), f"{pid}:{name}"
            continue
        if pid in ONE_BF16_ULP:
            # one ulp of a bf16 value: 2^-7 of it at most (just below a power of two); sums
            # that cancel to near zero keep the f32 adding order's own error (~1e-6)
            assert np.all(np.abs(g - ref) <= np.abs(ref) * 2.0 ** -7 + 2.0 ** -16), f"{pid}:{name}"
            continue
        # same formula at the same precision: bit-identical
        assert np.array_equal(g.astype(ref.dtype), ref), f"{pid}:{name}"


def test_bf16_round_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38], dtype=np.float32)
    r = bf16_round(x)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: even mantissa (1.0) wins
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.015625)
    assert r[3] == -2.5


def test_e4m3_round_saturates_and_rounds_even():
    x = np.array([0.0, 448.0, 500.0, -1000.0, 1.0625, 1.1875, 2 ** -9, 2 ** -10], dtype=np.float32)
    r = e4m3_round(x)
    assert list(r[:4]) == [0.0, 448.0, 448.0, -448.0]
    # 1.0625 is halfway between 1.0 and 1.125: ties to even -> 1.0; 1.1875 -> 1.25
    assert r[4] == 1.0 and r[5] == 1.25
    # smallest subnormal 2^-9 is kept, 2^-10 (a tie with 0) rounds to even 0
    assert r[6] == 2 ** -9 and r[7] == 0.0
