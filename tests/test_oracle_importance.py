"""CPU checks of the decode importance's fixed-point policy in the oracle.

Each route adds w * norm[e] (one fp32 product) in 2^-32 fixed point to its expert's int64 sum.
A NaN product counts 0, products are clamped to |p| <= 2^24 (at most 2^56 per route), and the
int64 sum wraps modulo 2^64 like the kernels' atomics, so an expert's importance is exact while
its true total stays below 2^31 in magnitude.
"""

from __future__ import annotations

import numpy as np

from oracle import oracle as O

Q = 2.0 ** 32


def fp(p: float) -> int:
    return int(O.lib().orc_fixed_point(float(p)))


def test_fixed_point_values():
    assert fp(0.0) == 0 and fp(-0.0) == 0
    assert fp(1.0) == 1 << 32
    assert fp(0.5) == 1 << 31
    assert fp(2.0 ** -33) == 0  # ties to even
    assert fp(3 * 2.0 ** -33) == 2  # 1.5 units -> 2
    assert fp(float("nan")) == 0
    assert fp(float("inf")) == 1 << 56 and fp(float("-inf")) == -(1 << 56)
    assert fp(1e30) == 1 << 56 and fp(-1e30) == -(1 << 56)
    assert fp(2.0 ** 24) == 1 << 56


def test_importance_nan_and_huge_routes():
    norms = np.ones(8, np.float32)
    w = np.array([[0.5, np.nan, 1e30, 0.25]], np.float32)
    ids = np.array([[0, 1, 2, 0]], np.int32)
    imp = O.importance(w, ids, norms)
    assert imp[0] == int(0.75 * Q)
    assert imp[1] == 0  # the NaN route counts nothing
    assert imp[2] == 1 << 56
    assert np.all(imp[3:] == 0)


def test_importance_sum_is_exact_within_the_bound():
    # 127 maximal routes of one expert: 127 * 2^56 < 2^63, exact
    w = np.full((127, 1), 2.0 ** 24, np.float32)
    imp = O.importance(w, np.zeros((127, 1), np.int32), np.ones(2, np.float32))
    assert imp[0] == 127 * (1 << 56)
    # mixed signs whose partial sums leave the int64 range still give the exact total (mod 2^64)
    w = np.array([[2.0 ** 24]] * 200 + [[-(2.0 ** 24)]] * 199, np.float32)
    imp = O.importance(w, np.zeros((399, 1), np.int32), np.ones(2, np.float32))
    assert imp[0] == 1 << 56
