"""The selection keys of the tile routers, restated in numpy (no GPU).

The tile routers (csrc/router_tpt.cu, csrc/router_biased.cu) key each group-of-4 maximum as its
raw float bits compared as a signed 32-bit integer, with the low bits replaced by the group's slot,
sort those keys, and take the fast path only under conditions that make the 8 named groups hold
the exact top 8.  This file checks the facts that argument rests on, over random and adversarial
rows:

* positive floats (and +inf, and the canonical NaN 0x7FFFFFFF) order by value as signed integers
  and above every negative float; negative floats order in reverse among themselves;
* clearing the low bits of a positive key rounds its value down, so a truncated positive key is a
  lower bound; for a negative key, setting the low bits rounds its value down;
* rounding a truncated key up (low bits set for a positive key, cleared for a negative one) gives
  an upper bound (router_biased's 9th and 10th maxima);
* with the 8th largest key positive and the 9th below it after truncation, the 8 named groups hold
  the exact top 8 of the row by (value desc, column asc), which is what the fast path inserts from;
* whatever the row, the exact path's bound (the 8th key rounded down in value) is at most the 8th
  largest element, so the exact insertion sees every element of the top 8.
"""

from __future__ import annotations

import numpy as np

SLOT_MASK = 31  # router_tpt: 32 groups, the slot in the low 5 bits


def f32_bits(x):
    return np.asarray(x, dtype=np.float32).view(np.int32)


def bits_f32(b):
    return np.asarray(b, dtype=np.int64).astype(np.uint32).view(np.float32)


def group_keys(row):
    """Keys of the 32 group maxima of a 128-wide row: raw bits with the low 5 bits = 31 - slot."""
    g = row.reshape(32, 4)
    m = np.where(np.isnan(g).any(axis=1), np.float32(np.nan), g.max(axis=1)).astype(np.float32)
    bits = f32_bits(m).astype(np.int64)
    bits = np.where(np.isnan(m), 0x7FFFFFFF, bits)  # max.NaN returns the canonical NaN
    slot = np.arange(32)
    keys = (bits & ~np.int64(SLOT_MASK)) | (SLOT_MASK - slot)
    return np.where(keys >= 2 ** 31, keys - 2 ** 32, keys).astype(np.int64)


def exact_top8(row):
    """Columns of the top 8 by (value desc, column asc), -0 equal to +0 (finite rows)."""
    v = np.where(row == 0, np.float32(0), row).astype(np.float64)
    return sorted(range(row.size), key=lambda c: (-v[c], c))[:8]


def rows(n, seed):
    rng = np.random.default_rng(seed)
    out = [rng.standard_normal(128).astype(np.float32) for _ in range(n)]
    # adversarial rows: coarse values (ties), negatives only, zeros, infinities, tiny values
    for i in range(n // 4):
        r = np.round(rng.standard_normal(128) * 2).astype(np.float32) / 2
        out.append(r)
        out.append(-np.abs(rng.standard_normal(128)).astype(np.float32))
        z = rng.standard_normal(128).astype(np.float32)
        z[rng.integers(0, 128, 20)] = 0.0
        z[rng.integers(0, 128, 5)] = -0.0
        out.append(z)
        s = rng.standard_normal(128).astype(np.float32)
        s[rng.integers(0, 128, 3)] = np.inf
        s[rng.integers(0, 128, 3)] = -np.inf
        out.append(s)
        out.append((rng.standard_normal(128) * 1e-40).astype(np.float32))
    return out


def test_signed_bits_order():
    rng = np.random.default_rng(1)
    scale = 10.0 ** rng.integers(-30, 30, 4000)
    x = np.concatenate([(rng.standard_normal(4000) * scale).astype(np.float32),
                        np.array([np.inf, -np.inf, 0.0, -0.0, 1e-45, -1e-45], np.float32)])
    b = f32_bits(x).astype(np.int64)
    pos = x > 0
    # positives by value
    order = np.argsort(b[pos], kind="stable")
    assert np.all(np.diff(x[pos][order]) >= 0)
    # every positive above every negative
    assert b[pos].min() > b[x < 0].max()
    # negatives in reverse
    neg = x < 0
    order = np.argsort(b[neg], kind="stable")
    assert np.all(np.diff(x[neg][order]) <= 0)
    # the canonical NaN sits above +inf
    assert 0x7FFFFFFF > int(f32_bits(np.float32(np.inf)))


def test_truncation_bounds():
    rng = np.random.default_rng(2)
    x = (rng.standard_normal(20000) * 10.0 ** rng.integers(-20, 20, 20000)).astype(np.float32)
    x = x[np.isfinite(x) & (x != 0)]
    b = f32_bits(x).astype(np.int64)
    for low in (31, 63):
        down = np.where(b >= 0, b & ~low, b | low)  # rounded down in value
        up = np.where(b >= 0, b | low, b & ~low)    # rounded up in value
        assert np.all(bits_f32(down) <= x)
        assert np.all(bits_f32(up) >= x)


def test_fast_path_condition_names_the_exact_top8():
    fast_rows = 0
    for row in rows(400, 3):
        keys = group_keys(row)
        order = np.argsort(-keys, kind="stable")
        pk = keys[order]
        p9, k8 = pk[8], pk[7]
        nan_row = pk[0] > 0x7F80001F
        fast = (p9 >> 5) < (k8 >> 5) and k8 >= 32 and not nan_row
        # exact path bound: the 8th key rounded down in value is at most the 8th largest element
        if not nan_row:
            b8 = int(k8)
            lb = bits_f32((b8 & ~31) if b8 >= 0 else (b8 | 31))
            v = np.where(row == 0, np.float32(0), row)
            eighth = np.sort(v)[::-1][7]
            assert lb <= eighth or np.isnan(lb)
        if not fast:
            continue
        fast_rows += 1
        named = {SLOT_MASK - int(k & SLOT_MASK) for k in pk[:8]}
        top = exact_top8(row)
        assert all(c // 4 in named for c in top), (row, named, top)
        # the named maxima are positive, so float compares and bits | sign give their order keys
        assert all(row.reshape(32, 4)[g].max() > 0 for g in named)
    assert fast_rows > 300
