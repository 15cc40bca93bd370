"""CPU oracle for the calibration accumulator (TEST INFRASTRUCTURE ONLY).

A float64 numpy restatement of PairwiseScalarStats (exfold/qwen3/calibration.py:9-140), used by
the tests to check the GPU calibration kernels; nothing in the product imports it.

update (calibration.py:49-95): for every token and every ordered pair of its routes (s, d) whose
expert ids differ, with u the unweighted expert outputs and w_s = ||u_s||:
    dot[e_s, e_d]       += w_s * <u_s, u_d>
    target_sq[e_s, e_d] += w_s * ||u_d||^2
    source_sq[e_s, e_d] += w_s * ||u_s||^2
and for every route: norm_sum[e] += ||u||, norm_count[e] += 1.  The reference forms the products
in fp32 and adds them in fp64; here everything is float64.  Routes with an expert id outside
[0, E) are skipped (the reference would index out of range).
finalize (calibration.py:97-126) and expert_norms (calibration.py:128-140) follow the reference
formulas in float64, then round to float32.
"""

from __future__ import annotations

import numpy as np

DEFAULT_LOSS = 1e30


def update(acc: dict, expert_ids, expert_outputs, num_experts: int) -> None:
    ids = np.asarray(expert_ids, np.int64)
    u = np.asarray(expert_outputs, np.float64)
    E = num_experts
    sq = np.einsum("tkh,tkh->tk", u, u)
    dots = np.einsum("tsh,tdh->tsd", u, u)
    w = np.sqrt(sq)
    T, k = ids.shape
    valid = (ids >= 0) & (ids < E)
    for s in range(k):
        for d in range(k):
            m = valid[:, s] & valid[:, d] & (ids[:, s] != ids[:, d])
            idx = ids[m, s] * E + ids[m, d]
            np.add.at(acc["dot"].reshape(-1), idx, (dots[:, s, d] * w[:, s])[m])
            np.add.at(acc["target_sq"].reshape(-1), idx, (sq[:, d] * w[:, s])[m])
            np.add.at(acc["source_sq"].reshape(-1), idx, (sq[:, s] * w[:, s])[m])
    np.add.at(acc["norm_sum"], ids[valid], w[valid])
    np.add.at(acc["norm_count"], ids[valid], 1.0)


def new_accumulators(num_experts: int) -> dict:
    E = num_experts
    return {"dot": np.zeros((E, E)), "target_sq": np.zeros((E, E)), "source_sq": np.zeros((E, E)),
            "norm_sum": np.zeros(E), "norm_count": np.zeros(E)}


def finalize(acc: dict, ridge: float = 1e-3, clip_min: float = -4.0, clip_max: float = 4.0):
    dot, tsq, ssq = acc["dot"], acc["target_sq"], acc["source_sq"]
    if not all(np.isfinite(v).all() for v in (dot, tsq, ssq)):
        raise RuntimeError("non-finite calibration statistics")
    observed = ssq > 0
    denom = tsq + ridge
    coeff = np.zeros_like(dot)
    usable = observed & (denom > 0)
    coeff[usable] = dot[usable] / denom[usable]
    coeff = np.clip(coeff, clip_min, clip_max)
    residual = ssq - 2 * coeff * dot + coeff * coeff * tsq
    loss = np.full_like(ssq, DEFAULT_LOSS)
    loss[observed] = np.maximum(residual[observed], 0) / ssq[observed]
    loss = np.minimum(loss, DEFAULT_LOSS)
    np.fill_diagonal(loss, DEFAULT_LOSS)
    coeff[~observed] = 0.0
    coeff[loss >= DEFAULT_LOSS] = 0.0
    np.fill_diagonal(coeff, 1.0)
    return coeff.astype(np.float32), loss.astype(np.float32)


def expert_norms(acc: dict):
    count = acc["norm_count"]
    norms = acc["norm_sum"] / np.maximum(count, 1)
    observed = count > 0
    if observed.any():
        obs = np.sort(norms[observed])
        fallback = obs[(obs.size - 1) // 2]  # torch.median: the lower of the two middle values
    else:
        fallback = 1.0
    return np.where(observed, norms, fallback).astype(np.float32)
