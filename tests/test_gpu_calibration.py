"""GPU parity of the calibration accumulator (exf_calibration_* through
exfold_b200.calibration.PairwiseScalarStats) against the reference's own statistics
(tests/golden/calibration_reference.npz, written by the reference's PairwiseScalarStats) and
against the float64 oracle (oracle/calibration.py).

Tolerances: the per-token dot products are fp32 sums in a different order than the reference's
einsum, so statistics agree to about 1e-7 of each array's scale (atol 1e-6 x max |value|, rtol
1e-6); the fp32 coefficient / loss tables and norms to 1e-5.  Ids of routes are integers and
the counts are exact.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from exfold_b200.calibration import PairwiseScalarStats
from oracle import calibration as C

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "calibration_reference.npz"
DEV = torch.device("cuda:0")


def cuda(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dtype is None else t.to(dtype)


def host(t):
    torch.cuda.synchronize(DEV)
    return t.detach().cpu().numpy()


def close_stats(got, want):
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6 * max(np.abs(want).max(), 1e-30))


@pytest.mark.parametrize("case", ["a", "b"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_matches_reference_accumulator(case, dtype):
    g = np.load(GOLDEN)
    ids, out = g[f"{case}_ids"], g[f"{case}_outputs"]
    E = g[f"{case}_dot"].shape[0]
    stats = PairwiseScalarStats(E, ridge=1e-3, clip_min=-4.0, clip_max=4.0, device=DEV)
    half = ids.shape[0] // 2
    stats.update(cuda(ids[:half]).long(), cuda(out[:half], dtype))
    stats.update(cuda(ids[half:]), cuda(out[half:], dtype))
    close_stats(host(stats.dot), g[f"{case}_dot"])
    close_stats(host(stats.target_sq_norm), g[f"{case}_target_sq"])
    close_stats(host(stats.source_sq_norm), g[f"{case}_source_sq"])
    close_stats(host(stats.expert_norm_sum), g[f"{case}_norm_sum"])
    np.testing.assert_array_equal(host(stats.expert_norm_count), g[f"{case}_norm_count"])
    coeff, loss = stats.finalize()
    np.testing.assert_allclose(host(coeff), g[f"{case}_coeff"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(loss), g[f"{case}_loss"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(stats.expert_norms()), g[f"{case}_norms"], rtol=1e-5)


def test_matches_oracle_at_qwen3_shape():
    """Qwen3 layer shape: 8 routes of 2048-wide bf16 expert outputs over 128 experts; ids with
    duplicates, out-of-range ids (skipped) and int32 ids; fp16 outputs for half the tokens."""
    rng = np.random.default_rng(11)
    T, K, H, E = 4096, 8, 2048, 128
    ids = rng.integers(0, E, (T, K)).astype(np.int32)
    ids[5, 3] = E + 7
    ids[6, 0] = -1
    out = rng.standard_normal((T, K, H)).astype(np.float32)
    out = torch.from_numpy(out).bfloat16().float().numpy()
    stats = PairwiseScalarStats(E, device=DEV)
    stats.update(cuda(ids[:2048]), cuda(out[:2048], torch.bfloat16))
    stats.update(cuda(ids[2048:]), cuda(out[2048:], torch.float16))
    acc = C.new_accumulators(E)
    C.update(acc, ids[:2048], out[:2048], E)
    C.update(acc, ids[2048:], torch.from_numpy(out[2048:]).half().float().numpy(), E)
    close_stats(host(stats.dot), acc["dot"])
    close_stats(host(stats.target_sq_norm), acc["target_sq"])
    close_stats(host(stats.source_sq_norm), acc["source_sq"])
    close_stats(host(stats.expert_norm_sum), acc["norm_sum"])
    np.testing.assert_array_equal(host(stats.expert_norm_count), acc["norm_count"])
    coeff, loss = stats.finalize()
    ec, el = C.finalize(acc)
    np.testing.assert_allclose(host(coeff), ec, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(loss), el, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(stats.expert_norms()), C.expert_norms(acc), rtol=1e-5)


def test_reference_closed_form_clipping_and_errors():
    stats = PairwiseScalarStats(3, ridge=1e-3, device=DEV)
    ids = torch.tensor([[0, 1], [0, 1]], device=DEV)
    out = torch.tensor([[[2.0, 0.0, 0, 0, 0, 0, 0, 0], [1.0, 0.0, 0, 0, 0, 0, 0, 0]],
                        [[0.0, 3.0, 0, 0, 0, 0, 0, 0], [0.0, 1.0, 0, 0, 0, 0, 0, 0]]], device=DEV)
    stats.update(ids, out)
    coeff, loss = stats.finalize()
    w = out[:, 0].norm(dim=-1)
    expected = (w * (out[:, 0] * out[:, 1]).sum(-1)).sum() / ((w * out[:, 1].square().sum(-1)).sum()
                                                             + 1e-3)
    assert torch.allclose(coeff[0, 1], expected.float())
    assert loss[0, 1] < 1.0 and coeff[2, 0] == 0 and loss[2, 0] == stats.default_loss
    assert torch.equal(coeff.diagonal().cpu(), torch.ones(3))
    stats = PairwiseScalarStats(2, ridge=1e-6, clip_min=-4.0, clip_max=4.0, device=DEV)
    stats.update(torch.tensor([[0, 1]], device=DEV),
                 torch.tensor([[[10.0] + [0.0] * 7, [1.0] + [0.0] * 7]], device=DEV))
    assert stats.finalize()[0][0, 1] == 4.0
    assert torch.allclose(stats.expert_norms().cpu(), torch.tensor([10.0, 1.0]))
    bad = PairwiseScalarStats(2, device=DEV)
    bad.update(torch.tensor([[0, 1]], device=DEV),
               torch.tensor([[[np.inf] + [0.0] * 7, [1.0] * 8]], device=DEV))
    with pytest.raises(RuntimeError, match="non-finite"):
        bad.finalize()
    with pytest.raises(ValueError):
        bad.update(torch.zeros(2, 2, dtype=torch.long, device=DEV), torch.zeros(2, 3, 8, device=DEV))
    with pytest.raises(RuntimeError):
        bad.update(torch.zeros(2, 2, dtype=torch.long), torch.zeros(2, 2, 8))


@pytest.mark.parametrize("k", [1, 2, 4, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tensor_core_pass_matches_oracle(k, dtype):
    """The tensor-core Gram pass (bf16 / fp16 outputs, k in {1, 2, 4, 8}, hidden a multiple of
    128): token counts that leave a partial last block, out-of-range and repeated expert ids,
    int32 and int64 ids, and an accumulation over two calls."""
    rng = np.random.default_rng(100 + k)
    E, H = 40, 256
    for T, id_dtype in ((1, np.int64), (37, np.int32), (1000, np.int64)):
        ids = rng.integers(0, E, (T, k)).astype(id_dtype)
        if T > 3 and k > 1:
            ids[1, 0] = -3
            ids[2, k - 1] = E
            ids[3, 1] = ids[3, 0]
        out = rng.standard_normal((T, k, H)).astype(np.float32) * 0.7
        out = torch.from_numpy(out).to(dtype).float().numpy()
        stats = PairwiseScalarStats(E, device=DEV)
        stats.update(cuda(ids), cuda(out, dtype))
        stats.update(cuda(ids[::-1].copy()), cuda(out[::-1].copy(), dtype))
        acc = C.new_accumulators(E)
        C.update(acc, ids, out, E)
        C.update(acc, ids[::-1], out[::-1], E)
        close_stats(host(stats.dot), acc["dot"])
        close_stats(host(stats.target_sq_norm), acc["target_sq"])
        close_stats(host(stats.source_sq_norm), acc["source_sq"])
        close_stats(host(stats.expert_norm_sum), acc["norm_sum"])
        np.testing.assert_array_equal(host(stats.expert_norm_count), acc["norm_count"])
