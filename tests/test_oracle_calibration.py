"""The calibration oracle (oracle/calibration.py) against the reference's own accumulator.

tests/golden/calibration_reference.npz holds the statistics, coefficient / loss tables and
expert norms that PairwiseScalarStats (exfold/qwen3/calibration.py) produced on CPU for random
routes with duplicate expert ids and never-routed experts (tests/golden/make_golden.py).  The
reference forms the per-token products in fp32; the oracle works in float64, hence the
tolerances.  The reference's own closed-form and clipping cases
(tests/test_qwen3_calibration.py) are restated at the end.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import calibration as C

GOLDEN = Path(__file__).resolve().parent / "golden" / "calibration_reference.npz"


@pytest.mark.parametrize("case", ["a", "b"])
def test_oracle_matches_reference_accumulator(case):
    g = np.load(GOLDEN)
    ids, outputs = g[f"{case}_ids"], g[f"{case}_outputs"]
    E = g[f"{case}_dot"].shape[0]
    acc = C.new_accumulators(E)
    half = ids.shape[0] // 2
    C.update(acc, ids[:half], outputs[:half], E)
    C.update(acc, ids[half:], outputs[half:], E)
    for key, ref in (("dot", "dot"), ("target_sq", "target_sq"), ("source_sq", "source_sq"),
                     ("norm_sum", "norm_sum"), ("norm_count", "norm_count")):
        # the reference's fp32 dot products carry rounding of about 1e-7 of the array's scale
        want = g[f"{case}_{ref}"]
        np.testing.assert_allclose(acc[key], want, rtol=1e-6, atol=1e-6 * np.abs(want).max())
    coeff, loss = C.finalize(acc)
    np.testing.assert_allclose(coeff, g[f"{case}_coeff"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(loss, g[f"{case}_loss"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(C.expert_norms(acc), g[f"{case}_norms"], rtol=1e-6)


def test_oracle_closed_form_and_clipping():
    acc = C.new_accumulators(3)
    ids = np.array([[0, 1], [0, 1]])
    out = np.array([[[2.0, 0.0], [1.0, 0.0]], [[0.0, 3.0], [0.0, 1.0]]])
    C.update(acc, ids, out, 3)
    coeff, loss = C.finalize(acc, ridge=1e-3)
    w = np.linalg.norm(out[:, 0], axis=-1)
    expected = (w * (out[:, 0] * out[:, 1]).sum(-1)).sum() / ((w * (out[:, 1] ** 2).sum(-1)).sum()
                                                               + 1e-3)
    assert np.isclose(coeff[0, 1], np.float32(expected))
    assert loss[0, 1] < 1.0 and coeff[2, 0] == 0 and loss[2, 0] == C.DEFAULT_LOSS
    assert np.array_equal(np.diag(coeff), np.ones(3, np.float32))
    acc = C.new_accumulators(2)
    C.update(acc, np.array([[0, 1]]), np.array([[[10.0, 0.0], [1.0, 0.0]]]), 2)
    assert C.finalize(acc, ridge=1e-6)[0][0, 1] == 4.0
    np.testing.assert_allclose(C.expert_norms(acc), [10.0, 1.0])
