"""CPU checks of the DeepSeek-V4 router extras in the oracle and the host layer.

* the sqrtsoftplus score (vLLM fused_topk_bias scoring_func="sqrtsoftplus", F.softplus(x).sqrt())
  against a float64 evaluation;
* the biased sqrtsoftplus top-k and hash routing (hash_indices_table[input_tokens]) against the
  torch semantics of vLLM's fused_topk_bias (restated below), as called from
  exfold/deepseek_v4/vllm_patch.py:175-209;
* EXFOLD_MAX_PROJECTION_LOSS in the DeepSeek-V4 calibration preparation
  (exfold/deepseek_v4/vllm_patch.py:154-157).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from exfold_b200 import calibration
from exfold_b200 import workloads as W
from oracle import oracle as O


def test_sqrtsoftplus_accuracy():
    x = np.linspace(-87, 40, 40001, dtype=np.float32)
    got = O.sqrtsoftplus(x).astype(np.float64)
    ref = F.softplus(torch.from_numpy(x).double()).sqrt().numpy()
    assert np.max(np.abs(got - ref) / ref) < 2e-7
    # below the exp clamp the score stays at its (negligible) value at -87
    low = O.sqrtsoftplus(np.array([-88.0, -1000.0, -np.inf], np.float32))
    assert np.all(low == O.sqrtsoftplus(np.array([-87.0], np.float32))[0])
    assert O.sqrtsoftplus(np.array([np.inf], np.float32))[0] == np.inf


def _torch_topk_bias(x, bias, k, renormalize, scaling, scores_fn):
    """vLLM fused_topk_bias restated: select on scores + bias, weight by the unbiased scores."""
    xt = torch.from_numpy(x).double()
    scores = scores_fn(xt)
    choice = scores + (0.0 if bias is None else torch.from_numpy(bias).double())
    ids = torch.topk(choice, k, dim=-1).indices
    w = scores.gather(1, ids)
    if renormalize:
        w = w / w.sum(-1, keepdim=True).clamp(min=1e-20)
    return (w * scaling).numpy(), ids.numpy(), np.sort(choice.numpy(), axis=1)[:, ::-1]


def test_sqrtsoftplus_router_matches_torch_semantics():
    x = W.logits(303, 3000, 256)
    bias = W.router_bias(303, 256)
    sqsp = lambda t: F.softplus(t).sqrt()
    for b in (bias, None):
        for renorm, scaling in ((True, 1.0), (False, 2.5)):
            w, ids = O.router_topk(x, 8, "sqrtsoftplus", b, renorm, scaling)
            rw, rids, srt = _torch_topk_bias(x, b, 8, renorm, scaling, sqsp)
            # rows whose 8th and 9th selection keys are not within float rounding of each other
            clear = (srt[:, 7] - srt[:, 8]) > 1e-5
            assert clear.mean() > 0.95
            np.testing.assert_array_equal(np.sort(ids[clear], 1), np.sort(rids[clear], 1))
            order = np.argsort(ids[clear], 1)
            np.testing.assert_allclose(np.take_along_axis(w[clear], order, 1),
                                       np.take_along_axis(rw[clear], np.argsort(rids[clear], 1), 1),
                                       rtol=1e-5, atol=0)


def test_hash_routing_matches_torch_semantics():
    x = W.logits(404, 500, 256)
    rng = np.random.default_rng(4)
    table = np.stack([rng.choice(256, 6, replace=False) for _ in range(1000)]).astype(np.int32)
    tokens = rng.integers(0, 1000, 500).astype(np.int64)
    for scoring, fn in (("sqrtsoftplus", lambda t: F.softplus(t).sqrt()),
                        ("sigmoid", torch.sigmoid)):
        w, ids = O.router_hash(x, tokens, table, scoring, True, 1.5)
        rids = table[tokens]
        np.testing.assert_array_equal(ids, rids)
        s = fn(torch.from_numpy(x).double()).gather(1, torch.from_numpy(rids).long())
        rw = (s / s.sum(-1, keepdim=True) * 1.5).numpy()
        np.testing.assert_allclose(w, rw, rtol=2e-6, atol=0)
    # out-of-range token ids and table entries never index outside the inputs
    bad_tab = table.copy()
    bad_tab[0, 2] = 999
    w, ids = O.router_hash(x[:3], np.array([0, -1, 1000], np.int64), bad_tab, "sigmoid")
    assert ids[0, 2] == 999 and w[0, 2] == 0.0 and np.isclose(w[0].sum(), 1.0)
    assert np.all(ids[1:] == -1) and np.all(w[1:] == 0.0)


def test_max_projection_loss_threshold(monkeypatch):
    rng = np.random.default_rng(5)
    L_, E = 2, 8
    payload = {
        "prefill_coeff": torch.from_numpy(rng.random((L_, E, E), dtype=np.float32)),
        "prefill_selection_loss": torch.from_numpy(rng.random((L_, E, E), dtype=np.float32)),
        "decode_coeff": torch.from_numpy(rng.random((L_, E, E), dtype=np.float32)),
        "decode_loss": torch.from_numpy(2 * rng.random((L_, E, E), dtype=np.float32)),
        "decode_norms": torch.from_numpy(rng.random((L_, E), dtype=np.float32)),
    }
    monkeypatch.setenv("EXFOLD_MAX_PROJECTION_LOSS", "0.75")
    dl = calibration.prepare_dsv4({k: v.clone() for k, v in payload.items()})[4]
    src = payload["decode_loss"]
    off = ~torch.eye(E, dtype=torch.bool).expand(L_, E, E)
    assert torch.all(dl[off & (src > 0.75)] == 1e30)
    assert torch.equal(dl[off & (src <= 0.75)], src[off & (src <= 0.75)])
    monkeypatch.delenv("EXFOLD_MAX_PROJECTION_LOSS")
    dl = calibration.prepare_dsv4({k: v.clone() for k, v in payload.items()})[4]
    assert torch.equal(dl[off], src[off])


def test_native_route_requires_input_ids_for_hash_layers():
    import pytest

    from exfold_b200.deepseek_v4.routing import native_route

    with pytest.raises(RuntimeError, match="requires input_ids"):
        native_route(torch.zeros(2, 256), 8, "sqrtsoftplus",
                     tid2eid=torch.zeros(10, 8, dtype=torch.int32))
