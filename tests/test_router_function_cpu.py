"""Host logic of the Qwen3 routing function (exfold/qwen3/vllm_patch.py:65-95, 115-121): phase
detection from EXFOLD_FORCE_PHASE or vLLM attention metadata, and the decode-policy check."""

from __future__ import annotations

import types

import pytest
import torch

from exfold_b200.qwen3 import router as R


def meta(prefill, decode):
    return types.SimpleNamespace(num_prefill_tokens=prefill, num_decode_tokens=decode)


def test_forced_phase(monkeypatch):
    monkeypatch.setenv("EXFOLD_FORCE_PHASE", "Prefill ")
    assert R.phase(7) == "prefill"
    monkeypatch.setenv("EXFOLD_FORCE_PHASE", "decode")
    assert R.phase(7) == "decode"
    monkeypatch.setenv("EXFOLD_FORCE_PHASE", "both")
    with pytest.raises(ValueError):
        R.phase(7)


def test_phase_from_metadata():
    assert R.phase_of_metadata(meta(12, 0), 12) == "prefill"
    assert R.phase_of_metadata(meta(0, 5), 5) == "decode"
    assert R.phase_of_metadata({"a": object(), "b": meta(0, 3)}, 3) == "decode"
    with pytest.raises(RuntimeError, match="mixed"):
        R.phase_of_metadata(meta(2, 3), 5)
    with pytest.raises(RuntimeError, match="disagrees"):
        R.phase_of_metadata(meta(2, 0), 5)
    with pytest.raises(RuntimeError, match="unavailable"):
        R.phase_of_metadata(None, 5)
    with pytest.raises(RuntimeError, match="unavailable"):
        R.phase_of_metadata({"a": object()}, 5)


def test_decode_policy_is_checked(monkeypatch):
    t = torch.zeros(4, 4)
    monkeypatch.setenv("EXFOLD_QWEN3_DECODE_POLICY", "random")
    with pytest.raises(ValueError, match="EXFOLD_QWEN3_DECODE_POLICY"):
        R.make_router(t, t, torch.ones(4), 4, 2)
    monkeypatch.setenv("EXFOLD_QWEN3_DECODE_POLICY", "STATIC_NORM")
    assert callable(R.make_router(t, t, torch.ones(4), 4, 2))


def test_decode_budget_below_one(monkeypatch):
    """select_and_reroute_decode clamps the subset to [1, E] (exfold/qwen3/kernels.py:447): a
    dynamic-policy budget of 0 or less decodes with a subset of 1; the static policy refuses it
    when the router is made (the reference's table build fails there)."""
    t = torch.zeros(8, 8)
    monkeypatch.setenv("EXFOLD_QWEN3_DECODE_POLICY", "static_norm")
    for budget in (0, -3):
        with pytest.raises(ValueError, match="decode_budget"):
            R.make_router(t, t, torch.ones(8), 4, budget)
    monkeypatch.setenv("EXFOLD_QWEN3_DECODE_POLICY", "dynamic")
    seen = []
    monkeypatch.setattr(R.ops, "router_topk", lambda logits, k, **kw: (
        torch.full((logits.shape[0], k), 1.0 / k), torch.zeros(logits.shape[0], k,
                                                                dtype=torch.int32)))
    monkeypatch.setattr(R.ops, "decode", lambda w, ids, n, c, l_, budget, **kw: (
        seen.append(budget), (w, ids))[1])
    for budget in (0, -3, 2):
        router = R.make_router(t, t, torch.ones(8), 4, budget, phase_fn=lambda n: "decode")
        router(None, torch.zeros(3, 8), 2, True)
    assert seen == [1, 1, 2]


# ---- DeepSeek-V4 (exfold/deepseek_v4/vllm_patch.py:30-70, 213-368) ---------------------------
def test_dsv4_phase_counts_and_padding():
    from exfold_b200.deepseek_v4 import router as D

    nested = {"x": [None, {"y": meta(6, 2)}]}
    assert D.find_phase_metadata(nested).num_prefill_tokens == 6
    assert D.phase_token_counts(8, metadata=nested) == (2, 6)
    with pytest.raises(RuntimeError, match="mismatch"):
        D.phase_token_counts(9, metadata=nested)
    assert D.phase_token_counts(5, unavailable=(0, 5), metadata={"x": 1}) == (0, 5)
    with pytest.raises(RuntimeError, match="unavailable"):
        D.phase_token_counts(5, metadata=[])
    w = torch.tensor([[0.5, 0.25, 0.125]])
    ids = torch.tensor([[7, 3, 9]], dtype=torch.int32)
    pw, pi = D.pad_routes(w, ids, 5)
    assert pw.tolist() == [[0.5, 0.25, 0.125, 0.0, 0.0]] and pi.tolist() == [[7, 3, 9, 9, 9]]
    assert D.pad_routes(w, ids, 3)[1] is ids


def test_dsv4_renorm_mode_is_checked(monkeypatch):
    from exfold_b200.deepseek_v4 import router as D

    module = types.SimpleNamespace(n_activated_experts=8, n_routed_experts=256)
    monkeypatch.setenv("EXFOLD_PREFILL_RENORM", "softmax")
    with pytest.raises(ValueError, match="EXFOLD_PREFILL_RENORM"):
        D.make_router(module, 0, None)
    monkeypatch.setenv("EXFOLD_PREFILL_RENORM", "Similarity_Blend")
    assert D.make_router(module, 0, None)._dsv4_accepts_input_ids
