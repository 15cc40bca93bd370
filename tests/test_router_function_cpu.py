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
