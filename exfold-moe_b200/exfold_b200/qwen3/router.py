"""The ExFold routing function of a Qwen3 MoE layer, on the B200 kernels.

`make_router` returns the callable that the reference installs as vLLM's
`FusedMoE.custom_routing_function` (exfold/qwen3/vllm_patch.py:108-217, `_make_router`), with the
same arguments, environment variables, phase detection, errors and results:

* prefill with a budget below top-k: router and fold in ONE kernel (`ops.router_fold_prefill`)
  instead of vLLM's `fused_topk` followed by `project_prefill_topk` (no [tokens, k] round trip);
* decode with a budget below the expert count: the router, then either the one-launch dynamic
  decode (`ops.decode`, policy "dynamic") or the static remap by the calibrated norms
  (`ops.static_table` once per device, then `ops.static_remap_`, policy "static_norm");
* otherwise the plain softmax top-k router.

Results are (weights fp32, ids int32) [tokens, k'], k' = min(prefill budget, top-k) at prefill.
"""

from __future__ import annotations

import os
from typing import Callable

import torch

from .. import ops


def phase(tokens: int) -> str:
    """"prefill" or "decode" for a batch of `tokens` (exfold/qwen3/vllm_patch.py:65-95):
    EXFOLD_FORCE_PHASE when set, else vLLM's attention metadata of the current forward pass.
    Mixed prefill/decode batches are refused, as in the reference."""
    forced = os.environ.get("EXFOLD_FORCE_PHASE", "").strip().lower()
    if forced:
        if forced not in {"prefill", "decode"}:
            raise ValueError("EXFOLD_FORCE_PHASE must be 'prefill' or 'decode'")
        return forced
    from vllm.forward_context import get_forward_context

    return phase_of_metadata(get_forward_context().attn_metadata, tokens)


def phase_of_metadata(metadata, tokens: int) -> str:
    """The phase from vLLM attention metadata (one object, or a dict of per-layer objects)."""
    if isinstance(metadata, dict):
        metadata = next((m for m in metadata.values() if hasattr(m, "num_prefill_tokens")), None)
    prefill = getattr(metadata, "num_prefill_tokens", None)
    decode = getattr(metadata, "num_decode_tokens", None)
    if prefill is None or decode is None:
        raise RuntimeError("vLLM attention metadata is unavailable")
    prefill, decode = int(prefill), int(decode)
    if prefill + decode != tokens:
        raise RuntimeError("MoE token count disagrees with vLLM attention metadata")
    if prefill and decode:
        raise RuntimeError("mixed prefill/decode batches are unsupported; disable chunked prefill")
    return "prefill" if prefill else "decode"


def make_router(coefficient: torch.Tensor, loss: torch.Tensor, norms: torch.Tensor,
                prefill_budget: int, decode_budget: int, *,
                phase_fn: Callable[[int], str] = phase) -> Callable:
    """Routing function of one layer; tables [E, E] and norms [E] as prepared by
    `exfold_b200.calibration.prepare_qwen3` (host or device tensors).  `phase_fn` maps a token
    count to "prefill" / "decode" (vLLM's forward context by default)."""
    policy = os.environ.get("EXFOLD_QWEN3_DECODE_POLICY", "dynamic").lower()
    if policy not in {"dynamic", "static_norm"}:
        raise ValueError("EXFOLD_QWEN3_DECODE_POLICY must be 'dynamic' or 'static_norm'")
    experts = int(coefficient.shape[0])
    if policy == "static_norm" and decode_budget < experts and decode_budget < 1:
        # the reference builds the static table here and fails on an empty retained set
        raise ValueError("decode_budget must be >= 1 for the static_norm decode policy")
    tables: dict[torch.device, tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}
    static: dict[torch.device, tuple[torch.Tensor, torch.Tensor]] = {}

    def tables_for(device: torch.device):
        t = tables.get(device)
        if t is None:
            t = tuple(x.to(device=device, dtype=torch.float32).contiguous()
                      for x in (coefficient, loss, norms))
            tables[device] = t
        return t

    def static_for(device: torch.device, budget: int):
        s = static.get(device)
        if s is None:
            c, l_, n = tables_for(device)
            s = ops.static_table(n, c, l_, budget)
            static[device] = s
        return s

    def router(hidden_states: torch.Tensor, gating_output: torch.Tensor, topk: int,
               renormalize: bool) -> tuple[torch.Tensor, torch.Tensor]:
        del hidden_states  # the routing depends on the gate logits only
        c, l_, n = tables_for(gating_output.device)
        if phase_fn(gating_output.shape[0]) == "prefill":
            target_k = min(prefill_budget, topk)
            if target_k < topk:
                w, ids = ops.router_fold_prefill(gating_output, topk, target_k, c, l_,
                                                 renormalize=renormalize)
            else:
                w, ids = ops.router_topk(gating_output, topk, renormalize=renormalize)
        else:
            w, ids = ops.router_topk(gating_output, topk, renormalize=renormalize)
            subset = min(decode_budget, gating_output.shape[1])
            if subset < gating_output.shape[1]:
                if policy == "static_norm":
                    target, scale = static_for(gating_output.device, decode_budget)
                    w, ids = ops.static_remap_(w, ids, target, scale)
                else:
                    # select_and_reroute_decode clamps the subset to [1, E]
                    # (exfold/qwen3/kernels.py:447)
                    w, ids = ops.decode(w, ids, n, c, l_, max(1, subset), variant="qwen3")
        return w.float(), ids.int()

    router.experts = experts
    return router
