"""The ExFold routing function of a DeepSeek-V4 MoE layer, on the B200 kernels.

`make_router(module, layer, calibration)` returns the callable that the reference installs on a
DeepSeek-V4 MoE layer (exfold/deepseek_v4/vllm_patch.py:213-368, `_make_router`), with the same
arguments, environment variables (EXFOLD_PREFILL_TOPK, EXFOLD_PREFILL_RENORM,
EXFOLD_DECODE_EXPERT_BUDGET), phase handling and results:

* prefill: the layer's router (biased sigmoid / sqrtsoftplus top-k, or the hash table on hash
  layers), then the DeepSeek-V4 prefill fold when EXFOLD_PREFILL_TOPK is below top-k.  On layers
  without a hash table the two are ONE kernel (`ops.router_fold_prefill`, variant "dsv4").
* decode: the router, then the decode budget (`fold_decode`) unless every active expert fits in
  the budget (B x k <= budget, or budget >= experts), which returns the routes unchanged.
* a batch with both decode and prefill tokens (decode tokens first, as vLLM orders them) is split,
  each part routed as above, the narrower result padded (zero weights, the last id repeated) and
  the two concatenated.

`calibration` is the 6-tuple of `exfold_b200.calibration.prepare_dsv4` ([layers, E, E] tables and
[layers, E] norms).
"""

from __future__ import annotations

import os
from collections.abc import Mapping, Sequence
from typing import Callable, Optional

import torch

from .. import ops
from .cuda_ops import fold_decode, fold_prefill
from .routing import native_route

_RENORM_MODES = {"none": 0, "router_l2": 1, "similarity_blend": 2}


def find_phase_metadata(metadata):
    """The first object with num_prefill_tokens / num_decode_tokens in vLLM's nested per-backend
    metadata containers (exfold/deepseek_v4/vllm_patch.py:51-70)."""
    pending = [metadata]
    visited: set[int] = set()
    while pending:
        item = pending.pop()
        if item is None or id(item) in visited:
            continue
        visited.add(id(item))
        if hasattr(item, "num_prefill_tokens") and hasattr(item, "num_decode_tokens"):
            return item
        if isinstance(item, Mapping):
            pending.extend(item.values())
        elif isinstance(item, Sequence) and not isinstance(item, (str, bytes, bytearray)):
            pending.extend(item)
    return None


def phase_token_counts(num_tokens: int, unavailable: Optional[tuple[int, int]] = None,
                       metadata=None) -> tuple[int, int]:
    """(decode tokens, prefill tokens) of the current batch (exfold/deepseek_v4/vllm_patch.py:
    30-48); `unavailable` is returned when vLLM has no attention metadata (e.g. profiling runs)."""
    if metadata is None:
        from vllm.forward_context import get_forward_context

        metadata = get_forward_context().attn_metadata
    item = find_phase_metadata(metadata)
    prefill = getattr(item, "num_prefill_tokens", None)
    decode = getattr(item, "num_decode_tokens", None)
    if prefill is None or decode is None:
        if unavailable is not None:
            return unavailable
        raise RuntimeError("vLLM attention metadata is unavailable")
    prefill, decode = int(prefill), int(decode)
    if prefill + decode != num_tokens:
        raise RuntimeError(
            f"MoE token mismatch: prefill={prefill}, decode={decode}, total={num_tokens}")
    return decode, prefill


def pad_routes(weights: torch.Tensor, ids: torch.Tensor, width: int):
    """Routes widened to `width` slots: zero weights, the last id repeated."""
    missing = width - ids.shape[1]
    if missing <= 0:
        return weights, ids
    zeros = torch.zeros((weights.shape[0], missing), dtype=weights.dtype, device=weights.device)
    return (torch.cat([weights, zeros], dim=1),
            torch.cat([ids, ids[:, -1:].expand(-1, missing)], dim=1))


def make_router(module, layer: int, calibration, *,
                counts_fn: Callable[[int], tuple[int, int]] | None = None) -> Callable:
    """Routing function of layer `layer` of a DeepSeek-V4 model.  `module` carries the layer's
    router settings as vLLM's DeepSeek-V4 MoE module does (n_activated_experts, n_routed_experts,
    scoring_func, renormalize, routed_scaling_factor, gate.e_score_correction_bias,
    gate.tid2eid).  `counts_fn(tokens)` gives (decode, prefill) token counts (vLLM's forward
    context by default; all prefill when it has no metadata)."""
    original_topk = int(module.n_activated_experts)
    prefill_topk = int(os.environ.get("EXFOLD_PREFILL_TOPK", original_topk))
    renorm_name = os.environ.get("EXFOLD_PREFILL_RENORM", "none").strip().lower()
    if renorm_name not in _RENORM_MODES:
        raise ValueError("EXFOLD_PREFILL_RENORM must be none, router_l2, or similarity_blend")
    renorm_mode = _RENORM_MODES[renorm_name]
    decode_budget = int(os.environ.get("EXFOLD_DECODE_EXPERT_BUDGET", 256))
    cache: dict[torch.device, tuple[torch.Tensor, ...]] = {}

    def counts(tokens: int) -> tuple[int, int]:
        if counts_fn is not None:
            return counts_fn(tokens)
        return phase_token_counts(tokens, unavailable=(0, tokens))

    def calibration_for(device: torch.device):
        c = cache.get(device)
        if c is None:
            if calibration is None:
                raise RuntimeError("ExFold routing requires calibration tensors")
            c = tuple(t[layer].to(device=device, dtype=torch.float32).contiguous()
                      for t in calibration)
            cache[device] = c
        return c

    def bias_of():
        b = getattr(module.gate, "e_score_correction_bias", None)
        return getattr(b, "data", b)

    def route_one(gating_output, phase: str, input_ids):
        tid2eid = getattr(module.gate, "tid2eid", None)
        if phase == "prefill" and prefill_topk < original_topk and tid2eid is None:
            pc, pl, pcl, _, _, _ = calibration_for(gating_output.device)
            return ops.router_fold_prefill(
                gating_output, original_topk, prefill_topk, pc, pl,
                scoring=module.scoring_func, bias=bias_of(), renormalize=module.renormalize,
                scaling=float(module.routed_scaling_factor), variant="dsv4",
                renorm_mode=renorm_mode, conf_loss=pcl)
        weights, ids = native_route(gating_output, original_topk, module.scoring_func, bias_of(),
                                    module.renormalize, float(module.routed_scaling_factor),
                                    input_ids=input_ids, tid2eid=tid2eid)
        if phase == "prefill":
            if prefill_topk >= original_topk:
                return weights, ids
            pc, pl, pcl, _, _, _ = calibration_for(gating_output.device)
            return fold_prefill(weights, ids, pc, pl, pcl, prefill_topk, renorm_mode)
        # with no more route slots than the budget every active expert is retained
        if decode_budget >= module.n_routed_experts or weights.numel() <= decode_budget:
            return weights, ids
        _, _, _, dc, dl, dn = calibration_for(gating_output.device)
        return fold_decode(weights, ids, dc, dl, dn, decode_budget)

    def router(hidden_states, gating_output, topk, renormalize, input_ids=None):
        del hidden_states, topk, renormalize  # the layer's own settings apply
        if input_ids is None:
            input_ids = getattr(module, "_dsv4_runtime_input_ids", None)
        tokens = int(gating_output.shape[0])
        num_decode, num_prefill = counts(tokens)
        if not (num_decode and num_prefill):
            w, ids = route_one(gating_output, "prefill" if num_prefill else "decode", input_ids)
        else:
            dw, di = route_one(gating_output[:num_decode], "decode",
                               None if input_ids is None else input_ids[:num_decode])
            pw, pi = route_one(gating_output[num_decode:], "prefill",
                               None if input_ids is None else input_ids[num_decode:])
            width = max(di.shape[1], pi.shape[1])
            dw, di = pad_routes(dw, di, width)
            pw, pi = pad_routes(pw, pi, width)
            w, ids = torch.cat([dw, pw], dim=0), torch.cat([di, pi], dim=0)
        dtype = getattr(module, "hash_indices_dtype", None)
        return w, (ids if dtype is None else ids.to(dtype))

    router._dsv4_accepts_input_ids = True
    return router
