"""DeepSeek-V4 router on the B200 kernels: the routing call of the patched DeepSeek-V4 MoE layer
(exfold/deepseek_v4/vllm_patch.py:175-209, `_native_route` -> vLLM fused_topk_bias).

`native_route` takes the same inputs as that call: router logits, top-k, the layer's scoring
function ("sigmoid" or "sqrtsoftplus"; "softmax" without hash routing), the expert-selection
correction bias, renormalize, routed_scaling_factor, and for hash-MoE layers the token ids with
the gate's tid2eid table.  It returns (weights fp32, ids int32) [tokens, top_k].  Errors follow
the reference: a hash table without input ids raises RuntimeError.
"""

from __future__ import annotations

import torch

from .. import ops


def native_route(router_logits: torch.Tensor, topk: int, scoring_func: str = "sigmoid",
                 correction_bias: torch.Tensor | None = None, renormalize: bool = True,
                 routed_scaling_factor: float = 1.0, input_ids: torch.Tensor | None = None,
                 tid2eid: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    if tid2eid is not None:
        if input_ids is None:
            raise RuntimeError("Hash-MoE routing requires input_ids")
        if tid2eid.dim() != 2 or tid2eid.shape[1] != topk:
            raise ValueError(f"tid2eid must be [vocab, {topk}], got {tuple(tid2eid.shape)}")
        return ops.router_hash(router_logits, input_ids, tid2eid, scoring_func, renormalize,
                               routed_scaling_factor)
    return ops.router_topk(router_logits, topk, scoring_func, correction_bias, renormalize,
                           routed_scaling_factor)
