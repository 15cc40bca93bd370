"""Drop-in for exfold/qwen3/kernels.py: the four Qwen3 ExFold routing functions on sm_100a.

Same names, arguments, return values and errors as the reference (ValueError for shapes,
RuntimeError for non-CUDA tensors); the Triton kernels are replaced by libexfold_b200.so.
Differences: the decode importance is summed exactly (2^-32 fixed point in int64) instead of by
float atomics, so the selected subset no longer depends on atomic order; and the four decode
launches (zero, accumulate, select, reroute) are one.
"""

from __future__ import annotations

import torch

from .. import ops


def project_prefill_topk(
    weights: torch.Tensor,
    expert_ids: torch.Tensor,
    coefficient: torch.Tensor,
    target_k: int,
    projection_loss: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Fold each removed slot into the retained expert with minimum loss.

    Reference: exfold/qwen3/kernels.py:97-151 (wrapper), 9-94 (kernel).
    """
    if weights.ndim != 2 or expert_ids.shape != weights.shape:
        raise ValueError("weights and expert_ids must be equally shaped matrices")
    if coefficient.ndim != 2 or coefficient.shape[0] != coefficient.shape[1]:
        raise ValueError("coefficient must be square")
    if projection_loss.shape != coefficient.shape:
        raise ValueError("projection_loss and coefficient must have the same shape")
    if not (weights.is_cuda and expert_ids.is_cuda and coefficient.is_cuda):
        raise RuntimeError("project_prefill_topk requires CUDA tensors")
    if not projection_loss.is_cuda:
        raise RuntimeError("projection_loss must be on CUDA")
    tokens, source_k = weights.shape
    target_k = max(1, min(int(target_k), source_k))
    if target_k == source_k:
        return weights.contiguous(), expert_ids.contiguous()
    if tokens == 0:
        return (torch.empty((0, target_k), device=weights.device, dtype=weights.dtype),
                torch.empty((0, target_k), device=expert_ids.device, dtype=expert_ids.dtype))
    return ops.fold_prefill(weights, expert_ids, coefficient, projection_loss, target_k,
                            variant="qwen3")


def reroute_decode_subset(
    weights: torch.Tensor,
    expert_ids: torch.Tensor,
    subset_ids: torch.Tensor,
    coefficient: torch.Tensor,
    projection_loss: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Remap decode routes outside the batch subset to minimum-loss targets.

    Reference: exfold/qwen3/kernels.py:235-292 (wrapper), 154-232 (kernel).
    """
    if weights.ndim != 2 or expert_ids.shape != weights.shape:
        raise ValueError("weights and expert_ids must be equally shaped matrices")
    if subset_ids.ndim != 1 or subset_ids.numel() == 0:
        raise ValueError("subset_ids must be a non-empty vector")
    if coefficient.ndim != 2 or coefficient.shape[0] != coefficient.shape[1]:
        raise ValueError("coefficient must be square")
    if projection_loss.shape != coefficient.shape:
        raise ValueError("projection_loss and coefficient must have the same shape")
    if not (weights.is_cuda and expert_ids.is_cuda and subset_ids.is_cuda and coefficient.is_cuda):
        raise RuntimeError("reroute_decode_subset requires CUDA tensors")
    if not projection_loss.is_cuda:
        raise RuntimeError("projection_loss must be on CUDA")
    if weights.shape[0] == 0:
        return torch.empty_like(weights), torch.empty_like(expert_ids)
    return ops.reroute_subset(weights, expert_ids, subset_ids, coefficient, projection_loss)


def remap_decode_static(
    weights: torch.Tensor,
    expert_ids: torch.Tensor,
    target_ids: torch.Tensor,
    target_scale: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Apply the precomputed source-to-target map in place.

    Reference: exfold/qwen3/kernels.py:322-356 (wrapper), 295-319 (kernel).
    """
    if weights.ndim != 2 or expert_ids.shape != weights.shape:
        raise ValueError("weights and expert_ids must be equally shaped matrices")
    if target_ids.ndim != 1 or target_scale.shape != target_ids.shape:
        raise ValueError("target_ids and target_scale must be equally shaped vectors")
    if not all(item.is_cuda for item in (weights, expert_ids, target_ids, target_scale)):
        raise RuntimeError("remap_decode_static requires CUDA tensors")
    if not weights.is_contiguous() or not expert_ids.is_contiguous():
        weights = weights.contiguous()
        expert_ids = expert_ids.contiguous()
    if weights.shape[0] == 0:
        return weights, expert_ids
    if weights.dtype in (torch.float32, torch.bfloat16, torch.float16) and \
            expert_ids.dtype in (torch.int32, torch.int64):
        return ops.static_remap_(weights, expert_ids, target_ids, target_scale)
    w = weights.float()
    i = expert_ids.to(torch.int32)
    ops.static_remap_(w, i, target_ids, target_scale)
    weights.copy_(w)
    expert_ids.copy_(i)
    return weights, expert_ids


def select_and_reroute_decode(
    weights: torch.Tensor,
    expert_ids: torch.Tensor,
    expert_norms: torch.Tensor,
    coefficient: torch.Tensor,
    projection_loss: torch.Tensor,
    subset_size: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Select the weighted Top-D expert pool and remap routes.

    Reference: exfold/qwen3/kernels.py:423-491 (wrapper), 359-420 (kernels).
    """
    if weights.ndim != 2 or expert_ids.shape != weights.shape:
        raise ValueError("weights and expert_ids must be equally shaped matrices")
    if expert_norms.ndim != 1:
        raise ValueError("expert_norms must be a vector")
    num_experts = expert_norms.numel()
    if coefficient.shape != (num_experts, num_experts):
        raise ValueError("coefficient shape does not match expert_norms")
    if projection_loss.shape != coefficient.shape:
        raise ValueError("projection_loss and coefficient must have the same shape")
    if not all(
        item.is_cuda
        for item in (weights, expert_ids, expert_norms, coefficient, projection_loss)
    ):
        raise RuntimeError("select_and_reroute_decode requires CUDA tensors")
    batch_size, _ = weights.shape
    subset_size = max(1, min(int(subset_size), num_experts))
    if subset_size == num_experts or batch_size == 0:
        return weights.contiguous(), expert_ids.contiguous()
    return ops.decode(weights, expert_ids, expert_norms, coefficient, projection_loss,
                      subset_size, variant="qwen3")
