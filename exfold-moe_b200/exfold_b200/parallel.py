"""Token sharding over the GPUs of one node (one process per GPU, torch.distributed).

Prefill: every rank routes and folds its own contiguous token shard; there is no exchange and
the ids are identical to a single-GPU run.

Decode: the expert budget needs the importance of the whole batch.  Each rank adds its routes'
importance, as exact 2^-32 fixed point, into an int64 [E] vector; one all-reduce (sum) gives
every rank the batch's vector; each rank then selects the same top-D subset and applies the
table to its own routes.  Integer sums are exact and order independent, so the result equals the
single-GPU decode bit for bit at any world size.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from . import ops


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, end) of `total` tokens owned by `rank` (sizes differ by at most one)."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _importance(weights, ids, norms, importance):
    return ops.decode_importance(weights, ids, norms, importance)


def _apply(importance, weights, ids, coeff, loss, budget, variant):
    return ops.decode_apply(importance, weights, ids, coeff, loss, budget, variant=variant)


def sharded_decode(weights: torch.Tensor, ids: torch.Tensor, norms: torch.Tensor,
                   coeff: torch.Tensor, loss: torch.Tensor, budget: int, *,
                   variant: str = "qwen3", group: dist.ProcessGroup | None = None,
                   importance_fn: Callable = _importance, apply_fn: Callable = _apply,
                   ) -> tuple[torch.Tensor, torch.Tensor]:
    """Decode budget for this rank's [B_local, k] routes of a batch sharded over `group`.

    Every rank of the group must call this with the same budget and variant (one all-reduce of
    E int64 values).  `importance_fn` / `apply_fn` default to the CUDA kernels; a test may pass
    stand-ins to exercise the exchange on CPU ranks.
    """
    experts = norms.numel()
    importance = torch.zeros(experts, dtype=torch.int64, device=norms.device)
    importance_fn(weights, ids, norms, importance)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(importance, op=dist.ReduceOp.SUM, group=group)
    return apply_fn(importance, weights, ids, coeff, loss, budget, variant)
