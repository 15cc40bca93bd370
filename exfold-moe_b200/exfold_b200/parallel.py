"""Token sharding over the GPUs of one node (one process per GPU, torch.distributed).

Prefill: every rank routes and folds its own contiguous token shard; there is no exchange and
the ids are identical to a single-GPU run.

Decode: the expert budget needs the importance of the whole batch.  Each rank adds its routes'
importance, as exact 2^-32 fixed point, into an int64 [E] vector; the ranks sum the vectors;
each rank then selects the same top-D subset and applies the table to its own routes.  Integer
sums are exact and order independent, so the result equals the single-GPU decode bit for bit at
any world size.  Two ways to sum:

* `DecodeExchange` (one launch per layer): every rank maps every other rank's exchange buffer
  (CUDA IPC), and the decode launch itself writes its vector into all of them over NVLink,
  waits for theirs and sums (`ops.decode_sharded`);
* `sharded_decode` (three steps): importance launch, an all-reduce of E int64 through the
  process group, apply launch.
"""

from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib as L
from . import ops


class DecodeExchange:
    """Exchange buffers of the sharded decode for the ranks of one process group, one process
    per GPU of a node (at most 8 ranks).

    Every rank allocates a zeroed buffer of exf_decode_exchange_bytes(E, R) bytes, exports it
    with CUDA IPC, the handles are all-gathered through the group, each rank maps the others'
    buffers, and a barrier makes sure that every buffer is zeroed before any rank's first call
    writes into it.  `decode` is then one launch per layer; every rank must make the same
    sequence of calls (like a collective).  A device int32 `status` is set to 1 when a rank's
    vector did not arrive within `wait_ns` (2 s by default); the exchange must then be rebuilt.
    """

    def __init__(self, experts: int, *, group: dist.ProcessGroup | None = None,
                 device: torch.device | None = None):
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.experts = int(experts)
        nbytes = int(L.lib().exf_decode_exchange_bytes(self.experts, self.world))
        if nbytes <= 0:
            raise ValueError(f"no exchange for {experts} experts over {self.world} ranks "
                             "(at most 1024 experts and 8 ranks)")
        self.buffer = torch.zeros(nbytes // 8, dtype=torch.int64, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.buffer.device)
        self._imported: list[tuple[int, int]] = []
        ptrs = (ctypes.c_void_p * self.world)()
        if self.world == 1:
            ptrs[0] = self.buffer.data_ptr()
        else:
            # every rank takes the same collective steps whether its own export / imports
            # succeed or not, and all of them raise together if any rank failed
            lib = L.lib()
            handle = (ctypes.c_char * 64)()
            offset = ctypes.c_int64()
            rc = lib.exf_ipc_export(self.buffer.data_ptr(), handle, ctypes.byref(offset))
            mine = (bytes(handle), offset.value) if rc == L.EXF_OK else None
            error = None if rc == L.EXF_OK else lib.exf_last_error().decode(errors="replace")
            entries: list = [None] * self.world
            dist.all_gather_object(entries, mine, group=group)
            if all(e is not None for e in entries):
                for r, (h, off) in enumerate(entries):
                    if r == self.rank:
                        ptrs[r] = self.buffer.data_ptr()
                        continue
                    mapped = ctypes.c_void_p()
                    if lib.exf_ipc_import(h, off, ctypes.byref(mapped)) != L.EXF_OK:
                        error = lib.exf_last_error().decode(errors="replace")
                        break
                    ptrs[r] = mapped.value
                    self._imported.append((mapped.value, off))
            else:
                error = error or "another rank could not export its exchange buffer"
            torch.cuda.synchronize(self.buffer.device)
            ok = torch.tensor([0 if error else 1], dtype=torch.int32, device=self.buffer.device)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
            if int(ok.item()) == 0:
                self.close()
                raise RuntimeError(f"decode exchange setup failed: {error or 'on another rank'}")
        self.peers = ptrs

    def decode(self, weights: torch.Tensor, ids: torch.Tensor, norms: torch.Tensor,
               coeff: torch.Tensor, loss: torch.Tensor, budget: int, *, variant: str = "qwen3",
               wait_ns: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
        return ops.decode_sharded(weights, ids, norms, coeff, loss, budget, world=self.world,
                                  rank=self.rank, peers=self.peers, variant=variant,
                                  status=self.status, wait_ns=wait_ns)

    def close(self) -> None:
        """Unmap the other ranks' buffers (after every call using them has finished)."""
        for ptr, off in self._imported:
            L.check(L.lib().exf_ipc_release(ctypes.c_void_p(ptr), off))
        self._imported = []


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
