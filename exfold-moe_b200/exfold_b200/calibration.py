"""Calibration table preparation and per-device caching.

The transforms consume the tensors the reference's artifact loaders produce; these helpers
restate those loaders' preparation steps so callers that build tables themselves get the same
values:

* prepare_qwen3: exfold/qwen3/vllm_patch.py:45-61 (shape and value checks; coeff := 0 where
  loss >= 1e30; coeff diagonal := 1; loss diagonal := 1e30).
* prepare_dsv4: exfold/deepseek_v4/vllm_patch.py:82-170 (key fallbacks; EXFOLD_MAX_PROJECTION_LOSS
  masking of the decode loss; diagonal fixes; norms clamped to float32 eps).
* DeviceTables: the per-device copy cache of vllm_patch.py:146-157 / 236-260.
* PairwiseScalarStats: the accumulator that builds the tables (exfold/qwen3/calibration.py:9-140)
  on the GPU kernels exf_calibration_update / _finalize / _norms.

Arrays may be numpy arrays or torch tensors; the result has the input's kind.
"""

from __future__ import annotations

import os

import numpy as np
import torch

_SENTINEL = 1.0e30


def _t(a) -> torch.Tensor:
    return a.detach().clone().float() if isinstance(a, torch.Tensor) else torch.from_numpy(
        np.array(a, dtype=np.float32, copy=True))


def _back(t: torch.Tensor, like):
    return t if isinstance(like, torch.Tensor) else t.numpy()


def prepare_qwen3(coeff, loss, norms, *, validate: bool = True):
    """[layers, E, E] coeff / loss and [layers, E] norms as the Qwen3 artifact loader leaves them."""
    c, l_, n = _t(coeff), _t(loss), _t(norms)
    if c.ndim != 3 or c.shape[1] != c.shape[2]:
        raise ValueError("coeff must have shape [layers, experts, experts]")
    if l_.shape != c.shape:
        raise ValueError("loss and coeff must have identical shapes")
    if n.shape != c.shape[:2]:
        raise ValueError("expert_norms must have shape [layers, experts]")
    if validate:
        if not all(torch.isfinite(x).all() for x in (c, l_, n)):
            raise ValueError("artifact contains non-finite values")
        if torch.any(l_ < 0) or torch.any(n <= 0):
            raise ValueError("loss must be non-negative and expert_norms positive")
    c = c.masked_fill(l_ >= _SENTINEL, 0.0)
    c.diagonal(dim1=-2, dim2=-1).fill_(1.0)
    l_.diagonal(dim1=-2, dim2=-1).fill_(_SENTINEL)
    return _back(c, coeff), _back(l_, loss), _back(n, norms)


def prepare_dsv4(payload: dict):
    """(prefill_coeff, prefill_loss, prefill_confidence_loss, decode_coeff, decode_loss, norms)
    from a DeepSeek-V4 calibration payload, as the DeepSeek-V4 loader builds them."""

    def get(*keys):
        for k in keys:
            if k in payload and payload[k] is not None:
                return payload[k]
        return None

    pc = _t(get("prefill_coeff", "coeff"))
    pl = _t(get("prefill_selection_loss", "selection_loss", "loss"))
    conf = get("prefill_confidence_loss")
    pcl = _t(conf) if conf is not None else pl.clone()
    dc = _t(get("decode_coeff", "routing_coeff", "coeff"))
    dl = _t(get("decode_loss", "routing_loss", "loss"))
    norms_payload = get("decode_norms", "routing_norms", "norms")
    if pc.ndim != 3 or pc.shape[1] != pc.shape[2]:
        raise ValueError(f"prefill_coeff must have shape [layers, experts, experts], got {pc.shape}")
    for name, t in (("prefill_loss", pl), ("prefill_confidence_loss", pcl), ("decode_coeff", dc),
                    ("decode_loss", dl)):
        if t.shape != pc.shape:
            raise ValueError(f"{name} shape {t.shape} does not match {pc.shape}")
    if norms_payload is None:
        raise ValueError("Calibration artifact is missing norms")
    if isinstance(norms_payload, dict):
        norms = torch.stack([_t(norms_payload[i]) for i in range(pc.shape[0])])
    else:
        norms = _t(norms_payload)
    if norms.shape != pc.shape[:2]:
        raise ValueError(f"norms must have shape {pc.shape[:2]}, got {norms.shape}")
    for name, t in (("prefill_coeff", pc), ("prefill_loss", pl), ("prefill_confidence_loss", pcl),
                    ("decode_coeff", dc), ("decode_loss", dl)):
        if not torch.isfinite(t).all():
            raise ValueError(f"Calibration {name} contains non-finite values")
    max_loss = float(os.environ.get("EXFOLD_MAX_PROJECTION_LOSS", "1e30"))
    dl.masked_fill_(dl > max_loss, _SENTINEL)
    pc.diagonal(dim1=-2, dim2=-1).fill_(1.0)
    pl.diagonal(dim1=-2, dim2=-1).fill_(_SENTINEL)
    pcl.diagonal(dim1=-2, dim2=-1).fill_(0.0)
    dc.diagonal(dim1=-2, dim2=-1).fill_(1.0)
    dl.diagonal(dim1=-2, dim2=-1).fill_(_SENTINEL)
    norms = norms.clamp_min(torch.finfo(torch.float32).eps).contiguous()
    return pc, pl, pcl, dc, dl, norms


class DeviceTables:
    """Per-device cache of one layer's tables (copied once per device, then reused)."""

    def __init__(self, *tables: torch.Tensor):
        self._host = tuple(t.contiguous() for t in tables)
        self._cache: dict[torch.device, tuple[torch.Tensor, ...]] = {}

    def on(self, device: torch.device) -> tuple[torch.Tensor, ...]:
        cached = self._cache.get(device)
        if cached is None:
            cached = tuple(t.to(device=device, non_blocking=True) for t in self._host)
            self._cache[device] = cached
        return cached


class PairwiseScalarStats(torch.nn.Module):
    """One MoE layer's directed scalar projectors, accumulated on the GPU: the drop-in for
    PairwiseScalarStats (exfold/qwen3/calibration.py:9-140) with the same constructor, buffers
    (dot, target_sq_norm, source_sq_norm, expert_norm_sum, expert_norm_count; fp64) and methods.
    update / finalize / expert_norms run the exf_calibration_* kernels; the inputs of update must
    be CUDA tensors (RuntimeError otherwise, as the reference's CUDA paths raise).  finalize reads
    back the kernel's non-finite flag (a host synchronisation, like the reference's isfinite
    checks)."""

    default_loss = _SENTINEL

    def __init__(self, num_experts: int, ridge: float = 1e-3, clip_min: float = -4.0,
                 clip_max: float = 4.0, device=None) -> None:
        super().__init__()
        if num_experts <= 1:
            raise ValueError("num_experts must be greater than one")
        if ridge <= 0:
            raise ValueError("ridge must be positive")
        if clip_min >= clip_max:
            raise ValueError("clip_min must be smaller than clip_max")
        if num_experts > 1024:
            raise ValueError("num_experts must be at most 1024")
        dev = torch.device(device) if device is not None else torch.device("cuda")
        shape = (num_experts, num_experts)
        for name, shp in (("dot", shape), ("target_sq_norm", shape), ("source_sq_norm", shape),
                          ("expert_norm_sum", (num_experts,)),
                          ("expert_norm_count", (num_experts,))):
            self.register_buffer(name, torch.zeros(shp, dtype=torch.float64, device=dev),
                                 persistent=False)
        self.num_experts = num_experts
        self.ridge = ridge
        self.clip_min = clip_min
        self.clip_max = clip_max

    @torch.no_grad()
    def update(self, expert_ids: torch.Tensor, expert_outputs: torch.Tensor) -> None:
        """Accumulate co-routed expert outputs: expert_ids [tokens, top_k], expert_outputs
        [tokens, top_k, hidden] (unweighted; fp32, bf16 or fp16)."""
        from . import _lib as L
        from .ops import _IDT, _WDT, _stream

        if expert_ids.ndim != 2:
            raise ValueError("expert_ids must have shape [tokens, top_k]")
        if expert_outputs.shape[:2] != expert_ids.shape or expert_outputs.ndim != 3:
            raise ValueError("expert_outputs must have shape [tokens, top_k, hidden_size]")
        if not (expert_ids.is_cuda and expert_outputs.is_cuda):
            raise RuntimeError("PairwiseScalarStats.update expects CUDA tensors")
        out = expert_outputs if expert_outputs.dtype in _WDT else expert_outputs.float()
        out = out.contiguous()
        if out.data_ptr() % 16:
            out = out.clone()
        ids = expert_ids if expert_ids.dtype in _IDT else expert_ids.to(torch.int64)
        ids = ids.contiguous()
        tokens, top_k, hidden = out.shape
        L.check(L.lib().exf_calibration_update(
            out.data_ptr(), _WDT[out.dtype], ids.data_ptr(), _IDT[ids.dtype], tokens, top_k,
            hidden, self.num_experts, self.dot.data_ptr(), self.target_sq_norm.data_ptr(),
            self.source_sq_norm.data_ptr(), self.expert_norm_sum.data_ptr(),
            self.expert_norm_count.data_ptr(), _stream(out.device)))

    @torch.no_grad()
    def finalize(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Return the clipped scalar matrix and relative projection loss (fp32 [E, E])."""
        from . import _lib as L
        from .ops import _stream

        E, dev = self.num_experts, self.dot.device
        coeff = torch.empty((E, E), dtype=torch.float32, device=dev)
        loss = torch.empty((E, E), dtype=torch.float32, device=dev)
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        L.check(L.lib().exf_calibration_finalize(
            self.dot.data_ptr(), self.target_sq_norm.data_ptr(), self.source_sq_norm.data_ptr(), E,
            float(self.ridge), float(self.clip_min), float(self.clip_max), coeff.data_ptr(),
            loss.data_ptr(), flag.data_ptr(), _stream(dev)))
        if int(flag.item()):
            raise RuntimeError("non-finite calibration statistics")
        return coeff, loss

    @torch.no_grad()
    def expert_norms(self) -> torch.Tensor:
        """Return the mean output norm of each routed expert (fp32 [E])."""
        from . import _lib as L
        from .ops import _stream

        dev = self.expert_norm_sum.device
        norms = torch.empty(self.num_experts, dtype=torch.float32, device=dev)
        L.check(L.lib().exf_calibration_norms(self.expert_norm_sum.data_ptr(),
                                              self.expert_norm_count.data_ptr(), self.num_experts,
                                              norms.data_ptr(), _stream(dev)))
        return norms
