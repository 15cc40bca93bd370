"""Drop-in for exfold/deepseek_v4/cuda_ops.py: registers torch.ops.dsv4_exfold on sm_100a.

Schemas are those of exfold/deepseek_v4/csrc/exfold_ops.cpp:22-31 and the fake (meta)
implementations those of cuda_ops.py:27-54, so torch.compile and CUDA-graph capture see the same
op.  The CUDA implementations call libexfold_b200.so.  Argument checks follow
exfold_kernels.cu:203-249, 288-292 and raise RuntimeError like TORCH_CHECK; the expert count is
any E <= 1024 instead of exactly 256.
"""

from __future__ import annotations

import torch

from .. import ops

_LIB = torch.library.Library("dsv4_exfold", "DEF")
_LIB.define(
    "prefill(Tensor weights, Tensor ids, Tensor coefficient, Tensor selection_loss, "
    "Tensor confidence_loss, int target_k, int renorm_mode) -> (Tensor, Tensor)")
_LIB.define(
    "decode(Tensor weights, Tensor ids, Tensor coefficient, Tensor loss, Tensor norms, "
    "int budget) -> (Tensor, Tensor)")

_WEIGHT_DTYPES = (torch.float32, torch.float16, torch.bfloat16, torch.float64)
_INDEX_DTYPES = (torch.uint8, torch.int8, torch.int16, torch.int32, torch.int64)


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_common(weights, ids, coefficient, loss) -> None:
    """exfold_kernels.cu:203-224."""
    _check(weights.is_cuda and ids.is_cuda, "routing tensors must be CUDA")
    _check(coefficient.is_cuda and loss.is_cuda, "calibration tensors must be CUDA")
    _check(weights.is_contiguous() and ids.is_contiguous(), "routing tensors must be contiguous")
    _check(coefficient.is_contiguous() and loss.is_contiguous(),
           "calibration tensors must be contiguous")
    _check(weights.dim() == 2 and ids.shape == weights.shape,
           "routing tensors must be [tokens, topk]")
    _check(coefficient.dtype == torch.float32 and loss.dtype == torch.float32,
           "calibration tensors must be float32")
    _check(coefficient.dim() == 2 and coefficient.shape[0] == coefficient.shape[1]
           and loss.shape == coefficient.shape and coefficient.shape[0] <= 1024,
           "calibration must be square [E, E] with E <= 1024")
    _check(weights.shape[1] <= 8, "topk exceeds the fused kernel limit")
    _check(weights.dtype in _WEIGHT_DTYPES and ids.dtype in _INDEX_DTYPES,
           "unsupported routing dtype")


def _prefill_cuda(weights, ids, coefficient, selection_loss, confidence_loss, target_k: int,
                  renorm_mode: int):
    """exfold_prefill_cuda (exfold_kernels.cu:228-278)."""
    _check_common(weights, ids, coefficient, selection_loss)
    _check(confidence_loss.is_cuda, "confidence_loss must be CUDA")
    _check(confidence_loss.is_contiguous(), "confidence_loss must be contiguous")
    _check(confidence_loss.dtype == torch.float32, "confidence_loss must be float32")
    _check(confidence_loss.shape == coefficient.shape,
           "confidence_loss must match coefficient shape")
    _check(0 < target_k <= weights.shape[1], "invalid target_k")
    _check(0 <= renorm_mode <= 2,
           "prefill renorm_mode must be 0 (none), 1 (router_l2), or 2 (similarity_blend)")
    return ops.fold_prefill(weights, ids, coefficient, selection_loss, int(target_k),
                            variant="dsv4", renorm_mode=int(renorm_mode),
                            conf_loss=confidence_loss)


def _decode_cuda(weights, ids, coefficient, loss, norms, budget: int):
    """exfold_decode_cuda (exfold_kernels.cu:280-322)."""
    _check_common(weights, ids, coefficient, loss)
    experts = coefficient.shape[0]
    _check(norms.is_cuda and norms.is_contiguous(), "norms must be contiguous CUDA")
    _check(norms.dtype == torch.float32 and norms.numel() == experts,
           f"norms must be float32 [{experts}]")
    _check(0 < budget <= experts, "invalid expert budget")
    if weights.shape[0] == 0:
        return torch.empty_like(weights), torch.empty_like(ids)
    return ops.decode(weights, ids, norms, coefficient, loss, int(budget), variant="dsv4")


_LIB.impl("prefill", _prefill_cuda, "CUDA")
_LIB.impl("decode", _decode_cuda, "CUDA")


@torch.library.register_fake("dsv4_exfold::prefill")
def _prefill_fake(weights, ids, coefficient, selection_loss, confidence_loss, target_k: int,
                  renorm_mode: int):
    del coefficient, selection_loss, confidence_loss, renorm_mode
    return (weights.new_empty((weights.shape[0], target_k)),
            ids.new_empty((ids.shape[0], target_k)))


@torch.library.register_fake("dsv4_exfold::decode")
def _decode_fake(weights, ids, coefficient, loss, norms, budget: int):
    del coefficient, loss, norms, budget
    return torch.empty_like(weights), torch.empty_like(ids)


def fold_prefill(weights, ids, coefficient, selection_loss, confidence_loss, target_k: int,
                 renorm_mode: int = 0):
    """exfold/deepseek_v4/cuda_ops.py:57-74."""
    return torch.ops.dsv4_exfold.prefill(weights.contiguous(), ids.contiguous(), coefficient,
                                         selection_loss, confidence_loss, target_k, renorm_mode)


def fold_decode(weights, ids, coefficient, loss, norms, budget: int):
    """exfold/deepseek_v4/cuda_ops.py:77-92."""
    return torch.ops.dsv4_exfold.decode(weights.contiguous(), ids.contiguous(), coefficient, loss,
                                        norms, budget)
