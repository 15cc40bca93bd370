"""torch front end of libexfold_b200.so.

Each function allocates its outputs with torch (so CUDA-graph capture uses the graph's memory
pool), passes raw device pointers to the C ABI and launches on the current CUDA stream.  Nothing
here synchronises with the host.  Weights are float32 / bfloat16 / float16 and ids int32 /
int64 natively; other dtypes are converted on the way in and back on the way out.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib as L

_WDT = {torch.float32: L.EXF_F32, torch.bfloat16: L.EXF_BF16, torch.float16: L.EXF_F16}
_IDT = {torch.int32: L.EXF_I32, torch.int64: L.EXF_I64}
_SCORING = {"softmax": L.EXF_SOFTMAX, "sigmoid": L.EXF_SIGMOID, "sqrtsoftplus": L.EXF_SQRTSOFTPLUS}
_VARIANT = {"qwen3": L.EXF_QWEN3, "dsv4": L.EXF_DSV4}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("ExFold B200 ops require CUDA tensors")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("ExFold B200 ops require all tensors on one device")
    return dev


def _f32c(t: torch.Tensor | None) -> torch.Tensor | None:
    if t is None:
        return None
    return t.contiguous() if t.dtype == torch.float32 else t.float().contiguous()


def _logits_in(t: torch.Tensor) -> torch.Tensor:
    """Router logits in their own dtype when it is fp32 / bf16 / fp16 (the kernels convert
    16-bit logits exactly), else as fp32; contiguous and 16-byte aligned."""
    t = t if t.dtype in _WDT else t.float()
    return _aligned(t)


def _aligned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _weights_in(w: torch.Tensor) -> torch.Tensor:
    return w.contiguous() if w.dtype in _WDT else w.float().contiguous()


def _ids_in(ids: torch.Tensor) -> torch.Tensor:
    return ids.contiguous() if ids.dtype in _IDT else ids.to(torch.int32).contiguous()


# ---- router ---------------------------------------------------------------------------------
def router_topk(logits: torch.Tensor, top_k: int, scoring: str = "softmax",
                bias: torch.Tensor | None = None, renormalize: bool = True,
                scaling: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k routing of [tokens, experts] logits (fp32, bf16 or fp16 natively) -> (weights fp32,
    ids int32) [tokens, top_k]."""
    dev = _require_cuda(logits, bias)
    x = _logits_in(logits)
    tokens, experts = x.shape
    b = None if bias is None else _aligned(_f32c(bias))
    w = torch.empty((tokens, top_k), dtype=torch.float32, device=dev)
    ids = torch.empty((tokens, top_k), dtype=torch.int32, device=dev)
    L.check(L.lib().exf_router_topk(x.data_ptr(), _WDT[x.dtype], tokens, experts, top_k,
                                    _SCORING[scoring],
                                    _ptr(b), int(renormalize), float(scaling), w.data_ptr(),
                                    ids.data_ptr(), _stream(dev)))
    return w, ids


def router_hash(logits: torch.Tensor, token_ids: torch.Tensor, table: torch.Tensor,
                scoring: str = "sqrtsoftplus", renormalize: bool = True,
                scaling: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Hash routing: routes table[token_ids] (table [rows, top_k], in table order) weighted by
    the unbiased scores of those experts -> (weights fp32, ids int32) [tokens, top_k]."""
    dev = _require_cuda(logits, token_ids, table)
    x = _logits_in(logits)
    tokens, experts = x.shape
    tid = _ids_in(token_ids.reshape(-1))
    if tid.numel() != tokens:
        raise ValueError(f"token_ids has {tid.numel()} entries for {tokens} tokens")
    tab = table.to(torch.int32).contiguous()
    if tab.dim() != 2:
        raise ValueError("table must be [rows, top_k]")
    top_k = tab.shape[1]
    w = torch.empty((tokens, top_k), dtype=torch.float32, device=dev)
    ids = torch.empty((tokens, top_k), dtype=torch.int32, device=dev)
    L.check(L.lib().exf_router_hash(x.data_ptr(), _WDT[x.dtype], tokens, experts, top_k,
                                    _SCORING[scoring],
                                    tid.data_ptr(), _IDT[tid.dtype], tab.data_ptr(), tab.shape[0],
                                    int(renormalize), float(scaling), w.data_ptr(), ids.data_ptr(),
                                    _stream(dev)))
    return w, ids


def router_fold_prefill(logits: torch.Tensor, top_k: int, target_k: int, coeff: torch.Tensor,
                        sel_loss: torch.Tensor, *, scoring: str = "softmax",
                        bias: torch.Tensor | None = None, renormalize: bool = True,
                        scaling: float = 1.0, variant: str = "qwen3", renorm_mode: int = 0,
                        conf_loss: torch.Tensor | None = None,
                        out: tuple[torch.Tensor, torch.Tensor] | None = None,
                        ) -> tuple[torch.Tensor, torch.Tensor]:
    """Router + prefill fold in one pass.

    logits [tokens, E] with tables [E, E], or [layers, tokens, E] with tables [layers, E, E]
    (and bias [layers, E]).  Returns (weights fp32, ids int32) [..., tokens, target_k].
    """
    dev = _require_cuda(logits, coeff, sel_loss, bias, conf_loss)
    x = _logits_in(logits)
    layers = 1 if x.dim() == 2 else x.shape[0]
    tokens, experts = x.shape[-2], x.shape[-1]
    coeff, sel_loss = _f32c(coeff), _f32c(sel_loss)
    conf_loss = _f32c(conf_loss)
    b = None if bias is None else _aligned(_f32c(bias))
    shape = (*x.shape[:-1], target_k)
    if out is None:
        w = torch.empty(shape, dtype=torch.float32, device=dev)
        ids = torch.empty(shape, dtype=torch.int32, device=dev)
    else:
        w, ids = out
    L.check(L.lib().exf_router_fold_prefill(
        x.data_ptr(), _WDT[x.dtype], tokens, layers, experts, top_k, _SCORING[scoring], _ptr(b),
        int(renormalize), float(scaling), target_k, _VARIANT[variant], int(renorm_mode),
        coeff.data_ptr(), sel_loss.data_ptr(), _ptr(conf_loss), w.data_ptr(), ids.data_ptr(),
        _stream(dev)))
    return w, ids


# ---- prefill fold of given routes -------------------------------------------------------------
def router_tile_min_rows(rows: int | None = None) -> int:
    """The launch size (tokens x layers) from which the router calls use the tile kernels
    (exf_router_tile_min_rows): smaller launches take the generic kernel, whose latency is lower
    there; both give identical results.  Sets it when `rows` is given; returns the previous value."""
    return int(L.lib().exf_router_tile_min_rows(-1 if rows is None else int(rows)))


def fold_prefill(weights: torch.Tensor, ids: torch.Tensor, coeff: torch.Tensor,
                 sel_loss: torch.Tensor, target_k: int, *, variant: str = "qwen3",
                 renorm_mode: int = 0, conf_loss: torch.Tensor | None = None,
                 ) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(weights, ids, coeff, sel_loss, conf_loss)
    w_in, i_in = _weights_in(weights), _ids_in(ids)
    tokens, top_k = w_in.shape
    coeff, sel_loss, conf_loss = _f32c(coeff), _f32c(sel_loss), _f32c(conf_loss)
    ow = torch.empty((tokens, target_k), dtype=w_in.dtype, device=dev)
    oi = torch.empty((tokens, target_k), dtype=i_in.dtype, device=dev)
    if tokens > 0:
        L.check(L.lib().exf_fold_prefill(
            w_in.data_ptr(), _WDT[w_in.dtype], i_in.data_ptr(), _IDT[i_in.dtype], tokens, top_k,
            target_k, coeff.shape[0], _VARIANT[variant], int(renorm_mode), coeff.data_ptr(),
            sel_loss.data_ptr(), _ptr(conf_loss), ow.data_ptr(), oi.data_ptr(), _stream(dev)))
    return ow.to(weights.dtype), oi.to(ids.dtype)


# ---- decode ---------------------------------------------------------------------------------
def decode(weights: torch.Tensor, ids: torch.Tensor, norms: torch.Tensor, coeff: torch.Tensor,
           loss: torch.Tensor, budget: int, *, variant: str = "qwen3",
           subset_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Importance, top-`budget` select, target table and apply in one launch."""
    dev = _require_cuda(weights, ids, norms, coeff, loss)
    w_in, i_in = _weights_in(weights), _ids_in(ids)
    batch, top_k = w_in.shape
    norms, coeff, loss = _f32c(norms), _f32c(coeff), _f32c(loss)
    ow, oi = torch.empty_like(w_in), torch.empty_like(i_in)
    L.check(L.lib().exf_decode(
        w_in.data_ptr(), _WDT[w_in.dtype], i_in.data_ptr(), _IDT[i_in.dtype], batch, top_k,
        coeff.shape[0], int(budget), _VARIANT[variant], norms.data_ptr(), coeff.data_ptr(),
        loss.data_ptr(), ow.data_ptr(), oi.data_ptr(), _ptr(subset_out), _stream(dev)))
    return ow.to(weights.dtype), oi.to(ids.dtype)


def decode_importance(weights: torch.Tensor, ids: torch.Tensor, norms: torch.Tensor,
                      importance: torch.Tensor) -> torch.Tensor:
    """Add this shard's fixed-point importance into `importance` (int64 [E], caller-zeroed)."""
    dev = _require_cuda(weights, ids, norms, importance)
    if importance.dtype != torch.int64 or not importance.is_contiguous():
        raise ValueError("importance must be a contiguous int64 vector")
    w_in, i_in = _weights_in(weights), _ids_in(ids)
    norms = _f32c(norms)
    L.check(L.lib().exf_decode_importance(
        w_in.data_ptr(), _WDT[w_in.dtype], i_in.data_ptr(), _IDT[i_in.dtype], w_in.numel(),
        norms.numel(), norms.data_ptr(), importance.data_ptr(), _stream(dev)))
    return importance


def decode_apply(importance: torch.Tensor, weights: torch.Tensor, ids: torch.Tensor,
                 coeff: torch.Tensor, loss: torch.Tensor, budget: int, *, variant: str = "qwen3",
                 subset_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Select / table / apply from an (all-reduced) importance vector."""
    dev = _require_cuda(importance, weights, ids, coeff, loss)
    w_in, i_in = _weights_in(weights), _ids_in(ids)
    batch, top_k = w_in.shape
    coeff, loss = _f32c(coeff), _f32c(loss)
    ow, oi = torch.empty_like(w_in), torch.empty_like(i_in)
    L.check(L.lib().exf_decode_apply(
        importance.data_ptr(), w_in.data_ptr(), _WDT[w_in.dtype], i_in.data_ptr(),
        _IDT[i_in.dtype], batch, top_k, coeff.shape[0], int(budget), _VARIANT[variant],
        coeff.data_ptr(), loss.data_ptr(), ow.data_ptr(), oi.data_ptr(), _ptr(subset_out),
        _stream(dev)))
    return ow.to(weights.dtype), oi.to(ids.dtype)


def decode_sharded(weights: torch.Tensor, ids: torch.Tensor, norms: torch.Tensor,
                   coeff: torch.Tensor, loss: torch.Tensor, budget: int, *, world: int, rank: int,
                   peers: "ctypes.Array", variant: str = "qwen3",
                   status: torch.Tensor | None = None, wait_ns: int = 0,
                   subset_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Decode budget of this rank's shard in one launch, the importance exchanged with the other
    ranks over peer memory (`peers`: every rank's exchange buffer as mapped here, a ctypes array
    of `world` device pointers; see `exfold_b200.parallel.DecodeExchange`)."""
    dev = _require_cuda(weights, ids, norms, coeff, loss, status)
    w_in, i_in = _weights_in(weights), _ids_in(ids)
    batch, top_k = w_in.shape
    norms, coeff, loss = _f32c(norms), _f32c(coeff), _f32c(loss)
    ow, oi = torch.empty_like(w_in), torch.empty_like(i_in)
    L.check(L.lib().exf_decode_sharded(
        w_in.data_ptr(), _WDT[w_in.dtype], i_in.data_ptr(), _IDT[i_in.dtype], batch, top_k,
        coeff.shape[0], int(budget), _VARIANT[variant], norms.data_ptr(), coeff.data_ptr(),
        loss.data_ptr(), int(world), int(rank), peers, int(wait_ns), ow.data_ptr(), oi.data_ptr(),
        _ptr(subset_out), _ptr(status), _stream(dev)))
    return ow.to(weights.dtype), oi.to(ids.dtype)


def reroute_subset(weights: torch.Tensor, ids: torch.Tensor, subset: torch.Tensor,
                   coeff: torch.Tensor, loss: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(weights, ids, subset, coeff, loss)
    w_in, i_in = _weights_in(weights), _ids_in(ids)
    batch, top_k = w_in.shape
    sub = subset.to(torch.int32).contiguous()
    coeff, loss = _f32c(coeff), _f32c(loss)
    ow, oi = torch.empty_like(w_in), torch.empty_like(i_in)
    L.check(L.lib().exf_reroute_subset(
        w_in.data_ptr(), _WDT[w_in.dtype], i_in.data_ptr(), _IDT[i_in.dtype], batch, top_k,
        coeff.shape[0], sub.data_ptr(), sub.numel(), coeff.data_ptr(), loss.data_ptr(),
        ow.data_ptr(), oi.data_ptr(), _stream(dev)))
    return ow.to(weights.dtype), oi.to(ids.dtype)


def static_table(norms: torch.Tensor, coeff: torch.Tensor, loss: torch.Tensor,
                 budget: int) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(norms, coeff, loss)
    norms, coeff, loss = _f32c(norms), _f32c(coeff), _f32c(loss)
    experts = norms.numel()
    target = torch.empty(experts, dtype=torch.int32, device=dev)
    scale = torch.empty(experts, dtype=torch.float32, device=dev)
    L.check(L.lib().exf_static_table(norms.data_ptr(), coeff.data_ptr(), loss.data_ptr(), experts,
                                     int(budget), target.data_ptr(), scale.data_ptr(),
                                     _stream(dev)))
    return target, scale


def static_remap_(weights: torch.Tensor, ids: torch.Tensor, target: torch.Tensor,
                  scale: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """In place: ids = target[ids], weights *= scale[ids] (contiguous natively-typed tensors)."""
    dev = _require_cuda(weights, ids, target, scale)
    if weights.dtype not in _WDT or ids.dtype not in _IDT:
        raise TypeError("static_remap_ needs float32/bfloat16/float16 weights and int32/int64 ids")
    if not (weights.is_contiguous() and ids.is_contiguous()):
        raise ValueError("static_remap_ works in place on contiguous tensors")
    t = target.to(torch.int32).contiguous()
    s = _f32c(scale)
    if weights.numel() > 0:
        L.check(L.lib().exf_static_remap(weights.data_ptr(), _WDT[weights.dtype], ids.data_ptr(),
                                         _IDT[ids.dtype], weights.numel(), t.numel(), t.data_ptr(),
                                         s.data_ptr(), _stream(dev)))
    return weights, ids


# ---- moe_align ------------------------------------------------------------------------------
def moe_align_capacity(numel: int, experts: int, block_size: int, pad_sorted: bool = False) -> int:
    return int(L.lib().exf_moe_align_capacity(numel, experts, block_size, int(pad_sorted)))


def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int,
                         pad_sorted_ids: bool = False,
                         ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(sorted_token_ids, expert_ids, num_tokens_post_padded) as vLLM's moe_align_block_size."""
    dev = _require_cuda(topk_ids)
    ids = _ids_in(topk_ids)
    numel = ids.numel()
    cap = moe_align_capacity(numel, num_experts, block_size, pad_sorted_ids)
    sorted_ids = torch.empty(cap, dtype=torch.int32, device=dev)
    expert_ids = torch.empty((cap + block_size - 1) // block_size, dtype=torch.int32, device=dev)
    post = torch.empty(1, dtype=torch.int32, device=dev)
    ws_bytes = int(L.lib().exf_moe_align_workspace_bytes(numel, num_experts))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    L.check(L.lib().exf_moe_align(ids.data_ptr(), _IDT[ids.dtype], numel, num_experts, block_size,
                                  cap, sorted_ids.data_ptr(), expert_ids.data_ptr(),
                                  post.data_ptr(), ws.data_ptr(), ws_bytes, _stream(dev)))
    return sorted_ids, expert_ids, post


# ---- grouped SwiGLU experts (tcgen05) ------------------------------------------------------------
def decode_fused_experts(x: torch.Tensor, weights: torch.Tensor, ids: torch.Tensor,
                         norms: torch.Tensor, coeff: torch.Tensor, loss: torch.Tensor, budget: int,
                         w13: torch.Tensor, w2: torch.Tensor, *, variant: str = "qwen3",
                         status: torch.Tensor | None = None
                         ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Decode expert budget, then the expert layer over the remapped routes: returns
    (y, w_out, ids_out).

    `decode` followed by `fused_experts`, with moe_align done inside the decode launch and the
    routes of a token that the budget sends to the same expert merged (weights summed, the
    expert computed once).  w_out / ids_out equal `decode`'s outputs bit for bit (fp32 / int32);
    y equals `fused_experts(x, w_out, ids_out, w13, w2)` within bf16 rounding.  At most 256
    experts, top_k <= 8 and 8192 routes.
    """
    dev = _require_cuda(x, weights, ids, norms, coeff, loss, w13, w2)
    if x.dtype != torch.bfloat16 or w13.dtype != torch.bfloat16 or w2.dtype != torch.bfloat16:
        raise TypeError("decode_fused_experts computes in bf16: x, w13 and w2 must be bfloat16")
    x, w13, w2 = x.contiguous(), w13.contiguous(), w2.contiguous()
    w_in = weights.float().contiguous()
    i_in = ids.to(torch.int32).contiguous()
    batch, top_k = w_in.shape
    hidden = x.shape[1]
    experts, two_i, _ = w13.shape
    inter = two_i // 2
    norms, coeff, loss = _f32c(norms), _f32c(coeff), _f32c(loss)
    ow, oi = torch.empty_like(w_in), torch.empty_like(i_in)
    y = torch.empty_like(x)
    ws_bytes = int(L.lib().exf_decode_fused_experts_workspace_bytes(batch, top_k, experts,
                                                                    hidden, inter))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    L.check(L.lib().exf_decode_fused_experts(
        x.data_ptr(), w_in.data_ptr(), i_in.data_ptr(), batch, top_k, experts, int(budget),
        _VARIANT[variant], norms.data_ptr(), coeff.data_ptr(), loss.data_ptr(), w13.data_ptr(),
        w2.data_ptr(), hidden, inter, ow.data_ptr(), oi.data_ptr(), y.data_ptr(), ws.data_ptr(),
        ws_bytes, _ptr(status), _stream(dev)))
    return y, ow, oi


def fused_experts(x: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor,
                  w13: torch.Tensor, w2: torch.Tensor,
                  status: torch.Tensor | None = None) -> torch.Tensor:
    """y = sum_j topk_w[:, j] * W2[e] (silu(W1[e] x) * (W3[e] x)), e = topk_ids[:, j].

    x bf16 [T, H]; w13 bf16 [E, 2I, H] (gate rows then up rows); w2 bf16 [E, H, I].  The layout
    and meaning follow vLLM's fused_experts.  `status` (int32 [1] on the device) is set to 1 if a
    pipeline wait timed out.
    """
    dev = _require_cuda(x, topk_w, topk_ids, w13, w2)
    if x.dtype != torch.bfloat16 or w13.dtype != torch.bfloat16 or w2.dtype != torch.bfloat16:
        raise TypeError("fused_experts computes in bf16: x, w13 and w2 must be bfloat16")
    x, w13, w2 = x.contiguous(), w13.contiguous(), w2.contiguous()
    tokens, hidden = x.shape
    experts, two_i, _ = w13.shape
    inter = two_i // 2
    top_k = topk_ids.shape[1]
    ids = topk_ids.to(torch.int32).contiguous()
    wts = topk_w.float().contiguous()
    y = torch.empty_like(x)
    ws_bytes = int(L.lib().exf_fused_experts_workspace_bytes(tokens, top_k, experts, hidden,
                                                             inter))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    L.check(L.lib().exf_fused_experts(x.data_ptr(), wts.data_ptr(), ids.data_ptr(), tokens, top_k,
                                      w13.data_ptr(), w2.data_ptr(), experts, hidden, inter,
                                      y.data_ptr(), ws.data_ptr(), ws_bytes, _ptr(status),
                                      _stream(dev)))
    return y
