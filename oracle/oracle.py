"""numpy front end of the CPU oracle (test infrastructure only).

Loads oracle/_build/libexfold_oracle.so (built from exfold_oracle.c by
oracle/build.py with -ffp-contract=off) and exposes each restated stage on
numpy arrays.  Only the tests, the smoke check and the benchmark's CPU
baseline use this module; the product library never does.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libexfold_oracle.so"

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_c = ctypes


def _load() -> ctypes.CDLL:
    if not LIB_PATH.is_file():
        from oracle import build  # noqa: WPS433 (local build recipe)

        build.build()
    lib = ctypes.CDLL(str(LIB_PATH))
    sig = {
        "orc_exp": (_c.c_float, [_c.c_float]),
        "orc_sigmoid": (_c.c_float, [_c.c_float]),
        "orc_sqrtsoftplus": (_c.c_float, [_c.c_float]),
        "orc_router_hash": (None, [_f32p, _c.c_int64, _c.c_int, _c.c_int, _c.c_int, _i64p, _i32p,
                                   _c.c_int64, _c.c_int, _c.c_float, _f32p, _i32p]),
        "orc_key": (_c.c_uint32, [_c.c_float]),
        "orc_fixed_point": (_c.c_int64, [_c.c_float]),
        "orc_router_topk": (None, [_f32p, _c.c_int64, _c.c_int, _c.c_int, _c.c_int, _c.c_void_p,
                                   _c.c_int, _c.c_float, _f32p, _i32p]),
        "orc_fold_qwen3": (None, [_f32p, _i32p, _c.c_int64, _c.c_int, _c.c_int, _f32p, _f32p,
                                  _c.c_int, _f32p, _i32p]),
        "orc_fold_dsv4": (None, [_f32p, _i32p, _c.c_int64, _c.c_int, _c.c_int, _f32p, _f32p,
                                 _f32p, _c.c_int, _c.c_int, _f32p, _i32p]),
        "orc_importance": (None, [_f32p, _i32p, _c.c_int64, _f32p, _c.c_int, _i64p]),
        "orc_order": (None, [_i64p, _c.c_int, _i32p]),
        "orc_decode_qwen3": (None, [_f32p, _i32p, _c.c_int64, _c.c_int, _f32p, _f32p, _f32p,
                                    _c.c_int, _c.c_int, _f32p, _i32p, _c.c_void_p]),
        "orc_reroute_qwen3": (None, [_f32p, _i32p, _c.c_int64, _i32p, _c.c_int, _f32p, _f32p,
                                     _c.c_int, _f32p, _i32p]),
        "orc_decode_dsv4": (None, [_f32p, _i32p, _c.c_int64, _c.c_int, _f32p, _f32p, _f32p,
                                   _c.c_int, _c.c_int, _f32p, _i32p]),
        "orc_decode_apply": (None, [_i64p, _f32p, _i32p, _c.c_int64, _f32p, _f32p, _c.c_int,
                                    _c.c_int, _c.c_int, _f32p, _i32p]),
        "orc_static_table": (None, [_f32p, _f32p, _f32p, _c.c_int, _c.c_int, _i32p, _f32p]),
        "orc_static_remap": (None, [_f32p, _i32p, _c.c_int64, _c.c_int, _i32p, _f32p]),
        "orc_moe_align_capacity": (_c.c_int64, [_c.c_int64, _c.c_int, _c.c_int, _c.c_int]),
        "orc_moe_align": (None, [_i32p, _c.c_int64, _c.c_int, _c.c_int, _c.c_int64, _i32p, _i32p,
                                 _i32p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = _load()
    return _LIB


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


SCORING = {"softmax": 0, "sigmoid": 1, "sqrtsoftplus": 2}


def router_topk(logits, top_k: int, scoring: str = "softmax", bias=None,
                renormalize: bool = True, scaling: float = 1.0):
    x = _f32(logits)
    tokens, experts = x.shape
    w = np.empty((tokens, top_k), np.float32)
    ids = np.empty((tokens, top_k), np.int32)
    b = None if bias is None else _f32(bias)
    lib().orc_router_topk(x, tokens, experts, top_k, SCORING[scoring],
                          None if b is None else b.ctypes.data, int(renormalize),
                          float(scaling), w, ids)
    return w, ids


def router_hash(logits, token_ids, table, scoring: str = "sqrtsoftplus", renormalize: bool = True,
                scaling: float = 1.0):
    """Hash routing: ids = table[token_ids] (table [rows, top_k]), weights = the unbiased
    scores at those ids."""
    x = _f32(logits)
    tokens, experts = x.shape
    tab = _i32(table)
    top_k = tab.shape[1]
    tid = np.ascontiguousarray(token_ids, dtype=np.int64)
    w = np.empty((tokens, top_k), np.float32)
    ids = np.empty((tokens, top_k), np.int32)
    lib().orc_router_hash(x, tokens, experts, top_k, SCORING[scoring], tid, tab, tab.shape[0],
                          int(renormalize), float(scaling), w, ids)
    return w, ids


def sqrtsoftplus(x):
    f = lib().orc_sqrtsoftplus
    return np.array([f(float(v)) for v in np.asarray(x, np.float32).ravel()], np.float32).reshape(
        np.shape(x))


def fold_qwen3(w, ids, coeff, loss, target_k: int):
    w, ids, coeff, loss = _f32(w), _i32(ids), _f32(coeff), _f32(loss)
    tokens, top_k = w.shape
    ow = np.empty((tokens, target_k), np.float32)
    oi = np.empty((tokens, target_k), np.int32)
    lib().orc_fold_qwen3(w, ids, tokens, top_k, target_k, coeff, loss, coeff.shape[0], ow, oi)
    return ow, oi


def fold_dsv4(w, ids, coeff, sel_loss, conf_loss, target_k: int, renorm_mode: int):
    w, ids = _f32(w), _i32(ids)
    coeff, sel_loss, conf_loss = _f32(coeff), _f32(sel_loss), _f32(conf_loss)
    tokens, top_k = w.shape
    ow = np.empty((tokens, target_k), np.float32)
    oi = np.empty((tokens, target_k), np.int32)
    lib().orc_fold_dsv4(w, ids, tokens, top_k, target_k, coeff, sel_loss, conf_loss,
                        coeff.shape[0], int(renorm_mode), ow, oi)
    return ow, oi


def importance(w, ids, norms):
    w, ids, norms = _f32(w).ravel(), _i32(ids).ravel(), _f32(norms)
    out = np.empty(norms.shape[0], np.int64)
    lib().orc_importance(w, ids, w.size, norms, norms.shape[0], out)
    return out


def order(imp):
    imp = np.ascontiguousarray(imp, dtype=np.int64)
    out = np.empty(imp.shape[0], np.int32)
    lib().orc_order(imp, imp.shape[0], out)
    return out


def decode_qwen3(w, ids, norms, coeff, loss, budget: int):
    w, ids, norms, coeff, loss = _f32(w), _i32(ids), _f32(norms), _f32(coeff), _f32(loss)
    batch, top_k = w.shape
    ow = np.empty_like(w)
    oi = np.empty_like(ids)
    subset = np.full(max(budget, 1), -1, np.int32)
    lib().orc_decode_qwen3(w, ids, batch, top_k, norms, coeff, loss, coeff.shape[0], budget,
                           ow, oi, subset.ctypes.data)
    return ow, oi, subset[:budget]


def reroute_qwen3(w, ids, subset, coeff, loss):
    w, ids, subset, coeff, loss = _f32(w), _i32(ids), _i32(subset), _f32(coeff), _f32(loss)
    ow = np.empty_like(w)
    oi = np.empty_like(ids)
    lib().orc_reroute_qwen3(w, ids, w.size, subset, subset.size, coeff, loss, coeff.shape[0], ow, oi)
    return ow, oi


def decode_dsv4(w, ids, norms, coeff, loss, budget: int):
    w, ids, norms, coeff, loss = _f32(w), _i32(ids), _f32(norms), _f32(coeff), _f32(loss)
    batch, top_k = w.shape
    ow = np.empty_like(w)
    oi = np.empty_like(ids)
    lib().orc_decode_dsv4(w, ids, batch, top_k, norms, coeff, loss, coeff.shape[0], budget,
                          ow, oi)
    return ow, oi


def decode_apply(imp, w, ids, coeff, loss, budget: int, variant: str = "qwen3"):
    """Select / table / apply from a given (e.g. all-reduced) importance vector."""
    imp = np.ascontiguousarray(imp, dtype=np.int64)
    w, ids, coeff, loss = _f32(w), _i32(ids), _f32(coeff), _f32(loss)
    ow = np.empty_like(w)
    oi = np.empty_like(ids)
    lib().orc_decode_apply(imp, w, ids, w.size, coeff, loss, coeff.shape[0], budget,
                           1 if variant == "dsv4" else 0, ow, oi)
    return ow, oi


def static_table(norms, coeff, loss, budget: int):
    norms, coeff, loss = _f32(norms), _f32(coeff), _f32(loss)
    experts = norms.shape[0]
    target = np.empty(experts, np.int32)
    scale = np.empty(experts, np.float32)
    lib().orc_static_table(norms, coeff, loss, experts, budget, target, scale)
    return target, scale


def static_remap(w, ids, target, scale):
    w, ids = _f32(w).copy(), _i32(ids).copy()
    lib().orc_static_remap(w.reshape(-1), ids.reshape(-1), w.size, _i32(target).size, _i32(target),
                           _f32(scale))
    return w, ids


def moe_align(ids, experts: int, block_size: int, pad_sorted: bool = False):
    flat = _i32(ids).ravel()
    cap = lib().orc_moe_align_capacity(flat.size, experts, block_size, int(pad_sorted))
    sorted_ids = np.empty(cap, np.int32)
    expert_ids = np.empty((cap + block_size - 1) // block_size, np.int32)
    post = np.empty(1, np.int32)
    lib().orc_moe_align(flat, flat.size, experts, block_size, cap, sorted_ids, expert_ids, post)
    return sorted_ids, expert_ids, post


def router_fold(logits, top_k: int, target_k: int, coeff, loss, *, scoring="softmax", bias=None,
                variant="qwen3", conf_loss=None, renorm_mode=0, renormalize=True, scaling=1.0):
    """Router top-k followed by the prefill fold (composition of the above)."""
    w, ids = router_topk(logits, top_k, scoring, bias, renormalize, scaling)
    if variant == "qwen3":
        return fold_qwen3(w, ids, coeff, loss, target_k)
    return fold_dsv4(w, ids, coeff, loss, loss if conf_loss is None else conf_loss, target_k,
                     renorm_mode)


def threads() -> int:
    return 1 if os.environ.get("EXF_ORACLE_THREADS") is None else int(os.environ["EXF_ORACLE_THREADS"])
