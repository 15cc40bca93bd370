"""ctypes binding of libexfold_b200.so (the C ABI declared in include/exfold_b200.h).

The library is loaded from exfold-moe_b200/lib/libexfold_b200.so, or from the path in the
EXFOLD_B200_LIBRARY environment variable.  There is no fallback: a missing library raises
RuntimeError at first use.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

DEFAULT_PATH = Path(__file__).resolve().parent.parent / "lib" / "libexfold_b200.so"

EXF_OK, EXF_ERR_INVALID, EXF_ERR_UNSUPPORTED, EXF_ERR_CUDA = 0, -1, -2, -3
EXF_F32, EXF_BF16, EXF_F16 = 0, 1, 2
EXF_I32, EXF_I64 = 0, 1
EXF_SOFTMAX, EXF_SIGMOID, EXF_SQRTSOFTPLUS = 0, 1, 2
EXF_QWEN3, EXF_DSV4 = 0, 1

_vp, _i, _i64, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float

# name -> (restype, argtypes); the order follows include/exfold_b200.h
SIGNATURES = {
    "exf_abi_version": (_i, []),
    "exf_last_error": (ctypes.c_char_p, []),
    "exf_router_tile_min_rows": (_i64, [_i64]),
    "exf_router_topk": (_i, [_vp, _i, _i64, _i, _i, _i, _vp, _i, _f, _vp, _vp, _vp]),
    "exf_router_fold_prefill": (_i, [_vp, _i, _i64, _i, _i, _i, _i, _vp, _i, _f, _i, _i, _i, _vp,
                                     _vp, _vp, _vp, _vp, _vp]),
    "exf_router_hash": (_i, [_vp, _i, _i64, _i, _i, _i, _vp, _i, _vp, _i64, _i, _f, _vp, _vp,
                             _vp]),
    "exf_calibration_update": (_i, [_vp, _i, _vp, _i, _i64, _i, _i, _i, _vp, _vp, _vp, _vp, _vp,
                                    _vp]),
    "exf_calibration_finalize": (_i, [_vp, _vp, _vp, _i, ctypes.c_double, ctypes.c_double,
                                      ctypes.c_double, _vp, _vp, _vp, _vp]),
    "exf_calibration_norms": (_i, [_vp, _vp, _i, _vp, _vp]),
    "exf_fold_prefill": (_i, [_vp, _i, _vp, _i, _i64, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp,
                              _vp]),
    "exf_decode": (_i, [_vp, _i, _vp, _i, _i64, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "exf_decode_importance": (_i, [_vp, _i, _vp, _i, _i64, _i, _vp, _vp, _vp]),
    "exf_decode_apply": (_i, [_vp, _vp, _i, _vp, _i, _i64, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp,
                              _vp]),
    "exf_decode_exchange_bytes": (_i64, [_i, _i]),
    "exf_decode_sharded": (_i, [_vp, _i, _vp, _i, _i64, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i, _vp,
                                ctypes.c_uint64, _vp, _vp, _vp, _vp, _vp]),
    "exf_ipc_export": (_i, [_vp, _vp, ctypes.POINTER(_i64)]),
    "exf_ipc_import": (_i, [_vp, _i64, ctypes.POINTER(_vp)]),
    "exf_ipc_release": (_i, [_vp, _i64]),
    "exf_reroute_subset": (_i, [_vp, _i, _vp, _i, _i64, _i, _i, _vp, _i, _vp, _vp, _vp, _vp, _vp]),
    "exf_static_table": (_i, [_vp, _vp, _vp, _i, _i, _vp, _vp, _vp]),
    "exf_static_remap": (_i, [_vp, _i, _vp, _i, _i64, _i, _vp, _vp, _vp]),
    "exf_moe_align_capacity": (_i64, [_i64, _i, _i, _i]),
    "exf_moe_align_workspace_bytes": (_i64, [_i64, _i]),
    "exf_moe_align": (_i, [_vp, _i, _i64, _i, _i, _i64, _vp, _vp, _vp, _vp, _i64, _vp]),
    "exf_moe_align_noalloc": (_i, [_vp, _i, _i64, _i, _i, _i64, _vp, _vp, _vp, _vp]),
    "exf_fused_experts_workspace_bytes": (_i64, [_i64, _i, _i, _i, _i]),
    "exf_fused_experts": (_i, [_vp, _vp, _vp, _i64, _i, _vp, _vp, _i, _i, _i, _vp, _vp, _i64, _vp,
                               _vp]),
    "exf_decode_fused_experts_workspace_bytes": (_i64, [_i64, _i, _i, _i, _i]),
    "exf_decode_fused_experts": (_i, [_vp, _vp, _vp, _i64, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp,
                                      _i, _i, _vp, _vp, _vp, _vp, _i64, _vp, _vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    return Path(os.environ.get("EXFOLD_B200_LIBRARY", str(DEFAULT_PATH)))


def lib() -> ctypes.CDLL:
    """The loaded library (RuntimeError if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not path.is_file():
                raise RuntimeError(
                    f"ExFold B200 library is missing: {path} "
                    "(build it with: python exfold-moe_b200/build.py)")
            handle = ctypes.CDLL(str(path))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


class ExfoldError(RuntimeError):
    """A CUDA-level failure reported by the library."""


def check(rc: int) -> None:
    if rc == EXF_OK:
        return
    msg = (lib().exf_last_error() or b"").decode(errors="replace")
    if rc == EXF_ERR_INVALID:
        raise ValueError(msg)
    if rc == EXF_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise ExfoldError(msg)
