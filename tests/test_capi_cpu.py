"""CPU checks of the C ABI: the library loads without a GPU, exports every symbol the header
declares, and rejects bad arguments before touching the device."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from exfold_b200 import _lib as L

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "exfold_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"EXF_API\s+[\w\s\*]+?\b(exf_\w+)\s*\(", text)))


def test_library_loads_and_exports_header_symbols():
    lib = L.lib()
    names = declared_symbols()
    assert len(names) >= 14
    for name in names:
        assert hasattr(lib, name), name
        assert name in L.SIGNATURES, f"{name} has no ctypes signature"
    assert set(L.SIGNATURES) == set(names)
    assert lib.exf_abi_version() == 3


def test_router_tile_threshold_knob():
    """exf_router_tile_min_rows sets the launch size from which the tile router kernels are
    taken and returns the previous value; a negative argument only reads it."""
    lib = L.lib()
    default = lib.exf_router_tile_min_rows(-1)
    assert default == 32768
    try:
        assert lib.exf_router_tile_min_rows(0) == default
        assert lib.exf_router_tile_min_rows(-1) == 0
        assert lib.exf_router_tile_min_rows(1 << 40) == 0
        assert lib.exf_router_tile_min_rows(-5) == 1 << 40
    finally:
        lib.exf_router_tile_min_rows(default)
    assert lib.exf_router_tile_min_rows(-1) == default


def test_capacity_matches_vllm_rule():
    lib = L.lib()
    assert lib.exf_moe_align_capacity(12, 5, 4, 0) == 12 + 5 * 3
    assert lib.exf_moe_align_capacity(12, 5, 4, 1) == 28
    assert lib.exf_moe_align_capacity(3, 128, 16, 0) == 48  # numel < experts
    assert lib.exf_moe_align_workspace_bytes(1000, 128) == 0
    assert lib.exf_moe_align_workspace_bytes(196608, 256) == 96 * 256 * 4


def call(name, *args):
    return getattr(L.lib(), name)(*args)


def last_error() -> str:
    return L.lib().exf_last_error().decode()


def test_argument_validation_without_gpu():
    fake = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    rc = call("exf_router_topk", fake, 0, 10, 96, 8, 0, None, 1, 1.0, fake, fake, None)
    assert rc == L.EXF_ERR_UNSUPPORTED and "experts" in last_error()
    rc = call("exf_router_topk", fake, 0, 10, 128, 9, 0, None, 1, 1.0, fake, fake, None)
    assert rc == L.EXF_ERR_INVALID and "top_k" in last_error()
    rc = call("exf_router_topk", ctypes.c_void_p(20), 0, 10, 128, 8, 0, None, 1, 1.0, fake, fake,
              None)
    assert rc == L.EXF_ERR_INVALID and "aligned" in last_error()
    rc = call("exf_router_topk", fake, 5, 10, 128, 8, 0, None, 1, 1.0, fake, fake, None)
    assert rc == L.EXF_ERR_INVALID and "EXF_BF16" in last_error()
    rc = call("exf_router_topk", ctypes.c_void_p(24), L.EXF_BF16, 10, 128, 8, 0, None, 1, 1.0,
              fake, fake, None)
    assert rc == L.EXF_ERR_INVALID and "aligned" in last_error()
    rc = call("exf_router_fold_prefill", fake, 0, 10, 1, 128, 8, 0, None, 1, 1.0, 9, 0, 0, fake,
              fake,
              None, fake, fake, None)
    assert rc == L.EXF_ERR_INVALID and "target_k" in last_error()
    rc = call("exf_router_fold_prefill", fake, 0, 10, 1, 128, 8, 0, None, 1, 1.0, 4, 0, 2, fake,
              fake,
              None, fake, fake, None)
    assert rc == L.EXF_ERR_INVALID and "renorm_mode" in last_error()
    rc = call("exf_fold_prefill", fake, 7, fake, 0, 10, 8, 4, 128, 0, 0, fake, fake, None, fake,
              fake, None)
    assert rc == L.EXF_ERR_INVALID and "dtype" in last_error()
    rc = call("exf_decode", fake, 0, fake, 0, 4, 8, 128, 0, 0, fake, fake, fake, fake, fake, None,
              None)
    assert rc == L.EXF_ERR_INVALID and "budget" in last_error()
    rc = call("exf_decode", fake, 0, fake, 0, 4, 8, 2048, 64, 0, fake, fake, fake, fake, fake,
              None, None)
    assert rc == L.EXF_ERR_INVALID
    rc = call("exf_reroute_subset", fake, 0, fake, 0, 4, 8, 128, fake, 0, fake, fake, fake, fake,
              None)
    assert rc == L.EXF_ERR_INVALID and "subset_size" in last_error()
    rc = call("exf_moe_align", fake, 0, 300000, 128, 64, 10, fake, fake, fake, None, 0, None)
    assert rc == L.EXF_ERR_INVALID and "capacity" in last_error()
    cap = L.lib().exf_moe_align_capacity(300000, 128, 64, 0)
    rc = call("exf_moe_align", fake, 0, 300000, 128, 64, cap, fake, fake, fake, None, 0, None)
    assert rc == L.EXF_ERR_INVALID and "workspace" in last_error()
    rc = call("exf_moe_align", fake, 0, 100, 2048, 64, 10 ** 6, fake, fake, fake, None, 0, None)
    assert rc == L.EXF_ERR_UNSUPPORTED
    # offsets are int32: a padded total or a capacity of 2^31 or more is refused by both entry
    # points (numel + experts * (block_size - 1) >= 2^31 here)
    for name, extra in (("exf_moe_align", (None, 0)), ("exf_moe_align_noalloc", ())):
        cap = L.lib().exf_moe_align_capacity(1000, 512, 1 << 22, 0)
        assert cap >= 1 << 31
        rc = call(name, fake, 0, 1000, 512, 1 << 22, cap, fake, fake, fake, *extra, None)
        assert rc == L.EXF_ERR_INVALID and "2^31" in last_error(), name
        rc = call(name, fake, 0, 1000, 128, 64, 1 << 31, fake, fake, fake, *extra, None)
        assert rc == L.EXF_ERR_INVALID and "2^31" in last_error(), name
    # decode fused with the expert layer: experts, routes and the workspace are bounded
    dfe = lambda batch, k, e, ws: call(  # noqa: E731
        "exf_decode_fused_experts", fake, fake, fake, batch, k, e, 8, 0, fake, fake, fake, fake,
        fake, 256, 128, fake, fake, fake, fake, ws, None, None)
    assert dfe(4, 8, 512, 1 << 30) == L.EXF_ERR_UNSUPPORTED and "256" in last_error()
    assert dfe(2048, 8, 128, 1 << 30) == L.EXF_ERR_UNSUPPORTED and "8192" in last_error()
    assert dfe(4, 8, 128, 16) == L.EXF_ERR_INVALID and "workspace" in last_error()
    assert dfe(0, 8, 128, 0) == 0
    # the expert layer sums at most 8 routes per token
    rc = call("exf_fused_experts", fake, fake, fake, 4, 9, fake, fake, 16, 256, 128, fake, fake,
              1 << 30, None, None)
    assert rc == L.EXF_ERR_UNSUPPORTED and "top_k" in last_error()


def test_empty_inputs_are_no_ops_without_gpu():
    # zero tokens returns before any CUDA call
    assert call("exf_router_topk", None, 0, 0, 128, 8, 0, None, 1, 1.0, None, None, None) == 0
    assert call("exf_router_topk", None, L.EXF_BF16, 0, 128, 8, 0, None, 1, 1.0, None, None,
                None) == 0
    assert call("exf_fold_prefill", None, 0, None, 0, 0, 8, 4, 128, 0, 0, None, None, None, None,
                None, None) == 0


def test_python_errors_follow_the_reference():
    import torch

    from exfold_b200.qwen3.kernels import project_prefill_topk, select_and_reroute_decode

    w = torch.rand(4, 8)
    ids = torch.randint(0, 16, (4, 8))
    c = torch.rand(16, 16)
    with pytest.raises(ValueError):
        project_prefill_topk(w, ids[:, :3], c, 4, c)
    with pytest.raises(RuntimeError):
        project_prefill_topk(w, ids, c, 4, c)  # CPU tensors
    with pytest.raises(ValueError):
        select_and_reroute_decode(w, ids, torch.rand(16, 2), c, c, 4)
