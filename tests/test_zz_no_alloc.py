"""GPU test of exf_moe_align_noalloc, the moe_align entry point that allocates nothing.

Some callers cannot allocate device memory when they call moe_align: an inference-engine
plugin whose execute step may not allocate, a host whose device memory all belongs to another
runtime's pool, or code that must avoid the device synchronisation of cudaMalloc/cudaFree.
exf_moe_align_noalloc serves them from a fixed scratch array inside the library.

The test calls it through the C ABI twice in a row, on inputs large enough to need the scratch
(and with different table shapes, so a stale table from the first call would show), and checks
each result against exf_moe_align given a caller-owned workspace.  It also checks that an input
beyond the scratch limit is refused with a message.  Every buffer here belongs to the test, which
plays the caller; the entry point itself allocates nothing.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from exfold_b200 import _lib as L

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def outputs(numel: int, experts: int, block: int):
    cap = int(L.lib().exf_moe_align_capacity(numel, experts, block, 0))
    sorted_ids = torch.full((cap,), -7, dtype=torch.int32, device=DEV)
    expert_ids = torch.full(((cap + block - 1) // block,), -7, dtype=torch.int32, device=DEV)
    post = torch.full((1,), -7, dtype=torch.int32, device=DEV)
    return cap, sorted_ids, expert_ids, post


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)


def id_dtype(ids: torch.Tensor) -> int:
    return L.EXF_I64 if ids.dtype == torch.int64 else L.EXF_I32


def with_workspace(ids: torch.Tensor, experts: int, block: int):
    numel = ids.numel()
    cap, s, e, n = outputs(numel, experts, block)
    ws_bytes = int(L.lib().exf_moe_align_workspace_bytes(numel, experts))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=DEV)
    L.check(L.lib().exf_moe_align(ids.data_ptr(), id_dtype(ids), numel, experts, block, cap,
                                  s.data_ptr(), e.data_ptr(), n.data_ptr(), ws.data_ptr(),
                                  ws_bytes, stream()))
    return s, e, n


def without_allocation(ids: torch.Tensor, experts: int, block: int):
    numel = ids.numel()
    cap, s, e, n = outputs(numel, experts, block)
    L.check(L.lib().exf_moe_align_noalloc(ids.data_ptr(), id_dtype(ids), numel, experts, block,
                                          cap, s.data_ptr(), e.data_ptr(), n.data_ptr(),
                                          stream()))
    return s, e, n


def check_equal(ids: torch.Tensor, experts: int, block: int):
    ref = with_workspace(ids, experts, block)
    got = without_allocation(ids, experts, block)
    torch.cuda.synchronize(DEV)
    for r, g in zip(ref, got):
        assert torch.equal(r, g)
    assert int(got[2].item()) >= ids.numel()


def test_noalloc_equals_workspace_entry_point_on_two_calls():
    torch.cuda.set_device(DEV)
    rng = np.random.default_rng(20261201)
    cases = [(65536, 3, 256, 64), (131072, 4, 128, 16)]  # 196,608 then 524,288 routes
    for tokens, k, experts, block in cases:
        ids = torch.from_numpy(rng.integers(0, experts, (tokens, k), dtype=np.int32)).to(DEV)
        assert int(L.lib().exf_moe_align_workspace_bytes(ids.numel(), experts)) > 0
        check_equal(ids, experts, block)


def test_noalloc_int64_ids_small_input_and_the_exact_limit():
    torch.cuda.set_device(DEV)
    rng = np.random.default_rng(20261202)
    # int64 ids through the scratch path
    ids = torch.from_numpy(rng.integers(0, 256, (32768, 8), dtype=np.int64)).to(DEV)
    check_equal(ids, 256, 64)
    # at most 8192 routes: one CTA, no scratch lookup
    for dt in (np.int32, np.int64):
        ids = torch.from_numpy(rng.integers(0, 128, (1024, 8)).astype(dt)).to(DEV)
        assert int(L.lib().exf_moe_align_workspace_bytes(ids.numel(), 128)) == 0
        check_equal(ids, 128, 16)
    # exactly at the limit, 2048 * floor(262144 / experts) routes, is accepted
    experts = 384
    numel = 2048 * (262144 // experts)
    ids = torch.from_numpy(rng.integers(0, experts, numel, dtype=np.int32)).to(DEV)
    check_equal(ids, experts, 32)


def test_noalloc_refuses_inputs_beyond_its_scratch():
    torch.cuda.set_device(DEV)
    experts, block = 512, 16
    numel = 2048 * (262144 // experts) + 1
    ids = torch.zeros(numel, dtype=torch.int32, device=DEV)
    cap, s, e, n = outputs(numel, experts, block)
    rc = L.lib().exf_moe_align_noalloc(ids.data_ptr(), L.EXF_I32, numel, experts, block, cap,
                                       s.data_ptr(), e.data_ptr(), n.data_ptr(), stream())
    assert rc == L.EXF_ERR_INVALID
    assert b"fixed scratch" in L.lib().exf_last_error()
