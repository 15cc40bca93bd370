"""GPU parity: moe_align / permute (single-CTA and chunked paths) against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from exfold_b200 import ops
from exfold_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def host(t):
    torch.cuda.synchronize(DEV)
    return t.cpu().numpy()


def check(ids: np.ndarray, experts: int, block: int, pad_sorted: bool = False):
    for dtype in (torch.int32, torch.int64):
        s, e, n = ops.moe_align_block_size(torch.from_numpy(ids).to(dtype).to(DEV), block, experts,
                                           pad_sorted_ids=pad_sorted)
        es, ee, en = O.moe_align(ids, experts, block, pad_sorted)
        np.testing.assert_array_equal(host(n), en)
        np.testing.assert_array_equal(host(s), es)
        np.testing.assert_array_equal(host(e), ee)


def test_documented_example():
    check(np.array([[2, 3, 4], [1, 2, 4], [1, 3, 4], [1, 2, 3]], np.int32), 5, 4)


@pytest.mark.parametrize("experts,block", [(128, 16), (128, 64), (256, 64), (256, 128), (512, 64)])
def test_random_routes_small_and_chunked(experts, block):
    rng = np.random.default_rng(experts + block)
    for tokens, k in ((1, 8), (37, 8), (256, 8), (1024, 8), (65536, 3), (4097, 5)):
        ids = np.stack([rng.choice(experts, k, replace=False) for _ in range(min(tokens, 64))])
        ids = np.resize(ids, (tokens, k)).astype(np.int32)
        ids = ids[rng.permutation(tokens)]
        check(ids, experts, block, pad_sorted=bool(tokens % 2))


def test_after_fold_config2_routes_and_skew():
    lay = W.layer("dsv4_prefill")
    w, ids = O.router_topk(lay.logits, 8, "sigmoid", lay.bias)
    check(ids[:, :3].copy(), 256, 64)
    skew = np.zeros((20000, 8), np.int32)  # every route to expert 0
    check(skew, 256, 64)
    bad = np.full((100, 8), 300, np.int32)  # out-of-range ids are not placed
    bad[:, 0] = 7
    check(bad, 256, 16)
    check(np.zeros((0, 8), np.int32), 256, 16)


def _vllm_moe_align():
    try:
        from vllm.model_executor.layers.fused_moe.moe_align_block_size import (
            moe_align_block_size)
    except Exception as exc:  # noqa: BLE001 - the library is optional at run time
        pytest.skip(f"vLLM's moe_align_block_size is not importable: {exc}")
    return moe_align_block_size


def segments(sorted_ids: np.ndarray, expert_ids: np.ndarray, post: int, block: int, numel: int):
    """expert -> sorted route indices of its padded segment; checks that padding is >= numel."""
    out: dict[int, list[int]] = {}
    for b in range(post // block):
        e = int(expert_ids[b])
        chunk = sorted_ids[b * block:(b + 1) * block]
        out.setdefault(e, []).extend(int(r) for r in chunk if r < numel)
    return {e: sorted(v) for e, v in out.items()}


@pytest.mark.parametrize("case", ["config2_after_fold", "qwen3_decode", "skew"])
def test_equal_to_vllm_moe_align_block_size(case):
    """Against vLLM's own moe_align_block_size (the op the expert layer replaces): the same
    padded total, the same expert for every used block, and the same routes in every expert's
    segment (vLLM does not fix their order within a segment; this library keeps flat order)."""
    vllm_align = _vllm_moe_align()
    if case == "config2_after_fold":
        lay = W.layer("dsv4_prefill")
        _, ids = O.router_topk(lay.logits, 8, "sigmoid", lay.bias)
        ids, experts, block = ids[:, :3].copy(), 256, 64
    elif case == "qwen3_decode":
        lay = W.layer("qwen3_decode")
        _, ids = O.router_topk(lay.logits, 8, "softmax")
        experts, block = 128, 16
    else:
        rng = np.random.default_rng(5)
        ids = np.where(rng.random((30000, 4)) < 0.7, 3, rng.integers(0, 64, (30000, 4)))
        ids, experts, block = ids.astype(np.int32), 64, 128
    t = torch.from_numpy(np.ascontiguousarray(ids)).to(DEV)
    vs, ve, vn = vllm_align(t, block, experts)
    s, e, n = ops.moe_align_block_size(t, block, experts)
    numel = ids.size
    post = int(host(n)[0])
    assert post == int(host(vn)[0])
    np.testing.assert_array_equal(host(e)[:post // block], host(ve)[:post // block])
    mine = segments(host(s), host(e), post, block, numel)
    theirs = segments(host(vs), host(ve), post, block, numel)
    assert mine == theirs
    assert sum(len(v) for v in mine.values()) == numel
    # this library's padding slots hold numel exactly
    got = host(s)[:post]
    assert np.all((got < numel) | (got == numel))
