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
