"""GPU parity of the Qwen3 routing function (`exfold_b200.qwen3.router.make_router`) with the
reference's composition (exfold/qwen3/vllm_patch.py:159-217): vLLM's softmax top-k, then
project_prefill_topk at prefill, select_and_reroute_decode or the static remap at decode.  The
oracle restates each step; ids and weights must match bit for bit."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from exfold_b200 import calibration
from exfold_b200 import workloads as W
from exfold_b200.qwen3.router import make_router
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def layer(seed, tokens):
    lay = W.Layer(seed=seed, tokens=tokens, experts=128, top_k=8, kind="qwen3")
    c, l_, n = calibration.prepare_qwen3(lay.coeff[None], lay.loss[None], lay.norms[None],
                                         validate=False)
    return lay.logits, c[0], l_[0], n[0]


def call(router, logits, topk=8, renormalize=True):
    w, ids = router(None, torch.from_numpy(logits).to(DEV), topk, renormalize)
    torch.cuda.synchronize()
    assert w.dtype == torch.float32 and ids.dtype == torch.int32
    return w.cpu().numpy(), ids.cpu().numpy()


@pytest.mark.parametrize("renormalize", [True, False])
def test_prefill_is_router_then_fold(renormalize):
    x, c, l_, n = layer(41, 3000)
    r = make_router(torch.from_numpy(c), torch.from_numpy(l_), torch.from_numpy(n), 4, 64,
                    phase_fn=lambda t: "prefill")
    w, ids = call(r, x, renormalize=renormalize)
    ew, ei = O.router_topk(x, 8, "softmax", None, renormalize, 1.0)
    fw, fi = O.fold_qwen3(ew, ei, c, l_, 4)

    def same_weights(a, b):
        if renormalize:
            np.testing.assert_array_equal(a, b)
        else:  # softmax over all experts: the GPU sums the 128 terms in another order
            np.testing.assert_allclose(a, b, rtol=2e-6, atol=0)

    np.testing.assert_array_equal(ids, fi)
    same_weights(w, fw)
    # a budget of at least top-k leaves the router's routes
    r8 = make_router(torch.from_numpy(c), torch.from_numpy(l_), torch.from_numpy(n), 8, 64,
                     phase_fn=lambda t: "prefill")
    w8, i8 = call(r8, x, renormalize=renormalize)
    np.testing.assert_array_equal(i8, ei)
    same_weights(w8, ew)


@pytest.mark.parametrize("policy", ["dynamic", "static_norm"])
def test_decode_policies(monkeypatch, policy):
    monkeypatch.setenv("EXFOLD_QWEN3_DECODE_POLICY", policy)
    x, c, l_, n = layer(42, 256)
    r = make_router(torch.from_numpy(c), torch.from_numpy(l_), torch.from_numpy(n), 4, 64,
                    phase_fn=lambda t: "decode")
    w, ids = call(r, x)
    ew, ei = O.router_topk(x, 8, "softmax", None, True, 1.0)
    if policy == "dynamic":
        dw, di, _ = O.decode_qwen3(ew, ei, n, c, l_, 64)
    else:
        target, scale = O.static_table(n, c, l_, 64)
        dw, di = O.static_remap(ew, ei, target, scale)
    np.testing.assert_array_equal(ids, di)
    np.testing.assert_array_equal(w, dw)
    w2, ids2 = call(r, x)  # the per-device tables are cached: same result again
    np.testing.assert_array_equal(ids2, di)
    # a budget of all experts leaves the router's routes
    rall = make_router(torch.from_numpy(c), torch.from_numpy(l_), torch.from_numpy(n), 4, 128,
                       phase_fn=lambda t: "decode")
    wa, ia = call(rall, x)
    np.testing.assert_array_equal(ia, ei)
    np.testing.assert_array_equal(wa, ew)
