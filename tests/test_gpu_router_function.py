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

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("router_kernel_choice")]
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


# ---- DeepSeek-V4 (exfold/deepseek_v4/vllm_patch.py:213-368) ----------------------------------
def dsv4_setup(seed, tokens, hash_table=False):
    import types

    lay = W.Layer(seed=seed, tokens=tokens, experts=256, top_k=8, kind="dsv4")
    coeff, loss = lay.coeff.copy(), lay.loss.copy()
    np.fill_diagonal(coeff, 1.0)
    np.fill_diagonal(loss, 1e30)
    conf = loss.copy()
    np.fill_diagonal(conf, 0.0)
    calib = tuple(torch.from_numpy(a[None].copy())
                  for a in (coeff, loss, conf, coeff, loss, lay.norms))
    rng = np.random.default_rng(seed)
    table = np.stack([rng.permutation(256)[:8] for _ in range(1000)]).astype(np.int32)
    gate = types.SimpleNamespace(e_score_correction_bias=torch.from_numpy(lay.bias).to(DEV),
                                 tid2eid=torch.from_numpy(table).to(DEV) if hash_table else None)
    module = types.SimpleNamespace(n_activated_experts=8, n_routed_experts=256,
                                   scoring_func="sigmoid", renormalize=True,
                                   routed_scaling_factor=2.5, gate=gate)
    token_ids = rng.integers(0, 1000, tokens)
    return lay, module, calib, (coeff, loss, conf), table, token_ids


def test_dsv4_prefill_decode_and_mixed(monkeypatch):
    from exfold_b200.deepseek_v4.router import make_router as make_dsv4

    monkeypatch.setenv("EXFOLD_PREFILL_TOPK", "3")
    monkeypatch.setenv("EXFOLD_PREFILL_RENORM", "similarity_blend")
    monkeypatch.setenv("EXFOLD_DECODE_EXPERT_BUDGET", "64")
    lay, module, calib, (coeff, loss, conf), _, _ = dsv4_setup(51, 128)
    x = lay.logits
    rw, ri = O.router_topk(x, 8, "sigmoid", lay.bias, True, 2.5)
    pw, pi = O.fold_dsv4(rw, ri, coeff, loss, conf, 3, 2)
    for counts, (ew, ei) in (((0, 128), (pw, pi)),
                             ((128, 0), O.decode_dsv4(rw, ri, lay.norms, coeff, loss, 64))):
        r = make_dsv4(module, 0, calib, counts_fn=lambda t, c=counts: c)
        w, ids = call(r, x)
        np.testing.assert_array_equal(ids, ei)
        np.testing.assert_array_equal(w, ew)
    # mixed: 40 decode tokens first, 88 prefill tokens after, prefill padded to 8 slots
    r = make_dsv4(module, 0, calib, counts_fn=lambda t: (40, t - 40))
    w, ids = call(r, x)
    dw, di = O.decode_dsv4(rw[:40], ri[:40], lay.norms, coeff, loss, 64)
    np.testing.assert_array_equal(ids[:40], di)
    np.testing.assert_array_equal(w[:40], dw)
    np.testing.assert_array_equal(ids[40:, :3], pi[40:])
    np.testing.assert_array_equal(w[40:, :3], pw[40:])
    np.testing.assert_array_equal(ids[40:, 3:], np.repeat(pi[40:, 2:3], 5, axis=1))
    assert not w[40:, 3:].any()
    # a decode batch whose routes fit in the budget keeps them
    r = make_dsv4(module, 0, calib, counts_fn=lambda t: (t, 0))
    w, ids = call(r, x[:8])
    np.testing.assert_array_equal(ids, ri[:8])
    np.testing.assert_array_equal(w, rw[:8])


def test_dsv4_hash_layer_prefill(monkeypatch):
    from exfold_b200.deepseek_v4.router import make_router as make_dsv4

    monkeypatch.setenv("EXFOLD_PREFILL_TOPK", "3")
    monkeypatch.setenv("EXFOLD_PREFILL_RENORM", "router_l2")
    lay, module, calib, (coeff, loss, conf), table, token_ids = dsv4_setup(52, 300, True)
    r = make_dsv4(module, 0, calib, counts_fn=lambda t: (0, t))
    w, ids = r(None, torch.from_numpy(lay.logits).to(DEV), 8, True,
               input_ids=torch.from_numpy(token_ids).to(DEV))
    torch.cuda.synchronize()
    hw, hi = O.router_hash(lay.logits, token_ids, table, "sigmoid", True, 2.5)
    ew, ei = O.fold_dsv4(hw, hi, coeff, loss, conf, 3, 1)
    np.testing.assert_array_equal(ids.cpu().numpy(), ei)
    np.testing.assert_array_equal(w.cpu().numpy(), ew)
    with pytest.raises(RuntimeError, match="input_ids"):
        r(None, torch.from_numpy(lay.logits).to(DEV), 8, True)
