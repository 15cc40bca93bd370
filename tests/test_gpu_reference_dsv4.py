"""GPU parity against the reference's own DeepSeek-V4 CUDA kernels on the same B200.

The reference's exfold/deepseek_v4/csrc/exfold_kernels.cu (prefill_kernel :17-118 with renorm
modes 0/1/2, fused_importance_select_and_apply_kernel :120-201), compiled from its source with
its own flags (-O3 --use_fast_math) by oracle/build_ref.py, is the checker here: the drop-in
torch.ops.dsv4_exfold.prefill / decode of this package run on identical seeded inputs of the
DeepSeek-style workloads (65536-token prefill fold at P=3, E=256; the decode sweep B in
{8, 32, 128, 512} x D in {64, 128}).  Ids must be identical; weights agree within 1e-5
relative in fp32 (the reference's fast-math build contracts its multiply-adds and approximates
sqrt and division; this package rounds every operation), within one bf16/fp16 unit for
half-precision weights.

The reference kernels index their 256-entry tables with the route ids unchecked, so every input
here holds ids in [0, 256) only.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from exfold_b200 import ops
from exfold_b200 import workloads as W
from oracle import build_ref

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("router_kernel_choice")]
DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def ref():
    mod = build_ref.load()
    if mod is None:
        pytest.skip("reference module oracle/_ref/exfold_ref_dsv4.so was not built "
                    "(python oracle/build_ref.py with the reference checkout present)")
    return mod


@pytest.fixture(scope="module")
def drop_in():
    from exfold_b200.deepseek_v4 import cuda_ops

    return cuda_ops


def tables(lay):
    """Served tables: coefficient diagonal 1, selection loss diagonal 1e30, confidence loss =
    the selection loss with a zero diagonal (the loader's fallback, exfold/deepseek_v4/
    vllm_patch.py:92-95, 160)."""
    coeff, loss = lay.coeff.copy(), lay.loss.copy()
    np.fill_diagonal(coeff, 1.0)
    np.fill_diagonal(loss, 1e30)
    conf = loss.copy()
    np.fill_diagonal(conf, 0.0)
    return (torch.from_numpy(a).to(DEV) for a in (coeff, loss, conf))


def routes(lay):
    w, ids = ops.router_topk(torch.from_numpy(lay.logits).to(DEV), 8, "sigmoid",
                             torch.from_numpy(lay.bias).to(DEV))
    return w, ids


def assert_weights(got, exp, dtype):
    g, e = got.float().cpu().numpy(), exp.float().cpu().numpy()
    if dtype == torch.float32:
        np.testing.assert_allclose(g, e, rtol=1e-5, atol=1e-7)
    else:
        ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
        np.testing.assert_allclose(g, e, rtol=ulp, atol=1e-6)


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_prefill_config2_all_modes(ref, drop_in, mode):
    lay = W.layer("dsv4_prefill")  # 65536 tokens, E=256, top-8
    c, l_, cf = tables(lay)
    w, ids = routes(lay)
    ew, ei = ref.prefill(w, ids, c, l_, cf, 3, mode)
    gw, gi = drop_in.fold_prefill(w, ids, c, l_, cf, 3, mode)
    torch.cuda.synchronize(DEV)
    assert torch.equal(gi, ei), f"mode {mode}: ids differ in {(gi != ei).any(1).sum()} tokens"
    assert_weights(gw, ew, torch.float32)


@pytest.mark.parametrize("target_k", [1, 2, 4, 7, 8])
@pytest.mark.parametrize("wdtype,idtype", [(torch.float32, torch.int64),
                                           (torch.bfloat16, torch.int32),
                                           (torch.float16, torch.int64)])
def test_prefill_budgets_and_dtypes(ref, drop_in, target_k, wdtype, idtype):
    lay = W.layer("dsv4_prefill", tokens=8192)
    c, l_, cf = tables(lay)
    w, ids = routes(lay)
    w, ids = w.to(wdtype), ids.to(idtype)
    for mode in (0, 1, 2):
        ew, ei = ref.prefill(w, ids, c, l_, cf, target_k, mode)
        gw, gi = drop_in.fold_prefill(w, ids, c, l_, cf, target_k, mode)
        torch.cuda.synchronize(DEV)
        assert gw.dtype == ew.dtype and gi.dtype == ei.dtype
        assert torch.equal(gi, ei), f"mode {mode}, P={target_k}: ids differ"
        assert_weights(gw, ew, wdtype)


def test_prefill_ties_and_unsorted_routes(ref, drop_in):
    """Equal weights (the reference's insertion sort is stable) and routes given out of weight
    order; quantised tables so that loss ties occur."""
    rng = np.random.default_rng(7)
    tokens = 4096
    ids = np.stack([rng.permutation(256)[:8] for _ in range(tokens)]).astype(np.int32)
    w = rng.choice(np.float32([0.05, 0.1, 0.125, 0.2]), (tokens, 8)).astype(np.float32)
    lay = W.layer("dsv4_prefill", tokens=16)
    coeff = np.round(lay.coeff * 8) / 8
    loss = np.round(lay.loss * 16) / 16
    np.fill_diagonal(coeff, 1.0)
    np.fill_diagonal(loss, 1e30)
    conf = loss.copy()
    np.fill_diagonal(conf, 0.0)
    c, l_, cf = (torch.from_numpy(a.astype(np.float32)).to(DEV) for a in (coeff, loss, conf))
    tw, ti = torch.from_numpy(w).to(DEV), torch.from_numpy(ids).to(DEV)
    for mode in (0, 1, 2):
        ew, ei = ref.prefill(tw, ti, c, l_, cf, 3, mode)
        gw, gi = drop_in.fold_prefill(tw, ti, c, l_, cf, 3, mode)
        torch.cuda.synchronize(DEV)
        assert torch.equal(gi, ei), f"mode {mode}: ids differ"
        assert_weights(gw, ew, torch.float32)


@pytest.mark.parametrize("batch", [8, 32, 128, 512])
@pytest.mark.parametrize("budget", [64, 128])
def test_decode_config3_sweep(ref, drop_in, batch, budget):
    cfg = W.WORKLOADS["dsv4_decode"]
    lay = W.Layer(seed=cfg["seed"], tokens=batch, experts=256, top_k=8, kind="dsv4")
    c, l_, _ = tables(lay)
    n = torch.from_numpy(lay.norms).to(DEV)
    w, ids = routes(lay)
    for wdtype, idtype in ((torch.float32, torch.int32), (torch.float32, torch.int64),
                           (torch.bfloat16, torch.int64)):
        tw, ti = w.to(wdtype), ids.to(idtype)
        ew, ei = ref.decode(tw, ti, c, l_, n, budget)
        gw, gi = drop_in.fold_decode(tw, ti, c, l_, n, budget)
        torch.cuda.synchronize(DEV)
        assert torch.equal(gi, ei), f"B={batch} D={budget} {wdtype}/{idtype}: ids differ"
        assert_weights(gw, ew, wdtype)


def test_decode_budget_edges(ref, drop_in):
    lay = W.Layer(seed=77, tokens=256, experts=256, top_k=8, kind="dsv4")
    c, l_, _ = tables(lay)
    n = torch.from_numpy(lay.norms).to(DEV)
    w, ids = routes(lay)
    for budget in (1, 2, 255, 256):
        ew, ei = ref.decode(w, ids, c, l_, n, budget)
        gw, gi = drop_in.fold_decode(w, ids, c, l_, n, budget)
        torch.cuda.synchronize(DEV)
        assert torch.equal(gi, ei), f"D={budget}: ids differ"
        assert_weights(gw, ew, torch.float32)
