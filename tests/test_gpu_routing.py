"""GPU parity: router top-k, fused router + prefill fold, prefill fold of given routes.

Every case runs the sm_100a kernels through the C ABI (exfold_b200.ops / the drop-in modules)
and compares with the CPU oracle on the same inputs: ids bit-exact, fp32 weights bit-exact
(both sides evaluate the same IEEE operation sequence) unless a test states a tolerance, and the
reference's own golden outputs (tests/golden) within the reference tests' tolerances.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from exfold_b200 import ops
from exfold_b200 import workloads as W
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("router_kernel_choice")]
GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda:0")


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def host(t):
    torch.cuda.synchronize(DEV)
    return t.cpu().numpy()


def dsv4_tables(lay):
    coeff, loss = lay.coeff.copy(), lay.loss.copy()
    np.fill_diagonal(coeff, 1.0)
    np.fill_diagonal(loss, 1e30)
    conf = loss.copy()
    np.fill_diagonal(conf, 0.0)
    return coeff, loss, conf


# ---- router ---------------------------------------------------------------------------------
@pytest.mark.parametrize("experts", [64, 128, 256, 512])
@pytest.mark.parametrize("scoring", ["softmax", "sigmoid"])
def test_router_topk_matches_oracle(experts, scoring):
    x = W.logits(31 + experts, 3000, experts)
    bias = W.router_bias(31, experts) if scoring == "sigmoid" else None
    for k in (8, 6, 1):
        w, ids = ops.router_topk(cuda(x), k, scoring, None if bias is None else cuda(bias))
        ew, ei = O.router_topk(x, k, scoring, bias)
        np.testing.assert_array_equal(host(ids), ei)
        np.testing.assert_array_equal(host(w), ew)


def test_router_softmax_golden_config0():
    wc = np.load(GOLDEN / "workload_cases.npz")
    lay = W.layer("qwen3_prefill")
    w, ids = ops.router_topk(cuda(lay.logits), 8, "softmax")
    np.testing.assert_array_equal(host(ids), wc["qp_router_ids"])
    np.testing.assert_allclose(host(w), wc["qp_router_w"], rtol=2e-6, atol=0)


def test_router_sigmoid_golden_config2_prefix():
    wc = np.load(GOLDEN / "workload_cases.npz")
    lay = W.layer("dsv4_prefill", tokens=4096)
    w, ids = ops.router_topk(cuda(lay.logits), 8, "sigmoid", cuda(lay.bias))
    np.testing.assert_array_equal(host(ids), wc["dp_router_ids"])
    np.testing.assert_allclose(host(w), wc["dp_router_w"], rtol=1e-6, atol=0)


@pytest.mark.parametrize("scoring", ["softmax", "sigmoid"])
def test_router_options(scoring):
    x = W.logits(77, 1000, 128)
    bias = W.router_bias(77, 128) if scoring == "sigmoid" else None
    for renorm, scaling in ((False, 1.0), (True, 2.5)):
        w, ids = ops.router_topk(cuda(x), 8, scoring, None if bias is None else cuda(bias),
                                 renormalize=renorm, scaling=scaling)
        ew, ei = O.router_topk(x, 8, scoring, bias, renorm, scaling)
        np.testing.assert_array_equal(host(ids), ei)
        # softmax without renormalisation sums all experts in a different order
        np.testing.assert_allclose(host(w), ew, rtol=1e-6, atol=0)


@pytest.mark.parametrize("experts", [64, 128, 256, 512])
def test_router_quantised_logits_tie_often(experts):
    """Logits on coarse grids tie inside the top-k on many tokens (a candidate equal to another
    candidate, to its own group maximum, or to the threshold); rows of mostly negative logits put
    zeros of both signs among the candidates; half-precision rows tie now and then.  Ids and
    weights stay bit-exact, also through the fused fold and over a ragged last tile."""
    x = W.logits(77 + experts, 4099, experts)
    x[1024:2048] = np.round(x[1024:2048] * 64) / 64       # ties within the top 8 on most rows
    x[2048:3072] = np.round(x[2048:3072] * 8) / 8         # ties with the threshold
    neg = -np.abs(x[3072:3584])
    neg[:, ::5] = 0.0
    neg[:, 1::7] = -0.0
    x[3072:3584] = neg
    x[3584:] = x[3584:].astype(np.float16).astype(np.float32)
    lay = W.layer("qwen3_prefill")
    coeff = np.resize(lay.coeff, (experts, experts)).astype(np.float32)
    loss = np.resize(lay.loss, (experts, experts)).astype(np.float32)
    for k in (8, 4):
        w, ids = ops.router_topk(cuda(x), k, "softmax")
        ew, ei = O.router_topk(x, k, "softmax")
        np.testing.assert_array_equal(host(ids), ei)
        np.testing.assert_array_equal(host(w), ew)
        for keep in (k // 2, 3):
            fw, fi = ops.router_fold_prefill(cuda(x), k, keep, cuda(coeff), cuda(loss))
            efw, efi = O.router_fold(x, k, keep, coeff, loss)
            np.testing.assert_array_equal(host(fi), efi)
            np.testing.assert_array_equal(host(fw), efw)


def test_router_sigmoid_e256_ties_and_options():
    """Biased-sigmoid router at 256 experts on quantised logits and biases (exact key ties,
    candidates within the approximate keys' margin of the threshold), without a bias, without
    renormalisation and with scaling; and the fused DeepSeek fold in every renorm mode on the same
    rows.  Ids and weights bit-exact."""
    E = 256
    x = W.logits(91, 4133, E)
    x[1000:2000] = np.round(x[1000:2000] * 16) / 16
    x[2000:3000] = np.round(x[2000:3000] * 2) / 2
    bias = W.router_bias(91, E)
    qbias = (np.round(bias * 8) / 8).astype(np.float32)
    lay = W.layer("dsv4_prefill", tokens=64)
    coeff, loss, conf = dsv4_tables(lay)
    for b in (bias, qbias, None):
        for renorm, scaling in ((True, 1.0), (False, 2.5)):
            w, ids = ops.router_topk(cuda(x), 8, "sigmoid", None if b is None else cuda(b),
                                     renormalize=renorm, scaling=scaling)
            ew, ei = O.router_topk(x, 8, "sigmoid", b, renorm, scaling)
            np.testing.assert_array_equal(host(ids), ei)
            np.testing.assert_array_equal(host(w), ew)
    for mode in (0, 1, 2):
        for keep in (3, 5):
            w, ids = ops.router_fold_prefill(cuda(x), 8, keep, cuda(coeff), cuda(loss),
                                             scoring="sigmoid", bias=cuda(qbias), variant="dsv4",
                                             renorm_mode=mode, conf_loss=cuda(conf))
            ew, ei = O.router_fold(x, 8, keep, coeff, loss, scoring="sigmoid", bias=qbias,
                                   variant="dsv4", conf_loss=conf, renorm_mode=mode)
            np.testing.assert_array_equal(host(ids), ei)
            np.testing.assert_array_equal(host(w), ew)


@pytest.mark.parametrize("experts", [64, 128, 256, 512])
def test_router_sqrtsoftplus_matches_oracle(experts):
    """DeepSeek-V4 sqrtsoftplus scoring (vLLM fused_topk_bias scoring_func="sqrtsoftplus"):
    exact keys sqrt(softplus(x)) + bias, with and without a bias, renormalised or not; logits
    include quantised rows, extremes and NaN."""
    x = W.logits(505 + experts, 2077, experts) * 3
    x[500:900] = np.round(x[500:900] * 4) / 4
    x[901, 3] = 95.0
    x[902, 5] = -120.0
    x[903, 7] = np.nan
    x[904] = -90.0
    bias = W.router_bias(505, experts)
    for b in (bias, None):
        for k, renorm, scaling in ((8, True, 1.0), (6, False, 2.5)):
            w, ids = ops.router_topk(cuda(x), k, "sqrtsoftplus", None if b is None else cuda(b),
                                     renormalize=renorm, scaling=scaling)
            ew, ei = O.router_topk(x, k, "sqrtsoftplus", b, renorm, scaling)
            np.testing.assert_array_equal(host(ids), ei)
            np.testing.assert_array_equal(host(w), ew)


def test_router_fold_sqrtsoftplus_dsv4_and_qwen3():
    lay = W.layer("dsv4_prefill", tokens=4101)
    coeff, loss, conf = dsv4_tables(lay)
    for mode in (0, 1, 2):
        w, ids = ops.router_fold_prefill(cuda(lay.logits), 8, 3, cuda(coeff), cuda(loss),
                                         scoring="sqrtsoftplus", bias=cuda(lay.bias),
                                         variant="dsv4", renorm_mode=mode, conf_loss=cuda(conf))
        ew, ei = O.router_fold(lay.logits, 8, 3, coeff, loss, scoring="sqrtsoftplus",
                               bias=lay.bias, variant="dsv4", conf_loss=conf, renorm_mode=mode)
        np.testing.assert_array_equal(host(ids), ei)
        np.testing.assert_array_equal(host(w), ew)
    w, ids = ops.router_fold_prefill(cuda(lay.logits), 8, 4, cuda(coeff), cuda(loss),
                                     scoring="sqrtsoftplus", bias=cuda(lay.bias))
    ew, ei = O.router_fold(lay.logits, 8, 4, coeff, loss, scoring="sqrtsoftplus", bias=lay.bias)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)


@pytest.mark.parametrize("id_dtype", [torch.int32, torch.int64])
def test_router_hash_matches_oracle(id_dtype):
    """Hash-MoE routing (tid2eid[input_ids]): table order kept, unbiased scores as weights;
    out-of-range token ids and table entries read nothing out of range."""
    rng = np.random.default_rng(6)
    x = W.logits(606, 3001, 256)
    table = np.stack([rng.choice(256, 8, replace=False) for _ in range(5000)]).astype(np.int32)
    table[7, 3] = 300
    table[8, 0] = -2
    tok = rng.integers(0, 5000, 3001).astype(np.int64)
    tok[:20] = np.arange(20)
    tok[20], tok[21] = -1, 5000
    for scoring in ("sqrtsoftplus", "sigmoid"):
        for renorm, scaling in ((True, 1.0), (False, 2.5)):
            w, ids = ops.router_hash(cuda(x), cuda(tok).to(id_dtype), cuda(table), scoring,
                                     renorm, scaling)
            ew, ei = O.router_hash(x, tok, table, scoring, renorm, scaling)
            np.testing.assert_array_equal(host(ids), ei)
            np.testing.assert_array_equal(host(w), ew)
    # the DeepSeek-V4 fold of hash routes (weights sorted inside the fold)
    w, ids = ops.router_hash(cuda(x), cuda(tok), cuda(table), "sqrtsoftplus")
    lay = W.layer("dsv4_prefill", tokens=64)
    coeff, loss, conf = dsv4_tables(lay)
    valid = (host(ids) >= 0).all(1) & (host(ids) < 256).all(1)
    fw, fi = ops.fold_prefill(w[cuda(valid)], ids[cuda(valid)], cuda(coeff), cuda(loss), 3,
                              variant="dsv4", renorm_mode=2, conf_loss=cuda(conf))
    efw, efi = O.fold_dsv4(host(w)[valid], host(ids)[valid], coeff, loss, conf, 3, 2)
    np.testing.assert_array_equal(host(fi), efi)
    np.testing.assert_array_equal(host(fw), efw)
    with pytest.raises(NotImplementedError):
        ops.router_hash(cuda(x), cuda(tok), cuda(table), "softmax")


def test_native_route_is_router_or_hash():
    from exfold_b200.deepseek_v4.routing import native_route

    x = W.logits(707, 1000, 256)
    bias = W.router_bias(707, 256)
    table = np.stack([np.roll(np.arange(256), i)[:8] for i in range(50)]).astype(np.int32)
    tok = np.arange(1000) % 50
    w, ids = native_route(cuda(x), 8, "sqrtsoftplus", cuda(bias), True, 2.0)
    ew, ei = O.router_topk(x, 8, "sqrtsoftplus", bias, True, 2.0)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)
    w, ids = native_route(cuda(x), 8, "sigmoid", cuda(bias), True, 1.0, input_ids=cuda(tok),
                          tid2eid=cuda(table))
    ew, ei = O.router_hash(x, tok, table, "sigmoid", True, 1.0)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)


def test_router_ties_constant_rows_and_specials():
    """Exact ties take the lower expert id; constant rows, +-inf and NaN stay in range."""
    x = W.logits(5, 256, 128)
    x[0] = 0.0                       # every expert ties
    x[1] = -1.0
    x[1, ::2] = 1.0                  # 64-way tie at the top
    x[2] = np.round(x[2] * 4) / 4    # heavily quantised: many ties
    x[3, 7] = np.inf
    x[4, 9] = -np.inf
    x[5, 11] = np.nan
    x[6] = -0.0
    x[6, 3] = 0.0
    for scoring in ("softmax", "sigmoid"):
        bias = np.zeros(128, np.float32) if scoring == "sigmoid" else None
        w, ids = ops.router_topk(cuda(x), 8, scoring, None if bias is None else cuda(bias))
        _, ei = O.router_topk(x, 8, scoring, bias)
        got = host(ids)
        assert got.min() >= 0 and got.max() < 128
        np.testing.assert_array_equal(got, ei)
        np.testing.assert_array_equal(got[0], np.arange(8))
        np.testing.assert_array_equal(got[1], np.arange(0, 16, 2))


# ---- fused router + fold ----------------------------------------------------------------------
def test_router_fold_qwen3_config0_full():
    wc = np.load(GOLDEN / "workload_cases.npz")
    lay = W.layer("qwen3_prefill")
    w, ids = ops.router_fold_prefill(cuda(lay.logits), 8, 4, cuda(lay.coeff), cuda(lay.loss))
    ew, ei = O.router_fold(lay.logits, 8, 4, lay.coeff, lay.loss)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)
    np.testing.assert_array_equal(host(ids), wc["qp_out_ids"])
    np.testing.assert_allclose(host(w), wc["qp_out_w"], rtol=1e-5, atol=0)


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_router_fold_dsv4_modes(mode):
    lay = W.layer("dsv4_prefill", tokens=8192)
    coeff, loss, conf = dsv4_tables(lay)
    w, ids = ops.router_fold_prefill(cuda(lay.logits), 8, 3, cuda(coeff), cuda(loss),
                                     scoring="sigmoid", bias=cuda(lay.bias), variant="dsv4",
                                     renorm_mode=mode, conf_loss=cuda(conf))
    ew, ei = O.router_fold(lay.logits, 8, 3, coeff, loss, scoring="sigmoid", bias=lay.bias,
                           variant="dsv4", conf_loss=conf, renorm_mode=mode)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)
    if mode == 2:
        wc = np.load(GOLDEN / "workload_cases.npz")
        np.testing.assert_array_equal(host(ids)[:4096], wc["dp_out_ids"])
        np.testing.assert_allclose(host(w)[:4096], wc["dp_out_w"], rtol=1e-5, atol=0)


def test_router_fold_dsv4_config2_full():
    """T=65536, E=256, P=3, similarity blend: the full DeepSeek-style prefill workload."""
    lay = W.layer("dsv4_prefill")
    coeff, loss, conf = dsv4_tables(lay)
    w, ids = ops.router_fold_prefill(cuda(lay.logits), 8, 3, cuda(coeff), cuda(loss),
                                     scoring="sigmoid", bias=cuda(lay.bias), variant="dsv4",
                                     renorm_mode=2, conf_loss=cuda(conf))
    ew, ei = O.router_fold(lay.logits, 8, 3, coeff, loss, scoring="sigmoid", bias=lay.bias,
                           variant="dsv4", conf_loss=conf, renorm_mode=2)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)


def test_router_fold_layers_batched_equals_per_layer():
    """One launch over 3 layers (own tables each) equals three single-layer launches."""
    lays = [W.layer("qwen3_layers", tokens=5000, layer_index=i) for i in range(3)]
    x = cuda(np.stack([l.logits for l in lays]))
    coeff = cuda(np.stack([l.coeff for l in lays]))
    loss = cuda(np.stack([l.loss for l in lays]))
    w, ids = ops.router_fold_prefill(x, 8, 4, coeff, loss)
    for i, lay in enumerate(lays):
        ew, ei = O.router_fold(lay.logits, 8, 4, lay.coeff, lay.loss)
        np.testing.assert_array_equal(host(ids[i]), ei)
        np.testing.assert_array_equal(host(w[i]), ew)


def test_router_fold_qwen3_layer_full_size():
    """One layer of the 48-layer workload at its full T=131072."""
    lay = W.layer("qwen3_layers", layer_index=7)
    w, ids = ops.router_fold_prefill(cuda(lay.logits), 8, 4, cuda(lay.coeff), cuda(lay.loss))
    ew, ei = O.router_fold(lay.logits, 8, 4, lay.coeff, lay.loss)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)


def test_router_fold_empty_and_ragged():
    lay = W.layer("qwen3_prefill", tokens=37)
    for t in (0, 1, 7, 37):
        w, ids = ops.router_fold_prefill(cuda(lay.logits[:t]), 8, 4, cuda(lay.coeff),
                                         cuda(lay.loss))
        assert w.shape == (t, 4)
        if t:
            ew, ei = O.router_fold(lay.logits[:t], 8, 4, lay.coeff, lay.loss)
            np.testing.assert_array_equal(host(ids), ei)
            np.testing.assert_array_equal(host(w), ew)


# ---- fold of given routes (reference API) ------------------------------------------------------
def test_project_prefill_topk_reference_fixture():
    from exfold_b200.qwen3.kernels import project_prefill_topk

    qt = np.load(GOLDEN / "qwen3_reference_tests.npz")
    ow, oi = project_prefill_topk(cuda(qt["prefill_w"]), cuda(qt["prefill_ids"]),
                                  cuda(qt["prefill_coeff"]), 4, cuda(qt["prefill_loss"]))
    np.testing.assert_array_equal(host(oi), qt["prefill_out_ids"])
    np.testing.assert_allclose(host(ow), qt["prefill_out_w"], atol=5e-5, rtol=5e-5)
    ew, _ = O.fold_qwen3(qt["prefill_w"], qt["prefill_ids"], qt["prefill_coeff"],
                         qt["prefill_loss"], 4)
    np.testing.assert_array_equal(host(ow), ew)
    # unobserved pairs are a no-op (tests/test_qwen3_kernels.py:98-116)
    w = cuda(np.full((1, 8), 0.125, np.float32))
    ids = cuda(np.arange(8, dtype=np.int32)[None])
    pw, pi = project_prefill_topk(w, ids, cuda(np.ones((8, 8), np.float32)), 4,
                                  cuda(np.full((8, 8), 1e30, np.float32)))
    np.testing.assert_array_equal(host(pw), qt["noop_prefill_w"])
    np.testing.assert_array_equal(host(pi), qt["noop_prefill_ids"])
    # passthrough when target_k >= top_k
    pw, pi = project_prefill_topk(w, ids, cuda(np.ones((8, 8), np.float32)), 9,
                                  cuda(np.ones((8, 8), np.float32)))
    assert pw.shape == (1, 8)


@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("idtype", [torch.int32, torch.int64])
def test_fold_prefill_dtypes_match_oracle(wdtype, idtype):
    lay = W.layer("qwen3_prefill", tokens=2000)
    rw, ri = O.router_topk(lay.logits, 8, "softmax")
    w_t = torch.from_numpy(rw).to(wdtype)
    w_in = w_t.float().numpy()  # what the kernel computes from
    coeff, loss, conf = dsv4_tables(lay)
    for variant, mode in (("qwen3", 0), ("dsv4", 0), ("dsv4", 1), ("dsv4", 2)):
        ow, oi = ops.fold_prefill(w_t.to(DEV), cuda(ri).to(idtype), cuda(coeff), cuda(loss), 4,
                                  variant=variant, renorm_mode=mode, conf_loss=cuda(conf))
        assert ow.dtype == wdtype and oi.dtype == idtype
        if variant == "qwen3":
            ew, ei = O.fold_qwen3(w_in, ri, coeff, loss, 4)
        else:
            ew, ei = O.fold_dsv4(w_in, ri, coeff, loss, conf, 4, mode)
        np.testing.assert_array_equal(host(oi).astype(np.int32), ei)
        exp = torch.from_numpy(ew).to(wdtype).float().numpy()
        np.testing.assert_array_equal(host(ow.float()), exp)


def test_dsv4_fold_prefill_reference_fixture():
    from exfold_b200.deepseek_v4.cuda_ops import fold_prefill

    dt = np.load(GOLDEN / "dsv4_reference_tests.npz")
    w = torch.from_numpy(dt["w_bf16_as_f32"]).to(torch.bfloat16).to(DEV)
    ow, oi = fold_prefill(w, cuda(dt["ids"]), cuda(dt["coeff"]), cuda(dt["sel"]),
                          cuda(dt["conf"]), 3, 2)
    assert ow.dtype == torch.bfloat16
    ew, ei = O.fold_dsv4(dt["w_bf16_as_f32"], dt["ids"], dt["coeff"], dt["sel"], dt["conf"], 3, 2)
    np.testing.assert_array_equal(host(oi), ei)
    np.testing.assert_array_equal(host(ow.float()),
                                  torch.from_numpy(ew).to(torch.bfloat16).float().numpy())
    # the reference test's own tolerance against its torch restatement (tie rows as sets)
    ws = -np.sort(-dt["w_bf16_as_f32"], axis=1)
    tie = np.any(ws[:, :4][:, 1:] == ws[:, :4][:, :-1], axis=1)
    np.testing.assert_array_equal(host(oi)[~tie], dt["prefill_out_ids"][~tie])
    np.testing.assert_allclose(host(ow.float())[~tie], dt["prefill_out_w"][~tie], atol=2e-2,
                               rtol=2e-2)


def test_dsv4_prefill_target_k_equal_topk_sorts():
    from exfold_b200.deepseek_v4.cuda_ops import fold_prefill

    lay = W.layer("dsv4_prefill", tokens=300)
    rw, ri = O.router_topk(lay.logits, 8, "sigmoid", lay.bias)
    coeff, loss, conf = dsv4_tables(lay)
    for mode in (0, 1, 2):
        ow, oi = fold_prefill(cuda(rw), cuda(ri), cuda(coeff), cuda(loss), cuda(conf), 8, mode)
        ew, ei = O.fold_dsv4(rw, ri, coeff, loss, conf, 8, mode)
        np.testing.assert_array_equal(host(oi), ei)
        np.testing.assert_array_equal(host(ow), ew)


def test_api_errors():
    from exfold_b200.deepseek_v4.cuda_ops import fold_prefill
    from exfold_b200.qwen3.kernels import project_prefill_topk

    w = torch.rand(4, 8, device=DEV)
    ids = torch.randint(0, 128, (4, 8), device=DEV, dtype=torch.int32)
    c = torch.rand(128, 128, device=DEV)
    with pytest.raises(ValueError):
        project_prefill_topk(w, ids[:, :4], c, 4, c)
    with pytest.raises(ValueError):
        project_prefill_topk(w, ids, c, 4, c[:64])
    with pytest.raises(RuntimeError):
        project_prefill_topk(w.cpu(), ids, c, 4, c)
    with pytest.raises(RuntimeError):
        fold_prefill(w, ids, c, c, c, 0, 2)
    with pytest.raises(RuntimeError):
        fold_prefill(w, ids, c, c, c, 3, 5)
    with pytest.raises(NotImplementedError):
        ops.router_topk(torch.rand(4, 96, device=DEV), 8)
