"""GPU parity of the 256-expert biased-sigmoid router (router_biased_kernel: top-8, with or without
the DeepSeek-V4 prefill fold) on the rows and tables that reach its rare paths: non-finite and
saturating logits, constant rows, large biases (the relative part of the approximate-score
bound), selection-loss tables whose 16-bit keys tie or sit at FLT_MAX, +inf and NaN losses,
ragged tiles and multi-layer launches.  Ids and weights bit-exact against the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from exfold_b200 import ops
from exfold_b200 import workloads as W
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("router_kernel_choice")]
DEV = torch.device("cuda:0")
E = 256


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def host(t):
    torch.cuda.synchronize(DEV)
    return t.cpu().numpy()


def tables(seed):
    lay = W.layer("dsv4_prefill", tokens=16)
    coeff, loss = lay.coeff.copy(), lay.loss.copy()
    rng = np.random.default_rng(seed)
    np.fill_diagonal(coeff, 1.0)
    np.fill_diagonal(loss, 1e30)
    conf = np.clip(loss.copy() * rng.uniform(0.5, 1.5, loss.shape), 0, 1.2).astype(np.float32)
    np.fill_diagonal(conf, 0.0)
    return coeff, loss, conf


def edge_logits(seed, tokens=1200):
    x = W.logits(seed, tokens, E)
    x[10, 7] = np.nan
    x[11] = np.nan
    x[12, 100] = np.inf
    x[13, 3] = -np.inf
    x[14, ::3] = np.inf
    x[15] = 1e30
    x[16, :128] = -1e30
    x[17] = 0.0
    x[18, ::2] = -0.0
    x[19] = 3.0
    x[20:400] = np.round(x[20:400] * 4) / 4
    x[400:500] *= 40.0
    return x


def check_router(x, bias, k=8, renorm=True, scaling=1.0):
    w, ids = ops.router_topk(cuda(x), k, "sigmoid", None if bias is None else cuda(bias),
                             renormalize=renorm, scaling=scaling)
    ew, ei = O.router_topk(x, k, "sigmoid", bias, renorm, scaling)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)


def check_fold(x, bias, keep, mode, coeff, loss, conf):
    w, ids = ops.router_fold_prefill(cuda(x), 8, keep, cuda(coeff), cuda(loss), scoring="sigmoid",
                                     bias=None if bias is None else cuda(bias), variant="dsv4",
                                     renorm_mode=mode, conf_loss=cuda(conf))
    ew, ei = O.router_fold(x, 8, keep, coeff, loss, scoring="sigmoid", bias=bias, variant="dsv4",
                           conf_loss=conf, renorm_mode=mode)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)


def test_edge_rows_and_biases():
    x = edge_logits(303)
    bias = W.router_bias(303, E)
    big = (bias * 300.0).astype(np.float32)       # scores dominated by the bias, |score| ~ 100
    huge = (bias * 3.0e5).astype(np.float32)      # relative error term dominates the bound
    for b in (bias, None, big, huge):
        check_router(x, b)
    check_router(x, bias, renorm=False, scaling=2.5)
    coeff, loss, conf = tables(303)
    for b in (bias, big):
        for mode in (0, 1, 2):
            check_fold(x, b, 3, mode, coeff, loss, conf)


@pytest.mark.parametrize("keep", [1, 2, 4, 5, 6, 7, 8])
def test_fold_keep_sizes(keep):
    x = edge_logits(404, tokens=700)
    bias = W.router_bias(404, E)
    coeff, loss, conf = tables(404)
    for mode in (0, 1, 2):
        check_fold(x, bias, keep, mode, coeff, loss, conf)


def test_loss_tables_with_16_bit_ties_and_specials():
    """Losses rounded to 5 significant bits (most argmins tie in the high 16 bits of the key),
    and FLT_MAX, just below FLT_MAX, +inf, NaN, -0 and negative entries."""
    x = W.logits(505, 3000, E)
    bias = W.router_bias(505, E)
    coeff, loss, conf = tables(505)
    m, e = np.frexp(loss)
    tied = np.ldexp(np.round(m * 32) / 32, e).astype(np.float32)
    rng = np.random.default_rng(505)
    special = tied.copy()
    for value in (np.finfo(np.float32).max, np.float32(3.0e38), np.inf, np.nan, -0.0, -0.25):
        sel = rng.random(special.shape) < 0.04
        special[sel] = value
    np.fill_diagonal(special, 1e30)
    for table in (tied, special):
        for mode in (0, 1, 2):
            check_fold(x, bias, 3, mode, coeff, table, conf)
    # rows whose every loss is unselectable: the transfer goes to the first retained expert
    allbad = np.full_like(loss, np.inf)
    allbad[::2] = np.finfo(np.float32).max
    check_fold(x, bias, 3, 2, coeff, allbad, conf)


@pytest.mark.parametrize("tokens", [0, 1, 15, 16, 17, 33, 1031])
def test_ragged_tiles(tokens):
    x = W.logits(606, max(tokens, 1), E)[:tokens]
    bias = W.router_bias(606, E)
    coeff, loss, conf = tables(606)
    w, ids = ops.router_topk(cuda(x), 8, "sigmoid", cuda(bias))
    assert w.shape == (tokens, 8)
    wf, idf = ops.router_fold_prefill(cuda(x), 8, 3, cuda(coeff), cuda(loss), scoring="sigmoid",
                                      bias=cuda(bias), variant="dsv4", renorm_mode=2,
                                      conf_loss=cuda(conf))
    assert wf.shape == (tokens, 3)
    if tokens:
        check_router(x, bias)
        check_fold(x, bias, 3, 2, coeff, loss, conf)


def test_layers_batched_equal_per_layer():
    """One launch over 3 layers (own logits, bias and tables each, 1031 tokens: a short last tile
    per layer) equals the oracle layer by layer, for the router alone and with the fold."""
    xs = np.stack([W.logits(700 + i, 1031, E) for i in range(3)])
    bs = np.stack([W.router_bias(700 + i, E) for i in range(3)])
    tabs = [tables(700 + i) for i in range(3)]
    coeff = np.stack([t[0] for t in tabs])
    loss = np.stack([t[1] for t in tabs])
    conf = np.stack([t[2] for t in tabs])
    w, ids = ops.router_fold_prefill(cuda(xs), 8, 3, cuda(coeff), cuda(loss), scoring="sigmoid",
                                     bias=cuda(bs), variant="dsv4", renorm_mode=2,
                                     conf_loss=cuda(conf))
    for i in range(3):
        ew, ei = O.router_fold(xs[i], 8, 3, coeff[i], loss[i], scoring="sigmoid", bias=bs[i],
                               variant="dsv4", conf_loss=conf[i], renorm_mode=2)
        np.testing.assert_array_equal(host(ids[i]), ei)
        np.testing.assert_array_equal(host(w[i]), ew)
