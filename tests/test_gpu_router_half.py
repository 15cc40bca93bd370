"""GPU parity of the routers on 16-bit (bf16 / fp16) logits.

vLLM hands the routing function the gate output in the model dtype (exfold/qwen3/vllm_patch.py:
98-109 -> fused_topk; exfold/deepseek_v4/vllm_patch.py:175-209 -> fused_topk_bias), bf16 for the
Qwen3 and DeepSeek models.  The kernels read 16-bit logits natively and convert each exactly to
fp32, so every result must equal the oracle's on logits.float() bit for bit: ids and fp32
weights.  Covered: every router kernel (the 128-expert softmax tile kernel, the 256-expert
biased-sigmoid tile kernel, the generic kernel for the other shapes and scorings, hash routing),
with and without the fold, ragged tiles, many ties (16-bit values repeat), non-finite logits,
layer-batched launches and one full-size layer of each tile kernel.
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
HALF = [torch.bfloat16, torch.float16]


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def host(t):
    torch.cuda.synchronize(DEV)
    return t.cpu().numpy()


def half_logits(lay, dtype):
    """The layer's logits rounded to `dtype` on the device, and the same values as fp32."""
    x = cuda(lay.logits).to(dtype)
    return x, host(x.float())


def dsv4_tables(lay):
    coeff, loss = lay.coeff.copy(), lay.loss.copy()
    np.fill_diagonal(coeff, 1.0)
    np.fill_diagonal(loss, 1e30)
    conf = loss.copy()
    np.fill_diagonal(conf, 0.0)
    return coeff, loss, conf


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize("experts", [64, 128, 256, 512])
@pytest.mark.parametrize("scoring", ["softmax", "sigmoid", "sqrtsoftplus"])
def test_router_topk(dtype, experts, scoring):
    lay = W.Layer(seed=300 + experts, tokens=1031, experts=experts, top_k=8,
                  kind="qwen3" if scoring == "softmax" else "dsv4")
    x, xf = half_logits(lay, dtype)
    bias = None if scoring == "softmax" else lay.bias
    w, ids = ops.router_topk(x, 8, scoring, None if bias is None else cuda(bias))
    ew, ei = O.router_topk(xf, 8, scoring, bias)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize("tokens", [1, 31, 33, 1031, 4096])
def test_router_fold_qwen3_tile_kernel(dtype, tokens):
    """E=128 softmax top-8 with the Qwen3 fold: the one-token-per-lane tile kernel."""
    lay = W.layer("qwen3_prefill", tokens=tokens)
    x, xf = half_logits(lay, dtype)
    for keep in (1, 4, 7):
        w, ids = ops.router_fold_prefill(x, 8, keep, cuda(lay.coeff), cuda(lay.loss))
        ew, ei = O.router_fold(xf, 8, keep, lay.coeff, lay.loss)
        np.testing.assert_array_equal(host(ids), ei)
        np.testing.assert_array_equal(host(w), ew)


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_router_fold_dsv4_tile_kernel(dtype, mode):
    """E=256 biased sigmoid top-8 with the DeepSeek-V4 fold: the 256-expert tile kernel."""
    lay = W.layer("dsv4_prefill", tokens=1031)
    x, xf = half_logits(lay, dtype)
    coeff, loss, conf = dsv4_tables(lay)
    w, ids = ops.router_fold_prefill(x, 8, 3, cuda(coeff), cuda(loss), scoring="sigmoid",
                                     bias=cuda(lay.bias), variant="dsv4", renorm_mode=mode,
                                     conf_loss=cuda(conf))
    ew, ei = O.router_fold(xf, 8, 3, coeff, loss, scoring="sigmoid", bias=lay.bias,
                           variant="dsv4", conf_loss=conf, renorm_mode=mode)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)


@pytest.mark.parametrize("dtype", HALF)
def test_router_fold_generic_kernel(dtype):
    """Shapes the tile kernels do not take: E=64 / 512 Qwen3 fold, sqrtsoftplus DeepSeek fold."""
    for experts in (64, 512):
        lay = W.Layer(seed=500 + experts, tokens=777, experts=experts, top_k=8, kind="qwen3")
        x, xf = half_logits(lay, dtype)
        w, ids = ops.router_fold_prefill(x, 8, 4, cuda(lay.coeff), cuda(lay.loss))
        ew, ei = O.router_fold(xf, 8, 4, lay.coeff, lay.loss)
        np.testing.assert_array_equal(host(ids), ei)
        np.testing.assert_array_equal(host(w), ew)
    lay = W.layer("dsv4_prefill", tokens=777)
    x, xf = half_logits(lay, dtype)
    coeff, loss, conf = dsv4_tables(lay)
    w, ids = ops.router_fold_prefill(x, 8, 3, cuda(coeff), cuda(loss), scoring="sqrtsoftplus",
                                     bias=cuda(lay.bias), variant="dsv4", renorm_mode=2,
                                     conf_loss=cuda(conf))
    ew, ei = O.router_fold(xf, 8, 3, coeff, loss, scoring="sqrtsoftplus", bias=lay.bias,
                           variant="dsv4", conf_loss=conf, renorm_mode=2)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)


@pytest.mark.parametrize("dtype", HALF)
def test_ties_and_non_finite_logits(dtype):
    """Coarse values (many ties at the 8th maximum), +-inf, NaN, zeros and constant rows."""
    rng = np.random.default_rng(12)
    for experts, scoring in ((128, "softmax"), (256, "sigmoid"), (64, "softmax")):
        x = np.round(rng.normal(size=(700, experts)) * 2) / 2
        x[0] = 0.0
        x[1] = 1.5
        x[2, 5] = np.inf
        x[3, :4] = -np.inf
        x[4, 7] = np.nan
        x[5, ::3] = -0.0
        xt = cuda(x.astype(np.float32)).to(dtype)
        xf = host(xt.float())
        bias = None if scoring == "softmax" else np.zeros(experts, np.float32)
        w, ids = ops.router_topk(xt, 8, scoring, None if bias is None else cuda(bias))
        ew, ei = O.router_topk(xf, 8, scoring, bias)
        np.testing.assert_array_equal(host(ids), ei)
        np.testing.assert_array_equal(host(w), ew)


@pytest.mark.parametrize("dtype", HALF)
def test_hash_routing(dtype):
    lay = W.layer("dsv4_prefill", tokens=513)
    x, xf = half_logits(lay, dtype)
    rng = np.random.default_rng(3)
    table = rng.integers(0, 256, (1000, 6), dtype=np.int32)
    tid = rng.integers(0, 1000, 513).astype(np.int64)
    w, ids = ops.router_hash(x, cuda(tid), cuda(table))
    ew, ei = O.router_hash(xf, tid, table)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)


@pytest.mark.parametrize("dtype", HALF)
def test_layers_batched_equal_per_layer(dtype):
    """Three layers of each tile kernel in one launch, tables per layer."""
    lays = [W.layer("qwen3_prefill", tokens=2000, layer_index=i) for i in range(3)]
    x = torch.stack([half_logits(lay, dtype)[0] for lay in lays])
    c = cuda(np.stack([lay.coeff for lay in lays]))
    l_ = cuda(np.stack([lay.loss for lay in lays]))
    w, ids = ops.router_fold_prefill(x, 8, 4, c, l_)
    for i in range(3):
        wi, ii = ops.router_fold_prefill(x[i], 8, 4, c[i], l_[i])
        assert torch.equal(ii, ids[i]) and torch.equal(wi, w[i])
    lays = [W.layer("dsv4_prefill", tokens=1000, layer_index=i) for i in range(3)]
    x = torch.stack([half_logits(lay, dtype)[0] for lay in lays])
    tabs = [dsv4_tables(lay) for lay in lays]
    c, l_, cf = (cuda(np.stack([t[j] for t in tabs])) for j in range(3))
    b = cuda(np.stack([lay.bias for lay in lays]))
    w, ids = ops.router_fold_prefill(x, 8, 3, c, l_, scoring="sigmoid", bias=b, variant="dsv4",
                                     renorm_mode=2, conf_loss=cf)
    for i in range(3):
        wi, ii = ops.router_fold_prefill(x[i], 8, 3, c[i], l_[i], scoring="sigmoid", bias=b[i],
                                         variant="dsv4", renorm_mode=2, conf_loss=cf[i])
        assert torch.equal(ii, ids[i]) and torch.equal(wi, w[i])


def test_full_size_layers_bf16():
    """One 131072-token Qwen3 layer (E=128, P=4) and the 65536-token DeepSeek-style layer (E=256,
    P=3, blend) on bf16 logits."""
    lay = W.layer("qwen3_layers", layer_index=3)
    x, xf = half_logits(lay, torch.bfloat16)
    w, ids = ops.router_fold_prefill(x, 8, 4, cuda(lay.coeff), cuda(lay.loss))
    ew, ei = O.router_fold(xf, 8, 4, lay.coeff, lay.loss)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)
    lay = W.layer("dsv4_prefill")
    x, xf = half_logits(lay, torch.bfloat16)
    coeff, loss, conf = dsv4_tables(lay)
    w, ids = ops.router_fold_prefill(x, 8, 3, cuda(coeff), cuda(loss), scoring="sigmoid",
                                     bias=cuda(lay.bias), variant="dsv4", renorm_mode=2,
                                     conf_loss=cuda(conf))
    ew, ei = O.router_fold(xf, 8, 3, coeff, loss, scoring="sigmoid", bias=lay.bias,
                           variant="dsv4", conf_loss=conf, renorm_mode=2)
    np.testing.assert_array_equal(host(ids), ei)
    np.testing.assert_array_equal(host(w), ew)
