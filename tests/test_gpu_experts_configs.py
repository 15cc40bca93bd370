"""GPU numerics of the expert layer at the benchmarked shapes, against a torch fp32 reference.

* DeepSeek-style prefill layer: 65536 tokens routed by the biased-sigmoid router and folded to
  top-3 (similarity blend) over 256 experts, hidden 4096, intermediate 2048 -- the layer the
  bench times (vLLM fused_experts, fused_moe.py:1587, is what it replaces).
* DeepSeek-style decode layers: B=512 tokens over 256 experts, the decode budget D in {64, 128}
  applied first (exfold_kernels.cu:120-201 semantics), hidden 4096, intermediate 2048, through
  both `fused_experts` after `decode` and the fused `decode_fused_experts`.

Tolerance as in tests/test_gpu_experts.py: 2e-2 of the output scale (bf16 operands, fp32
accumulation, the SwiGLU activation rounded to bf16 as vLLM's intermediate cache).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from exfold_b200 import ops
from exfold_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
H, I, E = 4096, 2048, 256


def reference(x, topk_w, topk_ids, w13, w2):
    tokens, hidden = x.shape
    inter = w13.shape[1] // 2
    y = torch.zeros(tokens, hidden, dtype=torch.float32, device=x.device)
    for e in torch.unique(topk_ids).tolist():
        if e < 0:
            continue
        rows, slots = torch.nonzero(topk_ids == e, as_tuple=True)
        h = x[rows].float()
        w = w13[e].float()
        a = (torch.nn.functional.silu(h @ w[:inter].T) * (h @ w[inter:].T)).to(torch.bfloat16)
        o = a.float() @ w2[e].float().T
        y.index_add_(0, rows, o * topk_w[rows, slots].unsqueeze(1).float())
    return y


@pytest.fixture(scope="module")
def weights():
    gen = torch.Generator(device=DEV)
    gen.manual_seed(404)
    w13 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16, device=DEV)
    w2 = torch.empty(E, H, I, dtype=torch.bfloat16, device=DEV)
    for e in range(E):  # N(0, 0.02), generated per expert to bound the fp32 temporaries
        w13[e] = 0.02 * torch.randn(2 * I, H, generator=gen, device=DEV)
        w2[e] = 0.02 * torch.randn(H, I, generator=gen, device=DEV)
    yield w13, w2
    del w13, w2
    torch.cuda.empty_cache()


def dsv4_tables(lay):
    coeff, loss = lay.coeff.copy(), lay.loss.copy()
    np.fill_diagonal(coeff, 1.0)
    np.fill_diagonal(loss, 1e30)
    conf = loss.copy()
    np.fill_diagonal(conf, 0.0)
    return (torch.from_numpy(a).to(DEV) for a in (coeff, loss, conf))


def check(y, ref):
    scale = ref.abs().max().item()
    assert scale > 0
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2 * scale)


def test_prefill_layer_config2(weights):
    w13, w2 = weights
    lay = W.layer("dsv4_prefill")  # 65536 tokens, top-8 of 256
    c, l_, cf = dsv4_tables(lay)
    tw, ti = ops.router_fold_prefill(
        torch.from_numpy(lay.logits).to(DEV), 8, 3, c, l_, scoring="sigmoid",
        bias=torch.from_numpy(lay.bias).to(DEV), variant="dsv4", renorm_mode=2, conf_loss=cf)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(405)
    x = torch.randn(lay.tokens, H, generator=gen, device=DEV).to(torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    y = ops.fused_experts(x, tw, ti, w13, w2, status=status)
    ref = reference(x, tw, ti, w13, w2)
    torch.cuda.synchronize(DEV)
    assert int(status.item()) == 0, "a pipeline wait timed out"
    assert int(torch.unique(ti).numel()) > 200  # the benchmarked routing: most experts active
    check(y, ref)


@pytest.mark.parametrize("budget", [64, 128])
def test_decode_layer_config3(weights, budget):
    w13, w2 = weights
    cfg = W.WORKLOADS["dsv4_decode"]
    lay = W.Layer(seed=cfg["seed"], tokens=512, experts=E, top_k=8, kind="dsv4")
    c, l_, _ = dsv4_tables(lay)
    n = torch.from_numpy(lay.norms).to(DEV)
    rw, ri = ops.router_topk(torch.from_numpy(lay.logits).to(DEV), 8, "sigmoid",
                             torch.from_numpy(lay.bias).to(DEV))
    gen = torch.Generator(device=DEV)
    gen.manual_seed(406 + budget)
    x = torch.randn(512, H, generator=gen, device=DEV).to(torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    dw, di = ops.decode(rw, ri, n, c, l_, budget, variant="dsv4")
    y = ops.fused_experts(x, dw, di, w13, w2, status=status)
    yf, fw, fi = ops.decode_fused_experts(x, rw, ri, n, c, l_, budget, w13, w2, variant="dsv4",
                                          status=status)
    ref = reference(x, dw, di, w13, w2)
    torch.cuda.synchronize(DEV)
    assert int(status.item()) == 0, "a pipeline wait timed out"
    assert int(torch.unique(di).numel()) <= budget
    assert torch.equal(fi, di) and torch.equal(fw, dw)
    check(y, ref)
    check(yf, ref)
