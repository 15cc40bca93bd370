"""GPU checks of `exf_decode_fused_experts`: the decode expert budget followed by the expert layer,
with moe_align inside the decode launch and duplicate (token, expert) routes merged.

The decode outputs must equal `decode` bit for bit; the layer output must equal `fused_experts`
over those outputs within bf16 tolerance (2e-2 of the output scale, as the expert tests), and a
plain torch fp32 reference of the routes.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from exfold_b200 import ops
from exfold_b200 import workloads as W

from test_gpu_experts import reference

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def weights(experts, hidden, inter, seed):
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    w13 = (0.02 * torch.randn(experts, 2 * inter, hidden, generator=gen, device=DEV)).to(
        torch.bfloat16)
    w2 = (0.02 * torch.randn(experts, hidden, inter, generator=gen, device=DEV)).to(torch.bfloat16)
    return gen, w13, w2


def duplicate_routes(ids):
    s = np.sort(ids, axis=1)
    return int(((s[:, 1:] == s[:, :-1]) & (s[:, 1:] >= 0)).sum())


def run(lay, budget, variant, hidden, inter, seed, edit_ids=None):
    coeff, loss = lay.coeff.copy(), lay.loss.copy()
    if variant == "dsv4":
        np.fill_diagonal(coeff, 1.0)
        np.fill_diagonal(loss, 1e30)
    scoring = "softmax" if variant == "qwen3" else "sigmoid"
    bias = None if lay.bias is None else cuda(lay.bias)
    rw, ri = ops.router_topk(cuda(lay.logits), lay.top_k, scoring, bias)
    if edit_ids is not None:
        ri = edit_ids(ri)
    gen, w13, w2 = weights(lay.experts, hidden, inter, seed)
    x = torch.randn(lay.tokens, hidden, generator=gen, device=DEV).to(torch.bfloat16)
    n, c, l_ = cuda(lay.norms), cuda(coeff), cuda(loss)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    y, ow, oi = ops.decode_fused_experts(x, rw, ri, n, c, l_, budget, w13, w2, variant=variant,
                                         status=status)
    ew, ei = ops.decode(rw, ri, n, c, l_, budget, variant=variant)
    ye = ops.fused_experts(x, ew, ei, w13, w2)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, "a pipeline wait timed out"
    assert torch.equal(oi, ei.to(torch.int32)) and torch.equal(ow, ew.float())
    valid = (ei >= 0) & (ei < lay.experts)
    ref = reference(x, torch.where(valid, ew, 0.0), torch.where(valid, ei, 0).to(torch.int64),
                    w13, w2)
    scale = ref.abs().max().item()
    torch.testing.assert_close(y.float(), ye.float(), rtol=2e-2, atol=2e-2 * scale)
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2 * scale)
    return y, oi.cpu().numpy()


def test_qwen3_decode_layer():
    """The Qwen3 decode layer: B=256, E=128, top-8, D=64, hidden 2048, intermediate 768."""
    lay = W.layer("qwen3_decode")
    _, oi = run(lay, 64, "qwen3", 2048, 768, seed=21)
    assert duplicate_routes(oi) > 0  # the merge path ran


@pytest.mark.parametrize("batch,budget", [(1, 64), (128, 64), (512, 128)])
def test_dsv4_decode_layer(batch, budget):
    lay = W.Layer(seed=2100 + batch, tokens=batch, experts=256, top_k=8, kind="dsv4")
    run(lay, budget, "dsv4", 512, 256, seed=22)


def test_largest_batch_and_small_budget():
    """8192 routes (the limit), a budget of 8 experts (many merged routes)."""
    lay = W.Layer(seed=3300, tokens=1024, experts=128, top_k=8, kind="qwen3")
    _, oi = run(lay, 8, "qwen3", 256, 128, seed=23)
    assert duplicate_routes(oi) > 1000


def test_invalid_router_ids_and_determinism():
    """Router ids of -1 and >= E pass through decode and contribute nothing to the layer."""
    def edit(ri):
        ri = ri.clone()
        ri[::7, 3] = -1
        ri[::11, 5] = 999
        return ri
    lay = W.Layer(seed=3400, tokens=200, experts=64, top_k=6, kind="qwen3")
    a, _ = run(lay, 16, "qwen3", 512, 256, seed=24, edit_ids=edit)
    b, _ = run(lay, 16, "qwen3", 512, 256, seed=24, edit_ids=edit)
    assert torch.equal(a, b)


def test_limits_are_errors():
    lay = W.Layer(seed=3500, tokens=8, experts=512, top_k=8, kind="qwen3")
    rw, ri = ops.router_topk(cuda(lay.logits), 8)
    _, w13, w2 = weights(512, 256, 128, 25)
    x = torch.zeros(8, 256, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError):
        ops.decode_fused_experts(x, rw, ri, cuda(lay.norms), cuda(lay.coeff), cuda(lay.loss), 64,
                                 w13, w2)
