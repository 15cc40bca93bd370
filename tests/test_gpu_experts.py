"""GPU numerics of the tcgen05 grouped SwiGLU expert layer against a plain torch fp32 reference.

The reference computes every route in fp32 from the same bf16 inputs, rounds the SwiGLU
activation to bf16 as the kernel (and vLLM's intermediate cache) does, and sums the weighted
routes.  Tolerance: bf16, 2e-2 relative to the output scale.
"""

from __future__ import annotations

import pytest
import torch

from exfold_b200 import ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def reference(x, topk_w, topk_ids, w13, w2):
    tokens, hidden = x.shape
    inter = w13.shape[1] // 2
    y = torch.zeros(tokens, hidden, dtype=torch.float32, device=x.device)
    xf = x.float()
    for e in torch.unique(topk_ids).tolist():
        rows, slots = torch.nonzero(topk_ids == e, as_tuple=True)
        h = xf[rows]
        w = w13[e].float()
        g = h @ w[:inter].T
        u = h @ w[inter:].T
        a = (torch.nn.functional.silu(g) * u).to(torch.bfloat16).float()
        o = a @ w2[e].float().T
        y.index_add_(0, rows, o * topk_w[rows, slots].unsqueeze(1).float())
    return y


def routing(tokens, experts, top_k, gen):
    logits = torch.randn(tokens, experts, generator=gen, device=DEV)
    w, ids = torch.softmax(logits, -1).topk(top_k, dim=-1)
    return (w / w.sum(-1, keepdim=True)).contiguous(), ids.to(torch.int32).contiguous()


def run_case(tokens, experts, top_k, hidden, inter, seed, ids=None):
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    x = torch.randn(tokens, hidden, generator=gen, device=DEV).to(torch.bfloat16)
    w13 = (0.02 * torch.randn(experts, 2 * inter, hidden, generator=gen, device=DEV)).to(
        torch.bfloat16)
    w2 = (0.02 * torch.randn(experts, hidden, inter, generator=gen, device=DEV)).to(torch.bfloat16)
    tw, ti = routing(tokens, experts, top_k, gen)
    if ids is not None:
        ti = ids.to(DEV, torch.int32).contiguous()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    y = ops.fused_experts(x, tw, ti, w13, w2, status=status)
    ref = reference(x, tw, ti, w13, w2)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, "a pipeline wait timed out"
    scale = ref.abs().max().item()
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2 * scale)
    return y, ref


def test_small_shapes():
    run_case(tokens=300, experts=16, top_k=4, hidden=512, inter=256, seed=1)
    run_case(tokens=1, experts=8, top_k=2, hidden=256, inter=128, seed=2)
    run_case(tokens=129, experts=64, top_k=8, hidden=1024, inter=384, seed=3)


def test_qwen3_decode_shape():
    """B=256 routed to E=128 experts, hidden 2048, intermediate 768 (the Qwen3 decode layer)."""
    run_case(tokens=256, experts=128, top_k=8, hidden=2048, inter=768, seed=4)


def test_decode_tiles_block_fill_levels():
    """Few routes per expert on average (the decode path: 128-wide N tile), with experts holding
    1, 63, 64, 65, 128, 129 and 200 routes: nearly empty, half-full, full and split blocks."""
    tokens, experts = 400, 64
    counts = {0: 1, 1: 63, 2: 64, 3: 65, 4: 128, 5: 129, 6: 200}
    slot0, slot1 = [], []
    for e, c in counts.items():
        (slot0 if len(slot0) + c <= tokens else slot1).extend([e] * c)
    rng = torch.Generator().manual_seed(11)
    fill0 = torch.randint(8, 36, (tokens - len(slot0),), generator=rng).tolist()
    fill1 = torch.randint(36, 64, (tokens - len(slot1),), generator=rng).tolist()
    ids = torch.stack([torch.tensor(slot0 + fill0), torch.tensor(slot1 + fill1)], 1)
    perm = torch.randperm(tokens, generator=rng)
    run_case(tokens, experts, 2, hidden=512, inter=256, seed=12, ids=ids[perm])


def test_prefill_many_rows_per_expert():
    """Several 128-row blocks per expert, hidden 4096, intermediate 2048 (DeepSeek-style)."""
    run_case(tokens=4096, experts=32, top_k=3, hidden=4096, inter=2048, seed=5)


def test_deterministic():
    a, _ = run_case(tokens=200, experts=16, top_k=4, hidden=512, inter=256, seed=6)
    b, _ = run_case(tokens=200, experts=16, top_k=4, hidden=512, inter=256, seed=6)
    assert torch.equal(a, b)
