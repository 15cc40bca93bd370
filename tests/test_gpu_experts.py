"""GPU numerics of the tcgen05 grouped SwiGLU expert layer against a plain torch fp32 reference.

The reference computes every route in fp32 from the same bf16 inputs, rounds the SwiGLU
activation to bf16 as the kernel (and vLLM's intermediate cache) does, and sums the weighted
routes; routes whose expert id is out of range contribute nothing.  Tolerance: bf16, 2e-2
relative to the output scale.  Both kernel paths are covered: blocks of 128 routes on the M side
(many routes per expert) and blocks of 64 routes on the N side with the combine inside GEMM-2
(64 routes per expert or fewer on average).
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
        if e < 0 or e >= w13.shape[0]:
            continue  # routes of an expert id out of range are dropped
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


@pytest.mark.parametrize("tokens,experts,top_k", [(300, 32, 4), (3000, 8, 4)])
def test_invalid_and_duplicate_expert_ids(tokens, experts, top_k):
    """Ids of -1 and >= experts are skipped; a token with no valid id gets y = 0; an expert named
    twice by one token counts twice.  (300, 32, 4) takes the decode kernels, (3000, 8, 4) the
    prefill ones."""
    gen = torch.Generator(device=DEV)
    gen.manual_seed(77)
    logits = torch.randn(tokens, experts, generator=gen, device=DEV)
    ids = logits.topk(top_k, dim=-1).indices.to(torch.int32)
    ids[0, :] = -1
    ids[1, 1] = experts
    ids[2, 1] = ids[2, 0]
    ids[3, :] = 5
    ids[4, :] = torch.tensor([-1, experts + 7, 3, -1], dtype=torch.int32)
    y, _ = run_case(tokens, experts, top_k, hidden=512, inter=256, seed=78, ids=ids)
    assert torch.count_nonzero(y[0]).item() == 0


def test_deterministic_prefill_path():
    a, _ = run_case(tokens=2000, experts=8, top_k=4, hidden=512, inter=256, seed=9)
    b, _ = run_case(tokens=2000, experts=8, top_k=4, hidden=512, inter=256, seed=9)
    assert torch.equal(a, b)
