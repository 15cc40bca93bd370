"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run in a container that has the reference project checked out (read-only)
at REFERENCE_ROOT (default /root/reference):

    python tests/golden/make_golden.py [calibration]

(with `calibration`, only calibration_reference.npz is written).  The reference's Triton kernels (exfold/qwen3/kernels.py) run on CPU tensors
under TRITON_INTERPRET=1, launched exactly as their host wrappers launch them
(the wrappers themselves refuse CPU tensors).  The DeepSeek-V4 CUDA kernels
cannot run without a GPU, so the DeepSeek-V4 fixtures come from the
reference's own torch restatements in tests/test_deepseek_v4_cuda.py
(imported with the CUDA op loader stubbed out).  The real Qwen3 calibration
artifact contributes two sanitized layers.  Nothing here is needed at test
time: the tests read only the .npz files this script writes.
"""

from __future__ import annotations

import hashlib
import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"
REFERENCE_ROOT = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))
HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REFERENCE_ROOT))
sys.path.insert(0, str(REPO / "exfold-moe_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402

from exfold.qwen3 import kernels as RK  # noqa: E402  (reference Triton kernels)
from exfold_b200 import workloads as W  # noqa: E402

# the DeepSeek-V4 test module imports the CUDA op loader at import time
_stub = types.ModuleType("exfold.deepseek_v4.cuda_ops")
_stub.fold_decode = _stub.fold_prefill = None
sys.modules["exfold.deepseek_v4.cuda_ops"] = _stub
sys.path.insert(0, str(REFERENCE_ROOT / "tests"))
import test_deepseek_v4_cuda as RDS  # noqa: E402
import test_qwen3_kernels as RQT  # noqa: E402

LARGE = 1e30


# --- reference Triton kernels launched as exfold/qwen3/kernels.py launches them ---------------
def ref_project_prefill(w, ids, coeff, target_k, loss):
    tokens, k = w.shape
    ow = torch.empty((tokens, target_k), dtype=w.dtype)
    oi = torch.empty((tokens, target_k), dtype=ids.dtype)
    bt = 128 if tokens >= 128 else triton.next_power_of_2(tokens)
    RK._project_prefill_kernel[(triton.cdiv(tokens, bt),)](
        w, ids, coeff, loss, ow, oi, tokens, w.stride(0), w.stride(1), ids.stride(0),
        ids.stride(1), coeff.stride(0), coeff.stride(1), ow.stride(0), ow.stride(1),
        oi.stride(0), oi.stride(1), K=k, TARGET_K=target_k, BLOCK_TOKENS=bt, num_warps=4)
    return ow, oi


def ref_reroute(w, ids, subset, coeff, loss):
    b, k = w.shape
    ow, oi = torch.empty_like(w), torch.empty_like(ids)
    bs = max(16, triton.next_power_of_2(subset.numel()))
    bb = triton.next_power_of_2(min(b, 64))
    RK._reroute_decode_kernel[(triton.cdiv(b, bb),)](
        w, ids, subset, coeff, loss, ow, oi, b, subset.numel(), w.stride(0), w.stride(1),
        ids.stride(0), ids.stride(1), coeff.stride(0), coeff.stride(1), ow.stride(0),
        ow.stride(1), oi.stride(0), oi.stride(1), K=k, BLOCK_SUBSET=bs, BLOCK_BATCH=bb,
        num_warps=4)
    return ow, oi


def ref_select_subset(w, ids, norms, subset_size):
    experts = norms.numel()
    b, k = w.shape
    imp = torch.empty(experts, dtype=torch.float32)
    subset = torch.empty(subset_size, dtype=torch.int32)
    RK._zero_importance_kernel[(triton.cdiv(experts, 128),)](imp, experts, BLOCK_EXPERTS=128,
                                                             num_warps=4)
    RK._accumulate_decode_importance_kernel[(triton.cdiv(b * k, 256),)](
        w, ids, norms, imp, b * k, w.stride(0), w.stride(1), ids.stride(0), ids.stride(1),
        K=k, BLOCK_ROUTES=256, num_warps=4)
    RK._select_decode_subset_kernel[(1,)](imp, subset, experts, SUBSET_SIZE=subset_size,
                                          BLOCK_EXPERTS=triton.next_power_of_2(experts),
                                          num_warps=4)
    return imp, subset


def ref_select_and_reroute(w, ids, norms, coeff, loss, subset_size):
    imp, subset = ref_select_subset(w, ids, norms, subset_size)
    ow, oi = ref_reroute(w, ids, subset, coeff, loss)
    return ow, oi, subset, imp


def ref_static_remap(w, ids, target, scale):
    b, k = w.shape
    bb = max(1, triton.next_power_of_2(min(b, 128)))
    RK._static_decode_remap_kernel[(triton.cdiv(b, bb),)](
        w, ids, target, scale, b, w.stride(0), w.stride(1), ids.stride(0), ids.stride(1),
        K=k, BLOCK_BATCH=bb, num_warps=4)
    return w, ids


def torch_softmax_router(logits, k):
    """tests/test_qwen3_kernels.py:35-37."""
    scores = torch.softmax(logits, dim=-1)
    w, ids = scores.topk(k, dim=-1)
    return w / w.sum(dim=-1, keepdim=True), ids.to(torch.int32)


def torch_sigmoid_bias_router(logits, bias, k):
    """vLLM fused_topk_bias torch path (sigmoid + bias select, unbiased renormalised weights)."""
    scores = logits.sigmoid()
    ids = torch.topk(scores + bias.unsqueeze(0), k=k, dim=-1, sorted=True)[1]
    w = scores.gather(1, ids)
    return (w / w.sum(dim=-1, keepdim=True)).float(), ids.to(torch.int32)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


def n(t):
    return t.detach().cpu().numpy()


# --- 1. reference Qwen3 kernel tests (tests/test_qwen3_kernels.py), seed 0 on CPU ------------
def qwen3_tests():
    torch.manual_seed(0)
    out = {}
    # test_prefill (29-59)
    experts, top_k, tokens = 128, 8, 257
    coeff = (torch.randn(experts, experts) * 0.1).contiguous()
    loss = torch.rand(experts, experts).contiguous()
    loss.diagonal().fill_(LARGE)
    scores = torch.softmax(torch.randn(tokens, experts), dim=-1)
    w, ids = scores.topk(top_k, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    ids = ids.to(torch.int32)
    ow, oi = ref_project_prefill(w, ids, coeff, 4, loss)
    out.update(prefill_w=n(w), prefill_ids=n(ids), prefill_coeff=n(coeff), prefill_loss=n(loss),
               prefill_out_w=n(ow), prefill_out_ids=n(oi))
    # test_decode (62-95)
    experts, top_k, batch, subset_size = 128, 8, 23, 64
    coeff = (torch.randn(experts, experts) * 0.1).contiguous()
    loss = torch.rand(experts, experts).contiguous()
    loss.diagonal().fill_(LARGE)
    scores = torch.softmax(torch.randn(batch, experts), dim=-1)
    w, ids = scores.topk(top_k, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    ids = ids.to(torch.int32)
    subset = torch.randperm(experts)[:subset_size].to(torch.int32)
    ow, oi = ref_reroute(w, ids, subset, coeff, loss)
    out.update(decode_w=n(w), decode_ids=n(ids), decode_coeff=n(coeff), decode_loss=n(loss),
               decode_subset=n(subset), decode_out_w=n(ow), decode_out_ids=n(oi))
    # test_unobserved_pair_is_noop (98-116)
    coeff = torch.ones((8, 8))
    loss = torch.full((8, 8), LARGE)
    w = torch.full((1, 8), 0.125)
    ids = torch.arange(8, dtype=torch.int32).unsqueeze(0)
    pw, pi = ref_project_prefill(w, ids, coeff, 4, loss)
    dw, di = ref_reroute(w, ids, ids[0, :4].contiguous(), coeff, loss)
    out.update(noop_prefill_w=n(pw), noop_prefill_ids=n(pi), noop_decode_w=n(dw),
               noop_decode_ids=n(di))
    # test_decode_selection (119-149)
    experts, top_k, batch, subset_size = 128, 8, 32, 32
    coeff = (torch.randn(experts, experts) * 0.1).contiguous()
    loss = torch.rand(experts, experts).contiguous()
    loss.diagonal().fill_(LARGE)
    norms = torch.rand(experts).add_(0.1).contiguous()
    scores = torch.softmax(torch.randn(batch, experts), dim=-1)
    w, ids = scores.topk(top_k, dim=-1)
    ids = ids.to(torch.int32)
    w = w.contiguous()
    ow, oi, subset, imp = ref_select_and_reroute(w, ids, norms, coeff, loss, subset_size)
    out.update(select_w=n(w), select_ids=n(ids), select_coeff=n(coeff), select_loss=n(loss),
               select_norms=n(norms), select_out_w=n(ow), select_out_ids=n(oi),
               select_subset=n(subset), select_importance=n(imp))
    # test_static_decode_remap (152-169)
    experts, top_k, batch = 128, 8, 37
    w = torch.rand(batch, top_k)
    ids = torch.randint(experts, (batch, top_k), dtype=torch.int32)
    target = torch.arange(experts, dtype=torch.int32)
    target[64:] -= 64
    scale = torch.linspace(0.5, 1.5, experts)
    out.update(static_w=n(w), static_ids=n(ids), static_target=n(target), static_scale=n(scale))
    rw, ri = ref_static_remap(w.clone(), ids.clone(), target, scale)
    out.update(static_out_w=n(rw), static_out_ids=n(ri))
    # cross-check: the reference test's own torch restatement agrees with its kernel
    tp = RQT.select_target  # noqa: F841  (kept importable: restatement used by the test)
    return out


# --- 2. DeepSeek-V4 correctness test (tests/test_deepseek_v4_cuda.py:59-93) on CPU -------------
def dsv4_tests():
    torch.manual_seed(20260809)
    experts, tokens, topk = 256, 64, 8
    w = torch.rand(tokens, topk, dtype=torch.bfloat16)
    ids = torch.stack([torch.randperm(experts)[:topk] for _ in range(tokens)]).to(torch.int32)
    coeff = torch.rand(experts, experts)
    sel = torch.rand(experts, experts)
    conf = torch.rand(experts, experts)
    norms = torch.rand(experts).add_(0.1)
    pw, pi = RDS.prefill_reference(w, ids, coeff, sel, conf)
    dw, di = RDS.decode_reference(w, ids, coeff, sel, norms, 64)
    return dict(w_bf16_as_f32=n(w.float()), ids=n(ids), coeff=n(coeff), sel=n(sel), conf=n(conf),
                norms=n(norms), prefill_out_w=n(pw), prefill_out_ids=n(pi).astype(np.int32),
                decode_out_w=n(dw), decode_out_ids=n(di).astype(np.int32))


# --- 3. real Qwen3 calibration artifact: two sanitized layers --------------------------------
def artifact_layers():
    from exfold.qwen3 import vllm_patch as RV

    path = REFERENCE_ROOT / "artifacts" / "qwen3-30b-a3b.pt"
    coeff_all, loss_all, norms_all = RV._load_artifact(str(path))
    out = {}
    os.environ["EXFOLD_QWEN3_DECODE_POLICY"] = "static_norm"
    for layer in (0, 47):
        coeff, loss, norms = coeff_all[layer], loss_all[layer], norms_all[layer]
        x = torch.from_numpy(W.logits(7000 + layer, 512, 128))
        w, ids = torch_softmax_router(x, 8)
        pw, pi = ref_project_prefill(w.contiguous(), ids.contiguous(), coeff, 4, loss)
        dw, di, subset, imp = ref_select_and_reroute(w[:64].contiguous(), ids[:64].contiguous(),
                                                     norms, coeff, loss, 64)
        router = RV._make_router(coeff, loss, norms, 8, 32)
        static = dict(zip(router.__code__.co_freevars, router.__closure__))
        target, scale = static["static_cpu"].cell_contents
        out.update({f"l{layer}_coeff": n(coeff), f"l{layer}_loss": n(loss),
                    f"l{layer}_norms": n(norms), f"l{layer}_logits": n(x),
                    f"l{layer}_prefill_out_w": n(pw), f"l{layer}_prefill_out_ids": n(pi),
                    f"l{layer}_decode_out_w": n(dw), f"l{layer}_decode_out_ids": n(di),
                    f"l{layer}_decode_subset": n(subset), f"l{layer}_static_target": n(target),
                    f"l{layer}_static_scale": n(scale)})
    return out


# --- 4. workload-sized cases: inputs regenerated from workloads.py, outputs stored -----------
def workload_cases():
    out = {}
    # qwen3 prefill, T=4096, E=128, P=4 (reference Triton fold on the torch router)
    lay = W.layer("qwen3_prefill")
    x = torch.from_numpy(lay.logits)
    w, ids = torch_softmax_router(x, 8)
    pw, pi = ref_project_prefill(w.contiguous(), ids.contiguous(), torch.from_numpy(lay.coeff), 4,
                                 torch.from_numpy(lay.loss))
    out.update(qp_digest=digest(lay.logits, lay.coeff, lay.loss), qp_router_w=n(w),
               qp_router_ids=n(ids).astype(np.int16), qp_out_w=n(pw),
               qp_out_ids=n(pi).astype(np.int16))
    # qwen3 decode, B=256, D=64 (reference Triton select + reroute chain)
    lay = W.layer("qwen3_decode")
    x = torch.from_numpy(lay.logits)
    w, ids = torch_softmax_router(x, 8)
    dw, di, subset, imp = ref_select_and_reroute(
        w.contiguous(), ids.contiguous(), torch.from_numpy(lay.norms),
        torch.from_numpy(lay.coeff), torch.from_numpy(lay.loss), 64)
    out.update(qd_digest=digest(lay.logits, lay.coeff, lay.loss, lay.norms), qd_out_w=n(dw),
               qd_out_ids=n(di).astype(np.int16), qd_subset=n(subset),
               qd_importance=n(imp))
    # DeepSeek-style prefill, first 4096 tokens of the T=65536 workload, P=3, similarity_blend
    # with confidence := selection loss (the loader's fallback), reference torch restatement
    lay = W.layer("dsv4_prefill", tokens=4096)
    x = torch.from_numpy(lay.logits)
    w, ids = torch_sigmoid_bias_router(x, torch.from_numpy(lay.bias), 8)
    coeff = torch.from_numpy(lay.coeff).clone()
    loss = torch.from_numpy(lay.loss).clone()
    coeff.diagonal().fill_(1.0)
    loss.diagonal().fill_(LARGE)
    conf = loss.clone()
    conf.diagonal().fill_(0.0)
    pw, pi = RDS.prefill_reference(w, ids, coeff, loss, conf)
    out.update(dp_digest=digest(lay.logits, lay.bias, lay.coeff, lay.loss), dp_router_w=n(w),
               dp_router_ids=n(ids).astype(np.int16), dp_out_w=n(pw),
               dp_out_ids=n(pi).astype(np.int16))
    # DeepSeek-style decode sweep, B in {8,32,128,512} x D in {64,128}
    cfg = W.WORKLOADS["dsv4_decode"]
    for b in cfg["batches"]:
        lay = W.Layer(seed=cfg["seed"], tokens=b, experts=256, top_k=8, kind="dsv4")
        x = torch.from_numpy(lay.logits)
        w, ids = torch_sigmoid_bias_router(x, torch.from_numpy(lay.bias), 8)
        coeff = torch.from_numpy(lay.coeff).clone()
        loss = torch.from_numpy(lay.loss).clone()
        coeff.diagonal().fill_(1.0)
        loss.diagonal().fill_(LARGE)
        for d in cfg["budgets"]:
            dw, di = RDS.decode_reference(w, ids, coeff, loss, torch.from_numpy(lay.norms), d)
            out[f"dd_b{b}_d{d}_out_w"] = n(dw)
            out[f"dd_b{b}_d{d}_out_ids"] = n(di).astype(np.int16)
        out[f"dd_b{b}_digest"] = digest(lay.logits, lay.bias, lay.coeff, lay.loss, lay.norms)
    return out


def calibration_cases():
    """The reference accumulator (exfold/qwen3/calibration.py PairwiseScalarStats) on CPU:
    random routes with duplicate expert ids and experts that are never routed (median fallback
    of expert_norms), outputs rounded to bf16 so the same values can be fed in bf16."""
    from exfold.qwen3.calibration import PairwiseScalarStats

    out = {}
    gen = torch.Generator().manual_seed(9001)
    for name, (E, T, k, H, hi) in {"a": (16, 300, 8, 96, 12), "b": (24, 64, 6, 520, 24)}.items():
        ids = torch.randint(0, hi, (T, k), generator=gen)
        outputs = torch.randn((T, k, H), generator=gen).bfloat16().float()
        stats = PairwiseScalarStats(E, ridge=1e-3, clip_min=-4.0, clip_max=4.0)
        half = T // 2
        stats.update(ids[:half], outputs[:half])
        stats.update(ids[half:], outputs[half:])
        coeff, loss = stats.finalize()
        out.update({f"{name}_ids": n(ids).astype(np.int32), f"{name}_outputs": n(outputs),
                    f"{name}_dot": n(stats.dot), f"{name}_target_sq": n(stats.target_sq_norm),
                    f"{name}_source_sq": n(stats.source_sq_norm),
                    f"{name}_norm_sum": n(stats.expert_norm_sum),
                    f"{name}_norm_count": n(stats.expert_norm_count),
                    f"{name}_coeff": n(coeff), f"{name}_loss": n(loss),
                    f"{name}_norms": n(stats.expert_norms())})
    return out


def main():
    if sys.argv[1:] == ["calibration"]:
        np.savez_compressed(HERE / "calibration_reference.npz", **calibration_cases())
        return
    np.savez_compressed(HERE / "calibration_reference.npz", **calibration_cases())
    np.savez_compressed(HERE / "qwen3_reference_tests.npz", **qwen3_tests())
    np.savez_compressed(HERE / "dsv4_reference_tests.npz", **dsv4_tests())
    np.savez_compressed(HERE / "qwen3_artifact_layers.npz", **artifact_layers())
    np.savez_compressed(HERE / "workload_cases.npz", **workload_cases())
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
