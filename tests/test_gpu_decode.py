"""GPU parity: decode budget (Qwen3 and DeepSeek-V4 semantics), reroute, static remap/table,
split (sharded) decode, CUDA-graph capture."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from exfold_b200 import ops
from exfold_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu
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
    return coeff, loss


def test_qwen3_reference_fixtures():
    from exfold_b200.qwen3.kernels import (remap_decode_static, reroute_decode_subset,
                                           select_and_reroute_decode)

    qt = np.load(GOLDEN / "qwen3_reference_tests.npz")
    ow, oi = reroute_decode_subset(cuda(qt["decode_w"]), cuda(qt["decode_ids"]),
                                   cuda(qt["decode_subset"]), cuda(qt["decode_coeff"]),
                                   cuda(qt["decode_loss"]))
    np.testing.assert_array_equal(host(oi), qt["decode_out_ids"])
    np.testing.assert_array_equal(host(ow), qt["decode_out_w"])
    w8 = cuda(np.full((1, 8), 0.125, np.float32))
    i8 = cuda(np.arange(8, dtype=np.int32)[None])
    dw, di = reroute_decode_subset(w8, i8, i8[0, :4], cuda(np.ones((8, 8), np.float32)),
                                   cuda(np.full((8, 8), 1e30, np.float32)))
    np.testing.assert_array_equal(host(dw), qt["noop_decode_w"])
    np.testing.assert_array_equal(host(di), qt["noop_decode_ids"])
    ow, oi = select_and_reroute_decode(cuda(qt["select_w"]), cuda(qt["select_ids"]),
                                       cuda(qt["select_norms"]), cuda(qt["select_coeff"]),
                                       cuda(qt["select_loss"]), 32)
    np.testing.assert_array_equal(host(oi), qt["select_out_ids"])
    np.testing.assert_allclose(host(ow), qt["select_out_w"], atol=5e-5, rtol=5e-5)
    sw, si = remap_decode_static(cuda(qt["static_w"]), cuda(qt["static_ids"]),
                                 cuda(qt["static_target"]), cuda(qt["static_scale"]))
    np.testing.assert_array_equal(host(si), qt["static_out_ids"])
    np.testing.assert_array_equal(host(sw), qt["static_out_w"])


def test_qwen3_decode_workload_config1():
    wc = np.load(GOLDEN / "workload_cases.npz")
    lay = W.layer("qwen3_decode")
    rw, ri = O.router_topk(lay.logits, 8, "softmax")
    subset = torch.empty(64, dtype=torch.int32, device=DEV)
    ow, oi = ops.decode(cuda(rw), cuda(ri), cuda(lay.norms), cuda(lay.coeff), cuda(lay.loss), 64,
                        variant="qwen3", subset_out=subset)
    ew, ei, es = O.decode_qwen3(rw, ri, lay.norms, lay.coeff, lay.loss, 64)
    np.testing.assert_array_equal(host(subset), es)
    np.testing.assert_array_equal(host(oi), ei)
    np.testing.assert_array_equal(host(ow), ew)
    np.testing.assert_array_equal(host(subset), wc["qd_subset"])
    np.testing.assert_array_equal(host(oi), wc["qd_out_ids"])
    np.testing.assert_allclose(host(ow), wc["qd_out_w"], rtol=1e-5, atol=0)


def test_dsv4_reference_fixture_and_graph():
    from exfold_b200.deepseek_v4.cuda_ops import fold_decode

    dt = np.load(GOLDEN / "dsv4_reference_tests.npz")
    w = torch.from_numpy(dt["w_bf16_as_f32"]).to(torch.bfloat16).to(DEV)
    ids = cuda(dt["ids"])
    ow, oi = fold_decode(w, ids, cuda(dt["coeff"]), cuda(dt["sel"]), cuda(dt["norms"]), 64)
    np.testing.assert_array_equal(host(oi), dt["decode_out_ids"])
    np.testing.assert_allclose(host(ow.float()), dt["decode_out_w"], atol=2e-2, rtol=2e-2)
    ew, ei = O.decode_dsv4(dt["w_bf16_as_f32"], dt["ids"], dt["norms"], dt["coeff"], dt["sel"], 64)
    np.testing.assert_array_equal(host(oi), ei)
    np.testing.assert_array_equal(host(ow.float()),
                                  torch.from_numpy(ew).to(torch.bfloat16).float().numpy())
    # CUDA graph capture + replay (tests/test_deepseek_v4_cuda.py:96-116), replay == eager
    coeff, sel, norms = cuda(dt["coeff"]), cuda(dt["sel"]), cuda(dt["norms"])
    for _ in range(3):
        fold_decode(w, ids, coeff, sel, norms, 64)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gw, gi = fold_decode(w, ids, coeff, sel, norms, 64)
    graph.replay()
    torch.cuda.synchronize()
    assert gw.shape == w.shape and gi.shape == ids.shape
    np.testing.assert_array_equal(host(gi), host(oi))
    np.testing.assert_array_equal(host(gw.float()), host(ow.float()))


def test_dsv4_decode_sweep_config3():
    from exfold_b200.deepseek_v4.cuda_ops import fold_decode

    wc = np.load(GOLDEN / "workload_cases.npz")
    cfg = W.WORKLOADS["dsv4_decode"]
    for b in cfg["batches"]:
        lay = W.Layer(seed=cfg["seed"], tokens=b, experts=256, top_k=8, kind="dsv4")
        rw, ri = O.router_topk(lay.logits, 8, "sigmoid", lay.bias)
        coeff, loss = dsv4_tables(lay)
        for d in cfg["budgets"]:
            ow, oi = fold_decode(cuda(rw), cuda(ri), cuda(coeff), cuda(loss), cuda(lay.norms), d)
            ew, ei = O.decode_dsv4(rw, ri, lay.norms, coeff, loss, d)
            np.testing.assert_array_equal(host(oi), ei)
            np.testing.assert_array_equal(host(ow), ew)
            np.testing.assert_array_equal(host(oi), wc[f"dd_b{b}_d{d}_out_ids"])
            np.testing.assert_allclose(host(ow), wc[f"dd_b{b}_d{d}_out_w"], rtol=1e-5, atol=0)


@pytest.mark.parametrize("variant", ["qwen3", "dsv4"])
@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("idtype", [torch.int32, torch.int64])
def test_decode_dtypes_and_sizes(variant, wdtype, idtype):
    for experts, batch, budget in ((128, 256, 64), (256, 1024, 128), (64, 3, 7), (512, 100, 500)):
        lay = W.Layer(seed=900 + batch, tokens=batch, experts=experts, top_k=8, kind="qwen3")
        rw, ri = O.router_topk(lay.logits, 8, "softmax")
        w_t = torch.from_numpy(rw).to(wdtype)
        w_in = w_t.float().numpy()
        ow, oi = ops.decode(w_t.to(DEV), cuda(ri).to(idtype), cuda(lay.norms), cuda(lay.coeff),
                            cuda(lay.loss), budget, variant=variant)
        if variant == "qwen3":
            # exfold/qwen3/kernels.py casts the scale to the weight dtype before multiplying,
            # so half-precision results may differ from the fp32 oracle by one unit in the last place
            ew, ei, _ = O.decode_qwen3(w_in, ri, lay.norms, lay.coeff, lay.loss, budget)
        else:
            ew, ei = O.decode_dsv4(w_in, ri, lay.norms, lay.coeff, lay.loss, budget)
        np.testing.assert_array_equal(host(oi).astype(np.int32), ei)
        got = host(ow.float())
        ref = torch.from_numpy(ew).to(wdtype).float().numpy()
        if wdtype == torch.float32:
            np.testing.assert_array_equal(got, ref)
        else:
            np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=0)


@pytest.mark.parametrize("variant", ["qwen3", "dsv4"])
def test_decode_table_paths(variant):
    """The decode reads its tables from shared memory at E <= 128 (even E, 16-byte aligned
    tables) and from L2 otherwise; both, and batches of more than one 8192-route load batch,
    equal the oracle bit for bit."""
    cases = ((128, 1500, 64), (96, 300, 40), (127, 200, 50), (128, 1024, 64))
    for n, (experts, batch, budget) in enumerate(cases):
        lay = W.Layer(seed=1700 + n, tokens=batch, experts=experts, top_k=8, kind="qwen3")
        rw, ri = O.router_topk(lay.logits, 8, "softmax")
        coeff, loss = cuda(lay.coeff), cuda(lay.loss)
        if n == 3:  # tables 4 bytes off a 16-byte boundary: the L2 path at E = 128
            cbuf = torch.zeros(experts * experts + 1, device=DEV)
            lbuf = torch.zeros(experts * experts + 1, device=DEV)
            cbuf[1:] = coeff.reshape(-1)
            lbuf[1:] = loss.reshape(-1)
            coeff = cbuf[1:].view(experts, experts)
            loss = lbuf[1:].view(experts, experts)
            assert coeff.data_ptr() % 16 != 0 and loss.data_ptr() % 16 != 0
        ow, oi = ops.decode(cuda(rw), cuda(ri), cuda(lay.norms), coeff, loss, budget,
                            variant=variant)
        if variant == "qwen3":
            ew, ei, _ = O.decode_qwen3(rw, ri, lay.norms, lay.coeff, lay.loss, budget)
        else:
            ew, ei = O.decode_dsv4(rw, ri, lay.norms, lay.coeff, lay.loss, budget)
        np.testing.assert_array_equal(host(oi), ei)
        np.testing.assert_array_equal(host(ow), ew)


def test_split_decode_equals_fused():
    """importance on shards + summed vector + apply == one fused decode (bit for bit)."""
    lay = W.layer("qwen3_layers", tokens=1024, layer_index=3)
    rw, ri = O.router_topk(lay.logits, 8, "softmax")
    for variant in ("qwen3", "dsv4"):
        fw, fi = ops.decode(cuda(rw), cuda(ri), cuda(lay.norms), cuda(lay.coeff), cuda(lay.loss),
                            64, variant=variant)
        imp = torch.zeros(128, dtype=torch.int64, device=DEV)
        for shard in np.array_split(np.arange(1024), 4):
            ops.decode_importance(cuda(rw[shard]), cuda(ri[shard]), cuda(lay.norms), imp)
        np.testing.assert_array_equal(host(imp), O.importance(rw, ri, lay.norms))
        outs = [ops.decode_apply(imp, cuda(rw[s]), cuda(ri[s]), cuda(lay.coeff), cuda(lay.loss),
                                 64, variant=variant) for s in np.array_split(np.arange(1024), 4)]
        np.testing.assert_array_equal(np.concatenate([host(o[1]) for o in outs]), host(fi))
        np.testing.assert_array_equal(np.concatenate([host(o[0]) for o in outs]), host(fw))


def test_static_table_artifact_layers():
    art = np.load(GOLDEN / "qwen3_artifact_layers.npz")
    for layer in (0, 47):
        p = f"l{layer}_"
        t, s = ops.static_table(cuda(art[p + "norms"]), cuda(art[p + "coeff"]),
                                cuda(art[p + "loss"]), 32)
        np.testing.assert_array_equal(host(t), art[p + "static_target"])
        np.testing.assert_array_equal(host(s), art[p + "static_scale"])
        rw, ri = O.router_topk(art[p + "logits"], 8, "softmax")
        dw, di = ops.decode(cuda(rw[:64]), cuda(ri[:64]), cuda(art[p + "norms"]),
                            cuda(art[p + "coeff"]), cuda(art[p + "loss"]), 64, variant="qwen3")
        np.testing.assert_array_equal(host(di), art[p + "decode_out_ids"])
        np.testing.assert_allclose(host(dw), art[p + "decode_out_w"], rtol=2e-6, atol=1e-8)


def test_decode_edge_cases():
    from exfold_b200.qwen3.kernels import select_and_reroute_decode

    lay = W.layer("qwen3_decode", tokens=16)
    rw, ri = O.router_topk(lay.logits, 8, "softmax")
    # budget >= experts and empty batch are passthrough (kernels.py:449-450)
    w, i = select_and_reroute_decode(cuda(rw), cuda(ri), cuda(lay.norms), cuda(lay.coeff),
                                     cuda(lay.loss), 500)
    np.testing.assert_array_equal(host(i), ri)
    w, i = select_and_reroute_decode(cuda(rw[:0]), cuda(ri[:0]), cuda(lay.norms),
                                     cuda(lay.coeff), cuda(lay.loss), 8)
    assert w.shape == (0, 8)
    # budget 1, all-equal importance (ties -> lowest expert id), out-of-range ids stay untouched
    ri2 = ri.copy()
    ri2[0, 0] = 1000
    ow, oi = ops.decode(cuda(np.ones_like(rw)), cuda(ri2), cuda(np.ones(128, np.float32)),
                        cuda(lay.coeff), cuda(lay.loss), 1, variant="dsv4")
    got = host(oi)
    assert got[0, 0] == 1000
    ew, ei = O.decode_dsv4(np.ones_like(rw), ri2, np.ones(128, np.float32), lay.coeff, lay.loss, 1)
    np.testing.assert_array_equal(got, ei)
    np.testing.assert_array_equal(host(ow), ew)


@pytest.mark.parametrize("variant", ["qwen3", "dsv4"])
def test_decode_nan_and_huge_products(variant):
    """A NaN product counts 0 and products are clamped to 2^24 in the importance, as in the
    oracle; the fused decode, the importance pass and the split decode agree with it."""
    lay = W.layer("qwen3_decode", tokens=64)
    rw, ri = O.router_topk(lay.logits, 8, "softmax")
    w = rw.copy()
    w[0, 0] = np.nan
    w[1, 1] = 1e30
    w[2, :] = np.inf
    w[3, 2] = 3.0e7  # above the clamp
    coeff, loss = (lay.coeff, lay.loss) if variant == "qwen3" else dsv4_tables(lay)
    ow, oi = ops.decode(cuda(w), cuda(ri), cuda(lay.norms), cuda(coeff), cuda(loss), 16,
                        variant=variant)
    if variant == "qwen3":
        ew, ei, _ = O.decode_qwen3(w, ri, lay.norms, coeff, loss, 16)
    else:
        ew, ei = O.decode_dsv4(w, ri, lay.norms, coeff, loss, 16)
    np.testing.assert_array_equal(host(oi), ei)
    np.testing.assert_array_equal(host(ow), ew)
    imp = torch.zeros(128, dtype=torch.int64, device=DEV)
    ops.decode_importance(cuda(w), cuda(ri), cuda(lay.norms), imp)
    np.testing.assert_array_equal(host(imp), O.importance(w, ri, lay.norms))
    sw, si = ops.decode_apply(imp, cuda(w), cuda(ri), cuda(coeff), cuda(loss), 16,
                              variant=variant)
    np.testing.assert_array_equal(host(si), ei)
    np.testing.assert_array_equal(host(sw), ew)


def test_sharded_exchange_single_rank_equals_decode():
    """The one-launch sharded decode with one rank (its own buffer as the only peer) equals the
    plain decode, over consecutive calls (the call counter advances) and in a replayed graph."""
    from exfold_b200.parallel import DecodeExchange

    xch = DecodeExchange(128, device=DEV)
    layers = [W.layer("qwen3_decode", layer_index=i) for i in range(3)]
    cases = []
    for lay in layers:
        rw, ri = O.router_topk(lay.logits, 8, "softmax")
        cases.append(tuple(cuda(a) for a in (rw, ri, lay.norms, lay.coeff, lay.loss)))
    for variant in ("qwen3", "dsv4"):
        for w, i, n, c, l_ in cases:
            gw, gi = xch.decode(w, i, n, c, l_, 64, variant=variant)
            ew, ei = ops.decode(w, i, n, c, l_, 64, variant=variant)
            assert torch.equal(gi, ei) and torch.equal(gw, ew)
    s = torch.cuda.Stream(DEV)
    outs = []
    with torch.cuda.stream(s):
        xch.decode(*cases[0], 64)
        torch.cuda.synchronize(DEV)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for case in cases:
                outs.append(xch.decode(*case, 64))
        for _ in range(3):
            g.replay()
    torch.cuda.synchronize(DEV)
    for (gw, gi), case in zip(outs, cases):
        ew, ei = ops.decode(*case, 64)
        assert torch.equal(gi, ei) and torch.equal(gw, ew)
    assert int(xch.status.item()) == 0
    assert int(xch.buffer[0].item()) == 6 + 1 + 3 * 3  # calls made on the buffer


def test_sharded_exchange_missing_rank_times_out_with_status():
    """Failure detection without a fault: rank 0 of two, the second rank's buffer a local one that
    no kernel ever publishes to.  The bounded wait (2 ms here) runs out, the status is set, and the
    result is the decode with this rank's importance alone; the context stays usable."""
    import ctypes

    from exfold_b200 import _lib as L

    nbytes = int(L.lib().exf_decode_exchange_bytes(128, 2))
    bufs = [torch.zeros(nbytes // 8, dtype=torch.int64, device=DEV) for _ in range(2)]
    peers = (ctypes.c_void_p * 2)(bufs[0].data_ptr(), bufs[1].data_ptr())
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    lay = W.layer("qwen3_decode")
    rw, ri = O.router_topk(lay.logits, 8, "softmax")
    w, i, n, c, l_ = (cuda(a) for a in (rw, ri, lay.norms, lay.coeff, lay.loss))
    for call in (1, 2):
        gw, gi = ops.decode_sharded(w, i, n, c, l_, 64, world=2, rank=0, peers=peers,
                                    status=status, wait_ns=2_000_000)
        ew, ei = ops.decode(w, i, n, c, l_, 64)
        torch.cuda.synchronize(DEV)
        assert int(status.item()) == 1
        assert torch.equal(gi, ei) and torch.equal(gw, ew)
        assert int(bufs[0][0].item()) == call
        # the words this rank published to its peer's slot (parity call & 1, rank 0) carry call
        word = int(bufs[1][16 + (call & 1) * 2 * 128 * 2].item())
        assert word >> 32 == call
    # the context is intact
    assert torch.equal(ops.decode(w, i, n, c, l_, 64)[1], ei)
