"""Benchmark of the ExFold routing transform on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Default workload (the 48-layer sharded run): each GPU routes and folds T = 131072 tokens per
layer through 48 Qwen3-shaped MoE layers (E = 128, top-8, keep P = 4, independent per-layer
calibration tables), so per-GPU work is fixed as N grows (weak scaling; prefill needs no
communication).  One step = 48 launches of the fused router + prefill-fold kernel, one per layer
as a model calls it, replayed from a CUDA graph.  The 3.2 GB of logits per step are larger than
L2, so no flush is needed between steps.  Rank 0 prints one JSON line.

--impl reference runs the reference's CPU path for the same metric: the CPU oracle (a scalar C
port of exfold/qwen3/kernels.py with the softmax/top-k router) on all host threads over a
bounded sample of the same workload; under torchrun only rank 0 works.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "exfold-moe_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402

LAYERS, TOKENS, EXPERTS, TOP_K, KEEP = 48, 131072, 128, 8, 4


def bytes_per_launch(tokens: int) -> int:
    """Algorithmic HBM bytes of one router + fold launch: logits in, P ids + P weights out, and
    the coefficient and loss tables once."""
    return tokens * (EXPERTS * 4 + KEEP * 8) + 2 * EXPERTS * EXPERTS * 4


def set_shape(layers: int, tokens: int) -> None:
    global LAYERS, TOKENS
    LAYERS, TOKENS = layers, tokens


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        d = json.loads(path.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def profiled_traffic(name: str):
    path = ROOT / "profiles" / "traffic.json"
    if path.is_file():
        return json.loads(path.read_text()).get(name)
    return None


# ---- clocks sampled during the timed region (NVML; read-only) ---------------------------------
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
            0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
            0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, device_index: int):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self._nv = pynvml
            try:
                p = torch.cuda.get_device_properties(device_index)
                bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
                self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:  # noqa: BLE001
                self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self._reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self._h = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = self._reasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._h is not None:
            self._stop.set()
            self._t.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        bits = 0
        for _, r in self.samples:
            bits |= r
        names = [n for b, n in _REASONS.items() if bits & b and b != 0x1]
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


# ---- workload ---------------------------------------------------------------------------------
def qwen3_tables(layers: int):
    """Per-layer calibration tables, prepared as exfold/qwen3/vllm_patch.py:59-61 prepares them."""
    from exfold_b200 import calibration
    from exfold_b200 import workloads as W

    cfg = W.WORKLOADS["qwen3_layers"]
    coeff, loss, norms = [], [], []
    for layer in range(layers):
        seed = cfg["seed"] + layer
        coeff.append(W.coefficient(seed, EXPERTS, 0.35, 0.15))
        loss.append(W.loss_matrix(seed, EXPERTS, 0.2, 1.0))
        norms.append(W.expert_norms(seed, EXPERTS))
    # the synthetic loss has a +inf diagonal, which the artifact check would reject
    return calibration.prepare_qwen3(np.stack(coeff), np.stack(loss), np.stack(norms),
                                     validate=False)


def cpu_oracle_rate(logits: np.ndarray, coeff: np.ndarray, loss: np.ndarray, threads: int,
                    budget_s: float) -> tuple[float, int]:
    """Tokens/s of the CPU oracle (router + fold) on `threads` host threads; ctypes releases the
    GIL, so threads run the C code in parallel.  Repeats the sample until budget_s is spent."""
    from oracle import oracle as O

    chunks = np.array_split(np.arange(logits.shape[0]), threads)

    def work(idx):
        O.router_fold(logits[idx], TOP_K, KEEP, coeff, loss)

    done = 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        while True:
            list(ex.map(work, chunks))
            done += logits.shape[0]
            if time.perf_counter() - t0 >= budget_s:
                break
    return done / (time.perf_counter() - t0), done


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from exfold_b200 import workloads as W

    threads = len(os.sched_getaffinity(0))
    coeff, loss, _ = qwen3_tables(1)
    sample = W.logits(W.WORKLOADS["qwen3_layers"]["seed"], 16384, EXPERTS)
    rate, _ = cpu_oracle_rate(sample, coeff[0], loss[0], threads, 1.0)  # warm-up
    # whole run bounded to ~2 minutes: at most 0.25 s of CPU work per step
    step_s = min(0.25, 120.0 / (args.steps + args.warmup))
    step_tokens = max(threads * 64, int(rate * step_s))
    step_tokens = min(step_tokens, sample.shape[0])
    sample = sample[:step_tokens]
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        cpu_oracle_rate(sample, coeff[0], loss[0], threads, 0.0)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    total = sum(times)
    value = step_tokens * len(times) / total
    line = {
        "metric": "fold-transform tokens/s (router + prefill fold, 48 layers, T=131072/GPU, P=4)",
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
        "data": "synthetic (seeded N(0,1) logits, seeded calibration tables)",
        "config": {"workload": "qwen3_layers_prefill", "layers": LAYERS, "tokens_per_gpu": TOKENS,
                   "experts": EXPERTS, "top_k": TOP_K, "keep": KEEP,
                   "sample_tokens_per_step": step_tokens},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{step_tokens} tokens of layer 0 per step, split over "
                                   f"{threads} threads"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- decode half of the 48-layer workload -----------------------------------------------------
DECODE_BATCH, DECODE_BUDGET = 1024, 64


def measure_decode(dev, world, rank, stream, coeff, loss, timed, args) -> dict:
    """Decode budget over all layers for a B=1024 batch split over the ranks: per layer one
    fixed-point importance launch, one int64 all-reduce of E values, one select/apply launch
    (a single fused launch on one GPU).  Replayed from a CUDA graph; microseconds per layer."""
    import torch
    import torch.distributed as dist

    from exfold_b200 import ops, parallel

    start, end = parallel.shard_range(DECODE_BATCH, world, rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(7000)
    logits = torch.randn((LAYERS, DECODE_BATCH, EXPERTS), generator=gen, device=dev)
    norms = torch.exp(0.5 * torch.randn((LAYERS, EXPERTS), generator=gen, device=dev))
    w = torch.empty((LAYERS, end - start, TOP_K), device=dev)
    ids = torch.empty((LAYERS, end - start, TOP_K), dtype=torch.int32, device=dev)
    for layer in range(LAYERS):
        lw, li = ops.router_topk(logits[layer, start:end].contiguous(), TOP_K)
        w[layer].copy_(lw)
        ids[layer].copy_(li)
    imp = torch.zeros((LAYERS, EXPERTS), dtype=torch.int64, device=dev)

    def step():
        for layer in range(LAYERS):
            if world == 1:
                ops.decode(w[layer], ids[layer], norms[layer], coeff[layer], loss[layer],
                           DECODE_BUDGET, variant="qwen3")
            else:
                imp[layer].zero_()
                ops.decode_importance(w[layer], ids[layer], norms[layer], imp[layer])
                dist.all_reduce(imp[layer])
                ops.decode_apply(imp[layer], w[layer], ids[layer], coeff[layer], loss[layer],
                                 DECODE_BUDGET, variant="qwen3")

    step()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    steps = max(10, args.steps // 10)
    ms = timed(graph.replay, steps) / steps
    del graph
    return {"workload": "qwen3_layers_decode", "batch": DECODE_BATCH, "batch_per_gpu": end - start,
            "budget": DECODE_BUDGET, "layers": LAYERS, "us_per_layer": 1e3 * ms / LAYERS,
            "launches_per_layer": 1 if world == 1 else 3,
            "collective": None if world == 1 else "all_reduce int64[128] per layer (NCCL)"}


# ---- our arm --------------------------------------------------------------------------------
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from exfold_b200 import ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    coeff_np, loss_np, _ = qwen3_tables(LAYERS)
    coeff = torch.from_numpy(coeff_np).to(dev)
    loss = torch.from_numpy(loss_np).to(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4000 + 7919 * rank)
    logits = torch.randn((LAYERS, TOKENS, EXPERTS), generator=gen, device=dev)
    out_w = torch.empty((LAYERS, TOKENS, KEEP), dtype=torch.float32, device=dev)
    out_ids = torch.empty((LAYERS, TOKENS, KEEP), dtype=torch.int32, device=dev)

    def step():
        for layer in range(LAYERS):
            ops.router_fold_prefill(logits[layer], TOP_K, KEEP, coeff[layer], loss[layer],
                                    out=(out_w[layer], out_ids[layer]))

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        step()  # eager warm-up (grid sizing queries happen outside capture)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            fn()
        end.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        ms = start.elapsed_time(end)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with torch.cuda.stream(stream):
        with ClockSampler(local) as clocks:
            ms = timed(graph.replay, args.steps)
    ms_per_step = ms / args.steps
    tokens_per_step = LAYERS * TOKENS * world
    value = tokens_per_step / (ms_per_step / 1e3)
    launch_s = ms_per_step / 1e3 / LAYERS
    peaks = measured_peaks()
    achieved = bytes_per_launch(TOKENS) / launch_s / 1e9

    # layer-batched variant: one launch over all 48 layers
    def batched():
        ops.router_fold_prefill(logits, TOP_K, KEEP, coeff, loss, out=(out_w, out_ids))

    with torch.cuda.stream(stream):
        batched()
        torch.cuda.synchronize(dev)
        gb = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gb, stream=stream):
            batched()
        ms_b = timed(gb.replay, max(1, args.steps // 4)) / max(1, args.steps // 4)

    # end to end through the public API: pinned host logits in, pinned host results out
    slots = min(4, LAYERS)
    host_in = torch.empty((slots, TOKENS, EXPERTS), dtype=torch.float32).pin_memory()
    host_in.copy_(logits[:slots].cpu())
    host_w = torch.empty((slots, TOKENS, KEEP), dtype=torch.float32).pin_memory()
    host_i = torch.empty((slots, TOKENS, KEEP), dtype=torch.int32).pin_memory()
    dev_in = torch.empty((2, TOKENS, EXPERTS), dtype=torch.float32, device=dev)
    dev_w = torch.empty((2, TOKENS, KEEP), dtype=torch.float32, device=dev)
    dev_i = torch.empty((2, TOKENS, KEEP), dtype=torch.int32, device=dev)
    # Host->device copies, the router calls and device->host copies on three streams, double
    # buffered, so that layer l's results go back while layer l+1's logits come in (PCIe runs
    # both directions at once).  Every copy of the step stays inside the timed region.
    copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]    # logits of buffer b are on the device
    ev_done = [torch.cuda.Event() for _ in range(2)]  # the call reading buffer b has finished
    ev_back = [torch.cuda.Event() for _ in range(2)]  # results of buffer b are on the host

    def e2e_step():
        copy_in.wait_stream(stream)
        for layer in range(LAYERS):
            b = layer % 2
            copy_in.wait_event(ev_done[b])
            with torch.cuda.stream(copy_in):
                dev_in[b].copy_(host_in[layer % slots], non_blocking=True)
            ev_in[b].record(copy_in)
            stream.wait_event(ev_in[b])
            stream.wait_event(ev_back[b])
            ops.router_fold_prefill(dev_in[b], TOP_K, KEEP, coeff[layer], loss[layer],
                                    out=(dev_w[b], dev_i[b]))
            ev_done[b].record(stream)
            copy_out.wait_event(ev_done[b])
            with torch.cuda.stream(copy_out):
                host_w[layer % slots].copy_(dev_w[b], non_blocking=True)
                host_i[layer % slots].copy_(dev_i[b], non_blocking=True)
            ev_back[b].record(copy_out)
        stream.wait_stream(copy_out)

    e2e_steps = max(2, min(10, args.steps // 100))
    saved_warmup = args.warmup
    args.warmup = 1
    with torch.cuda.stream(stream):
        ms_e2e = timed(e2e_step, e2e_steps) / e2e_steps
    args.warmup = saved_warmup
    h2d = LAYERS * TOKENS * EXPERTS * 4
    d2h = LAYERS * TOKENS * KEEP * 8

    with torch.cuda.stream(stream):
        decode = measure_decode(dev, world, rank, stream, coeff, loss, timed, args)

    cpu = None
    if rank == 0 and world == 1:
        sample = logits[0, :8192].cpu().numpy()
        rate, done = cpu_oracle_rate(sample, coeff_np[0], loss_np[0], 1, 10.0)
        cpu = {"value": rate, "unit": "tokens/s", "cores": 1, "kind": "port",
               "sample": f"{done} tokens (8192-token slices of layer 0), single thread, ~10 s"}

    if rank == 0:
        line = {
            "metric": "fold-transform tokens/s (router + prefill fold, 48 layers, T=131072/GPU, P=4)",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) logits, seeded calibration tables)",
            "config": {"workload": "qwen3_layers_prefill", "layers": LAYERS,
                       "tokens_per_gpu": TOKENS, "experts": EXPERTS, "top_k": TOP_K,
                       "keep": KEEP, "parallelism": f"token-sharded x{world}",
                       "l2": "inputs 3.2 GB/step per GPU > L2, no flush"},
            "gpu_launches": LAYERS * args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                         "traffic": profiled_traffic("router_fold_qwen3_layer"),
                         "peak_source": peaks["source"],
                         "kernel": "exf::router_tpt_kernel<qwen3 fold, P=4>",
                         "bytes_per_launch": bytes_per_launch(TOKENS),
                         "us_per_launch": launch_s * 1e6},
            "layer_batched": {"ms_per_step": ms_b, "tokens_per_s": tokens_per_step / (ms_b / 1e3),
                              "launches_per_step": 1},
            "e2e": {"value": tokens_per_step / (ms_e2e / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": ms_e2e},
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "decode": decode,
        }
        print(json.dumps(line), flush=True)
    del graph, gb
    if world > 1:
        dist.destroy_process_group()


# ---- additional single-GPU workloads (--workload NAME): one JSON line each --------------------
def _timed_graph(fn, steps: int, warmup: int, dev) -> float:
    """ms per call of fn, replayed from a CUDA graph, CUDA events on the capture stream."""
    import torch

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        fn()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            fn()
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize(dev)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
        torch.cuda.synchronize(dev)
    ms = start.elapsed_time(end) / steps
    del graph
    return ms


def run_extra(args) -> None:
    import torch

    from exfold_b200 import ops
    from exfold_b200 import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (
        ROOT / "MEASURED_PEAKS.json").is_file() else {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    steps = max(5, min(args.steps, 200))
    out = {"workload": args.workload}
    if args.workload in ("moe_dsv4_prefill", "moe_qwen3_decode"):
        if args.workload == "moe_dsv4_prefill":
            # --tokens / --experts shrink the case for profiling (defaults: the full workload)
            lay = W.layer("dsv4_prefill", tokens=args.tokens)
            tokens, experts, hidden, inter = lay.tokens, 256, 4096, 2048
            coeff, loss = lay.coeff.copy(), lay.loss.copy()
            np.fill_diagonal(coeff, 1.0)
            np.fill_diagonal(loss, 1e30)
            conf = loss.copy()
            np.fill_diagonal(conf, 0.0)
            w, ids = ops.router_fold_prefill(
                torch.from_numpy(lay.logits).to(dev), 8, 3, torch.from_numpy(coeff).to(dev),
                torch.from_numpy(loss).to(dev), scoring="sigmoid",
                bias=torch.from_numpy(lay.bias).to(dev), variant="dsv4", renorm_mode=2,
                conf_loss=torch.from_numpy(conf).to(dev))
        else:
            lay = W.layer("qwen3_decode")
            tokens, experts, hidden, inter = lay.tokens, 128, 2048, 768
            rw, ri = ops.router_topk(torch.from_numpy(lay.logits).to(dev), 8)
            w, ids = ops.decode(rw, ri, torch.from_numpy(lay.norms).to(dev),
                                torch.from_numpy(lay.coeff).to(dev),
                                torch.from_numpy(lay.loss).to(dev), 64, variant="qwen3")
        if args.experts and args.experts < experts:  # profiling: fold the routes onto fewer experts
            ids = (ids % args.experts).to(ids.dtype)
            experts = args.experts
        x = torch.randn(tokens, hidden, generator=gen, device=dev).to(torch.bfloat16)
        w13 = torch.empty(experts, 2 * inter, hidden, dtype=torch.bfloat16, device=dev)
        w2 = torch.empty(experts, hidden, inter, dtype=torch.bfloat16, device=dev)
        for e in range(experts):  # N(0, 0.02) weights, generated per expert to bound memory
            w13[e] = (0.02 * torch.randn(2 * inter, hidden, generator=gen, device=dev))
            w2[e] = (0.02 * torch.randn(hidden, inter, generator=gen, device=dev))
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        ms = _timed_graph(lambda: ops.fused_experts(x, w, ids, w13, w2, status=status), steps,
                          max(3, args.warmup), dev)
        numel = ids.numel()
        active = int(torch.unique(ids).numel())
        flops = 6.0 * numel * hidden * inter
        wbytes = active * 3.0 * hidden * inter * 2
        out.update(tokens=tokens, routes=numel, active_experts=active, hidden=hidden, inter=inter,
                   ms_per_layer=ms, tflops=flops / ms / 1e9,
                   tensor_frac_of_measured_peak=flops / ms / 1e9 / peaks["bf16_tflops"],
                   weight_gbs=wbytes / ms / 1e6,
                   hbm_frac_of_measured_peak=wbytes / ms / 1e6 / peaks["hbm_gbs"],
                   status=int(status.item()), launches=7)
        if args.workload == "moe_qwen3_decode" and not args.experts:
            # the decode budget and the expert layer: two calls, and the fused entry (moe_align
            # inside the decode launch, duplicate (token, expert) routes merged)
            n, c, l_ = (torch.from_numpy(a).to(dev) for a in (lay.norms, lay.coeff, lay.loss))

            def two_calls():
                dw, di = ops.decode(rw, ri, n, c, l_, 64, variant="qwen3")
                ops.fused_experts(x, dw, di, w13, w2, status=status)

            def fused():
                ops.decode_fused_experts(x, rw, ri, n, c, l_, 64, w13, w2, variant="qwen3",
                                         status=status)

            ms_two = _timed_graph(two_calls, steps, max(3, args.warmup), dev)
            ms_fused = _timed_graph(fused, steps, max(3, args.warmup), dev)
            merged = int((ids.sort(dim=1).values.diff(dim=1) == 0).sum().item())
            out["decode_layer"] = {"us_decode_then_experts": ms_two * 1e3,
                                   "us_decode_fused_experts": ms_fused * 1e3,
                                   "merged_routes": merged, "status": int(status.item())}
    elif args.workload == "dsv4_prefill_fold":
        lay = W.layer("dsv4_prefill")
        coeff, loss = lay.coeff.copy(), lay.loss.copy()
        np.fill_diagonal(coeff, 1.0)
        np.fill_diagonal(loss, 1e30)
        conf = loss.copy()
        np.fill_diagonal(conf, 0.0)
        xs = torch.from_numpy(lay.logits).to(dev)
        c, l_, cf = (torch.from_numpy(a).to(dev) for a in (coeff, loss, conf))
        b = torch.from_numpy(lay.bias).to(dev)
        ow = torch.empty((lay.tokens, 3), device=dev)
        oi = torch.empty((lay.tokens, 3), dtype=torch.int32, device=dev)
        ms = _timed_graph(lambda: ops.router_fold_prefill(
            xs, 8, 3, c, l_, scoring="sigmoid", bias=b, variant="dsv4", renorm_mode=2,
            conf_loss=cf, out=(ow, oi)), steps, max(3, args.warmup), dev)
        nbytes = lay.tokens * (256 * 4 + 3 * 8) + 3 * 256 * 256 * 4 + 256 * 4
        out.update(tokens=lay.tokens, us_per_launch=ms * 1e3, tokens_per_s=lay.tokens / ms * 1e3,
                   gbs=nbytes / ms / 1e6, hbm_frac_of_measured_peak=nbytes / ms / 1e6 / peaks["hbm_gbs"])
    elif args.workload == "calibration_update":
        # PairwiseScalarStats.update (exfold/qwen3/calibration.py:49-95) at the Qwen3 layer shape:
        # 8 routes of 2048-wide bf16 expert outputs over 128 experts, 16384 tokens per call
        # (512 MiB of outputs > L2); the pass is bound by reading the outputs.
        from exfold_b200.calibration import PairwiseScalarStats

        T, K, H, E = (args.tokens or 16384), 8, 2048, 128
        outs = torch.randn((T, K, H), generator=gen, device=dev).to(torch.bfloat16)
        ids = torch.randint(0, E, (T, K), generator=gen, device=dev, dtype=torch.int32)
        stats = PairwiseScalarStats(E, device=dev)
        ms = _timed_graph(lambda: stats.update(ids, outs), steps, max(3, args.warmup), dev)
        nbytes = T * K * H * 2 + T * K * 4
        out.update(tokens=T, top_k=K, hidden=H, experts=E, us_per_call=ms * 1e3,
                   tokens_per_s=T / ms * 1e3, gbs=nbytes / ms / 1e6,
                   hbm_frac_of_measured_peak=nbytes / ms / 1e6 / peaks["hbm_gbs"])
    elif args.workload == "dsv4_decode":
        cfg = W.WORKLOADS["dsv4_decode"]
        rows = []
        for batch in cfg["batches"]:
            lay = W.Layer(seed=cfg["seed"], tokens=batch, experts=256, top_k=8, kind="dsv4")
            coeff, loss = lay.coeff.copy(), lay.loss.copy()
            np.fill_diagonal(coeff, 1.0)
            np.fill_diagonal(loss, 1e30)
            xs = torch.from_numpy(lay.logits).to(dev)
            b = torch.from_numpy(lay.bias).to(dev)
            c, l_, n = (torch.from_numpy(a).to(dev) for a in (coeff, loss, lay.norms))
            for budget in cfg["budgets"]:
                def step():
                    rw, ri = ops.router_topk(xs, 8, "sigmoid", b)
                    ops.decode(rw, ri, n, c, l_, budget, variant="dsv4")
                ms = _timed_graph(step, steps, max(3, args.warmup), dev)
                rows.append({"batch": batch, "budget": budget, "us_router_plus_decode": ms * 1e3})
        out["sweep"] = rows
    print(json.dumps(out), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=LAYERS, help="smaller cases for profiling")
    ap.add_argument("--tokens", type=int, default=None, help="smaller cases for profiling")
    ap.add_argument("--experts", type=int, default=0, help="fewer experts (profiling cases)")
    ap.add_argument("--workload", default="qwen3_layers",
                    choices=["qwen3_layers", "moe_dsv4_prefill", "moe_qwen3_decode",
                             "dsv4_prefill_fold", "dsv4_decode", "calibration_update"])
    args = ap.parse_args()
    set_shape(args.layers, args.tokens or TOKENS)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload != "qwen3_layers":
        run_extra(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
