"""Benchmark of the ExFold routing transform on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Headline (the 48-layer sharded run): each GPU routes and folds T = 131072 tokens per layer
through 48 Qwen3-shaped MoE layers (E = 128, top-8, keep P = 4, independent per-layer
calibration tables), so per-GPU work is fixed as N grows (weak scaling; prefill needs no
communication).  One step = 48 launches of the fused router + prefill-fold kernel, one per layer
as a model calls it, replayed from a CUDA graph.  The 3.2 GB of logits per step are larger than
L2, so no flush is needed between steps.  `value` counts token-layers per second (tokens routed
through one layer; a forward pass over all 48 layers is `value` / 48 tokens per second).

The same line carries the rest of the metric "fold-transform tokens/s & MoE-layer us":
* `decode`: the decode budget of the 48-layer run (B = 1024 batch-sharded, D = 64; at N > 1 one
  launch per layer exchanges the int64 importance with the other ranks over NVLink peer memory,
  and the NCCL all-reduce path is timed beside it), with `decode_parity` at N > 1 (each rank's
  sharded results, both paths, equal the single-GPU decode of the whole batch);
* `configs` (N = 1): the single-layer configurations -- config 0 (Qwen3 prefill fold, T = 4096),
  config 1 (Qwen3 decode transform and expert layer, B = 256, D = 64, H = 2048, I = 768),
  config 2 (DeepSeek-style fold, T = 65536, P = 3, E = 256, and its expert layer, H = 4096,
  I = 2048), config 3 (DeepSeek-style decode sweep, B in {8, 32, 128, 512} x D in {64, 128},
  transform and expert layer).  Inputs that fit in L2 are timed one launch at a time with L2
  flushed (a 512 MiB write) between launches, outside the timed events;
* `bf16_logits`: the headline step on bf16 logits (read natively, converted exactly);
* `cpu_baseline`: the CPU oracle on every host core over a bounded sample of the 48 layers.

--impl reference runs the reference's CPU path for the same metric and config: the CPU oracle (a
scalar C port of the reference's fold kernels with the softmax/top-k router) on all host threads,
each step all 48 layers' tables over T tokens per layer (T = 131072 unless the run would exceed
about two and a half minutes, then fewer, stated); under torchrun only rank 0 works.
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
METRIC = "fold-transform token-layers/s (router + prefill fold, 48 layers, T=131072/GPU, P=4)"
UNIT = "token-layers/s"


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
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def profiled_traffic(name: str):
    path = ROOT / "profiles" / "traffic.json"
    if path.is_file():
        return json.loads(path.read_text()).get(name)
    return None


# ---- clocks sampled during the timed regions (NVML; read-only) ------------------------------
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
            0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
            0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self.period_s = period_s
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
            time.sleep(self.period_s)

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


def host_threads() -> int:
    return len(os.sched_getaffinity(0))


def cpu_layers_pass(pool: ThreadPoolExecutor, threads: int, logits: list, coeff, loss) -> int:
    """One pass of the CPU oracle's router + Qwen3 fold over layers 0..len(logits)-1 (layer l:
    logits[l] with tables coeff[l], loss[l]), each layer's tokens split over `threads` host
    threads (ctypes releases the GIL, so the C code runs in parallel).  Returns token-layers."""
    from oracle import oracle as O

    def work(job):
        x, c, l_ = job
        O.router_fold(x, TOP_K, KEEP, c, l_)

    jobs = []
    for layer, x in enumerate(logits):
        bounds = np.linspace(0, x.shape[0], threads + 1).astype(int)
        jobs += [(x[a:b], coeff[layer], loss[layer]) for a, b in zip(bounds[:-1], bounds[1:])
                 if b > a]
    list(pool.map(work, jobs))
    return sum(x.shape[0] for x in logits)


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from exfold_b200 import workloads as W

    threads = host_threads()
    coeff, loss, _ = qwen3_tables(LAYERS)
    full = W.logits(W.WORKLOADS["qwen3_layers"]["seed"], TOKENS, EXPERTS)
    with ThreadPoolExecutor(max_workers=threads) as pool:
        # calibrate on 4096 tokens of every layer, then size the step so that the whole run
        # stays within about 150 s
        t0 = time.perf_counter()
        done = cpu_layers_pass(pool, threads, [full[:4096]] * LAYERS, coeff, loss)
        rate = done / (time.perf_counter() - t0)
        budget_s = 150.0 / (args.steps + args.warmup)
        tokens = int(min(TOKENS, max(threads * 16, rate * budget_s / LAYERS)))
        step_logits = [full[:tokens]] * LAYERS
        times = []
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            cpu_layers_pass(pool, threads, step_logits, coeff, loss)
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
    total = sum(times)
    value = tokens * LAYERS * len(times) / total
    sample = (f"{tokens} tokens x all {LAYERS} layers' tables per step (the full workload is "
              f"{TOKENS} tokens per layer), one seeded {TOKENS}-token logit matrix shared by "
              f"the layers, split over {threads} threads")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
        "data": "synthetic (seeded N(0,1) logits, seeded calibration tables)",
        "config": {"workload": "qwen3_layers_prefill", "layers": LAYERS, "tokens_per_gpu": TOKENS,
                   "experts": EXPERTS, "top_k": TOP_K, "keep": KEEP,
                   "sample_tokens_per_layer": tokens, "same_config": tokens == TOKENS},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- timing helpers --------------------------------------------------------------------------
class Timer:
    """CUDA-event timing on one stream: `graph(fn)` captures fn into a CUDA graph; `replays`
    times back-to-back replays (inputs larger than L2); `flushed` times single replays with L2
    flushed between them (a 512 MiB write outside the timed events) for inputs that fit in L2."""

    def __init__(self, dev, stream, warmup: int):
        import torch

        self.torch, self.dev, self.stream, self.warmup = torch, dev, stream, warmup
        self._flush = None

    def graph(self, fn):
        torch = self.torch
        with torch.cuda.stream(self.stream):
            fn()
            torch.cuda.synchronize(self.dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                fn()
        return g

    def replays(self, fn, steps: int) -> float:
        """ms per call, `steps` back-to-back graph replays."""
        torch = self.torch
        g = self.graph(fn)
        with torch.cuda.stream(self.stream):
            for _ in range(self.warmup):
                g.replay()
            torch.cuda.synchronize(self.dev)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(self.stream)
            for _ in range(steps):
                g.replay()
            b.record(self.stream)
            torch.cuda.synchronize(self.dev)
        del g
        return a.elapsed_time(b) / steps

    def flushed(self, fn, steps: int) -> float:
        """median ms of single graph replays, L2 flushed before each (outside the events)."""
        torch = self.torch
        if self._flush is None:
            self._flush = torch.empty(1 << 29, dtype=torch.uint8, device=self.dev)
        g = self.graph(fn)
        times = []
        with torch.cuda.stream(self.stream):
            for i in range(self.warmup + steps):
                self._flush.fill_(i & 0xFF)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(self.stream)
                g.replay()
                b.record(self.stream)
                b.synchronize()
                if i >= self.warmup:
                    times.append(a.elapsed_time(b))
        del g
        return statistics.median(times)


# ---- decode half of the 48-layer workload -----------------------------------------------------
DECODE_BATCH, DECODE_BUDGET = 1024, 64


def measure_decode(dev, world, rank, stream, coeff, loss, timed, args) -> dict:
    """Decode budget over all layers for a B=1024 batch split over the ranks, replayed from a
    CUDA graph; microseconds per layer.  One GPU: one fused launch per layer.  N > 1: one launch
    per layer that exchanges the fixed-point importance with the other ranks over NVLink peer
    memory (`DecodeExchange`); the three-step path (importance launch, NCCL all-reduce of E
    int64, apply launch) is timed beside it.  Each rank's results of every layer, both paths,
    are compared with the single-GPU decode of the whole batch (every rank generates the whole
    batch from the same seed)."""
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
    xch, xch_error = None, None
    if world > 1:
        try:
            xch = parallel.DecodeExchange(EXPERTS, device=dev)
        except RuntimeError as exc:  # every rank sees the same outcome
            xch_error = str(exc)

    def step(outs: list, how: str):
        for layer in range(LAYERS):
            args_ = (w[layer], ids[layer], norms[layer], coeff[layer], loss[layer], DECODE_BUDGET)
            if world == 1:
                dw, di = ops.decode(*args_, variant="qwen3")
            elif how == "exchange":
                dw, di = xch.decode(*args_, variant="qwen3")
            else:
                imp[layer].zero_()
                ops.decode_importance(w[layer], ids[layer], norms[layer], imp[layer])
                dist.all_reduce(imp[layer])
                dw, di = ops.decode_apply(imp[layer], w[layer], ids[layer], coeff[layer],
                                          loss[layer], DECODE_BUDGET, variant="qwen3")
            outs.append((dw, di))

    def capture(how: str):
        step([], how)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        results: list = []  # the graph's output tensors: each replay rewrites them
        with torch.cuda.graph(graph, stream=stream):
            step(results, how)
        return graph, results

    steps = max(10, args.steps // 10)
    main = "all_reduce" if xch_error else "exchange"
    graph, results = capture(main)
    ms = timed(graph.replay, steps) / steps
    out = {"workload": "qwen3_layers_decode", "batch": DECODE_BATCH,
           "batch_per_gpu": end - start, "budget": DECODE_BUDGET, "layers": LAYERS,
           "us_per_layer": 1e3 * ms / LAYERS, "scaling": "strong (B fixed)",
           "launches_per_layer": 2 if xch_error else 1,
           "collective": None if world == 1 else (
               "NCCL all_reduce int64[128] per layer" if xch_error else
               "in-launch exchange of int64[128] over NVLink peer memory (CUDA IPC)")}
    if xch_error:
        out["exchange_unavailable"] = xch_error
    if world > 1:
        runs = {main: (graph, results)}
        graph_nccl, results_nccl = None, None
        if not xch_error:
            graph_nccl, results_nccl = capture("all_reduce")
            ms_nccl = timed(graph_nccl.replay, steps) / steps
            runs["all_reduce"] = (graph_nccl, results_nccl)
            out["all_reduce_path"] = {"us_per_layer": 1e3 * ms_nccl / LAYERS,
                                      "launches_per_layer": 2,
                                      "collective": "NCCL all_reduce int64[128] per layer"}
        same = True
        with torch.cuda.stream(stream):
            refs = []
            for layer in range(LAYERS):
                fw, fi = ops.router_topk(logits[layer], TOP_K)
                ew, ei = ops.decode(fw, fi, norms[layer], coeff[layer], loss[layer],
                                    DECODE_BUDGET, variant="qwen3")
                refs.append((ew[start:end], ei[start:end]))
            for g, res in runs.values():
                g.replay()
                for (gw, gi), (ew, ei) in zip(res, refs):
                    same = same and bool(torch.equal(ei, gi)) and bool(torch.equal(ew, gw))
        same = same and (xch is None or int(xch.status.item()) == 0)
        flag = torch.tensor([1 if same else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        out["decode_parity"] = bool(flag.item())
        del runs, graph_nccl, results_nccl
        torch.cuda.synchronize(dev)
        dist.barrier()
        if xch is not None:
            xch.close()
    del graph, results
    return out


# ---- the single-layer configurations (N = 1) --------------------------------------------------
def _dsv4_tables(lay, dev):
    import torch

    coeff, loss = lay.coeff.copy(), lay.loss.copy()
    np.fill_diagonal(coeff, 1.0)
    np.fill_diagonal(loss, 1e30)
    conf = loss.copy()
    np.fill_diagonal(conf, 0.0)
    return tuple(torch.from_numpy(a).to(dev) for a in (coeff, loss, conf))


def _qwen3_tables(lay, dev):
    import torch

    from exfold_b200 import calibration

    c, l_, n = calibration.prepare_qwen3(lay.coeff[None], lay.loss[None], lay.norms[None],
                                         validate=False)
    return tuple(torch.from_numpy(np.ascontiguousarray(a[0])).to(dev) for a in (c, l_, n))


def _expert_weights(experts, hidden, inter, seed, dev):
    """bf16 SwiGLU expert weights ~ N(0, 0.02), generated per expert to bound temporaries."""
    import torch

    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    w13 = torch.empty(experts, 2 * inter, hidden, dtype=torch.bfloat16, device=dev)
    w2 = torch.empty(experts, hidden, inter, dtype=torch.bfloat16, device=dev)
    for e in range(experts):
        w13[e] = 0.02 * torch.randn(2 * inter, hidden, generator=gen, device=dev)
        w2[e] = 0.02 * torch.randn(hidden, inter, generator=gen, device=dev)
    return w13, w2


def _gpu_local_cpus(dev):
    """The CPUs of the GPU's NUMA node (sysfs local_cpulist), within this process's affinity;
    None when unknown."""
    import torch

    try:
        pr = torch.cuda.get_device_properties(dev)
        bdf = "%04x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
        with open(f"/sys/bus/pci/devices/{bdf}/local_cpulist") as f:
            text = f.read().strip()
        cpus = set()
        for part in text.split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except (OSError, ValueError, AttributeError, RuntimeError):
        return None


class near_gpu:
    """Pinned host buffers allocated inside this block get their pages on the GPU's NUMA node
    (the calling thread runs there while they are allocated and first written); the process's
    CPU affinity is restored on exit, so later CPU work still uses every core."""

    def __init__(self, dev):
        self.dev = dev
        self.saved = None

    def __enter__(self):
        cpus = _gpu_local_cpus(self.dev)
        if cpus is not None:
            self.saved = os.sched_getaffinity(0)
            os.sched_setaffinity(0, cpus)
        return self

    def __exit__(self, *exc):
        if self.saved is not None:
            os.sched_setaffinity(0, self.saved)
        return False


def _hbm(nbytes, ms, peaks):
    gbs = nbytes / ms / 1e6
    return {"bytes": int(nbytes), "gbs": gbs, "frac": gbs / peaks["hbm_gbs"]}


def config0(t: Timer, dev, peaks, steps) -> dict:
    """Qwen3 prefill fold, T=4096, E=128, top-8, P=4: one fused router + fold launch."""
    import torch

    from exfold_b200 import ops
    from exfold_b200 import workloads as W

    lay = W.layer("qwen3_prefill")
    c, l_, _ = _qwen3_tables(lay, dev)
    x = torch.from_numpy(lay.logits).to(dev)
    ow = torch.empty((lay.tokens, KEEP), device=dev)
    oi = torch.empty((lay.tokens, KEEP), dtype=torch.int32, device=dev)
    ms = t.flushed(lambda: ops.router_fold_prefill(x, TOP_K, KEEP, c, l_, out=(ow, oi)), steps)
    x16 = x.to(torch.bfloat16)
    ms_16 = t.flushed(lambda: ops.router_fold_prefill(x16, TOP_K, KEEP, c, l_, out=(ow, oi)),
                      steps)
    nbytes = lay.tokens * (128 * 4 + KEEP * 8) + 2 * 128 * 128 * 4
    return {"tokens": lay.tokens, "us": ms * 1e3, "tokens_per_s": lay.tokens / ms * 1e3,
            "l2": "flushed between launches", "launches": 1, **_hbm(nbytes, ms, peaks),
            "bf16_logits_us": ms_16 * 1e3}


def config1(t: Timer, dev, peaks, steps) -> dict:
    """Qwen3 decode, B=256, E=128, D=64: the transform (router + decode budget) and the expert
    layer (H=2048, I=768): the layer alone, the decode fused with the layer, and the whole step
    (router + fused decode and layer)."""
    import torch

    from exfold_b200 import ops
    from exfold_b200 import workloads as W

    cfg = W.WORKLOADS["qwen3_decode"]
    lay = W.layer("qwen3_decode")
    c, l_, n = _qwen3_tables(lay, dev)
    x_logits = torch.from_numpy(lay.logits).to(dev)
    hidden, inter, budget = cfg["hidden"], cfg["intermediate"], cfg["budget"]

    def transform():
        rw, ri = ops.router_topk(x_logits, TOP_K)
        return ops.decode(rw, ri, n, c, l_, budget, variant="qwen3")

    us_transform = t.flushed(transform, steps) * 1e3
    tbytes = lay.tokens * 128 * 4 + 2 * 128 * 128 * 4 + 128 * 4 + lay.tokens * TOP_K * 8
    w13, w2 = _expert_weights(128, hidden, inter, 111, dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(112)
    x = torch.randn(lay.tokens, hidden, generator=gen, device=dev).to(torch.bfloat16)
    rw, ri = ops.router_topk(x_logits, TOP_K)
    dw, di = ops.decode(rw, ri, n, c, l_, budget, variant="qwen3")
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ms_layer = t.replays(lambda: ops.fused_experts(x, dw, di, w13, w2, status=status), steps)
    ms_fused = t.replays(lambda: ops.decode_fused_experts(
        x, rw, ri, n, c, l_, budget, w13, w2, variant="qwen3", status=status), steps)

    def whole():
        a, b = ops.router_topk(x_logits, TOP_K)
        ops.decode_fused_experts(x, a, b, n, c, l_, budget, w13, w2, variant="qwen3",
                                 status=status)

    ms_step = t.replays(whole, steps)
    active = int(torch.unique(di).numel())
    wbytes = active * 3 * hidden * inter * 2
    torch.cuda.synchronize(dev)
    out = {"batch": lay.tokens, "budget": budget, "hidden": hidden, "inter": inter,
           "transform_us": us_transform, "transform": _hbm(tbytes, us_transform / 1e3, peaks),
           "active_experts": active, "moe_layer_us": ms_layer * 1e3,
           "moe_layer_weights": _hbm(wbytes, ms_layer, peaks),
           "decode_fused_layer_us": ms_fused * 1e3,
           "step_us_router_decode_layer": ms_step * 1e3, "status": int(status.item()),
           "l2": "transform flushed between launches; expert weights > L2"}
    del w13, w2
    return out


def config2_fold(t: Timer, dev, peaks, steps, tokens=None):
    """DeepSeek-style prefill fold: biased-sigmoid router + DeepSeek-V4 fold (P=3, similarity
    blend) over T=65536 tokens (or `tokens`) and E=256 in one launch.  Returns the result and
    the routes."""
    import torch

    from exfold_b200 import ops
    from exfold_b200 import workloads as W

    lay = W.layer("dsv4_prefill", tokens=tokens)
    c, l_, cf = _dsv4_tables(lay, dev)
    x_logits = torch.from_numpy(lay.logits).to(dev)
    b = torch.from_numpy(lay.bias).to(dev)
    ow = torch.empty((lay.tokens, 3), device=dev)
    oi = torch.empty((lay.tokens, 3), dtype=torch.int32, device=dev)

    def fold():
        ops.router_fold_prefill(x_logits, 8, 3, c, l_, scoring="sigmoid", bias=b,
                                variant="dsv4", renorm_mode=2, conf_loss=cf, out=(ow, oi))

    ms_fold = t.flushed(fold, steps)
    x16 = x_logits.to(torch.bfloat16)
    ms_16 = t.flushed(lambda: ops.router_fold_prefill(
        x16, 8, 3, c, l_, scoring="sigmoid", bias=b, variant="dsv4", renorm_mode=2,
        conf_loss=cf, out=(ow, oi)), steps)
    fold()
    fbytes = lay.tokens * (256 * 4 + 3 * 8) + 3 * 256 * 256 * 4 + 256 * 4
    fbytes16 = fbytes - lay.tokens * 256 * 2
    out = {"tokens": lay.tokens, "keep": 3, "renorm": "similarity_blend",
           "fold_us": ms_fold * 1e3, "fold_tokens_per_s": lay.tokens / ms_fold * 1e3,
           "fold": _hbm(fbytes, ms_fold, peaks), "fold_l2": "flushed between launches",
           "fold_bf16_logits": {"us": ms_16 * 1e3, **_hbm(fbytes16, ms_16, peaks)}}
    return out, ow, oi


def config2(t: Timer, dev, peaks, steps, weights) -> dict:
    """DeepSeek-style prefill: the fold (config2_fold), then the expert layer (H=4096, I=2048)
    over its routes."""
    import torch

    from exfold_b200 import ops

    out, ow, oi = config2_fold(t, dev, peaks, steps)
    tokens = ow.shape[0]
    w13, w2 = weights
    gen = torch.Generator(device=dev)
    gen.manual_seed(212)
    x = torch.randn(tokens, 4096, generator=gen, device=dev).to(torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ms_layer = t.replays(lambda: ops.fused_experts(x, ow, oi, w13, w2, status=status),
                         max(3, steps // 4))
    flops = 6.0 * oi.numel() * 4096 * 2048
    tflops = flops / ms_layer / 1e9
    out.update({"active_experts": int(torch.unique(oi).numel()), "routes": oi.numel(),
                "moe_layer_ms": ms_layer,
                "moe_layer_tensor": {"tflops": tflops, "peak": peaks["bf16_tflops"],
                                     "frac": tflops / peaks["bf16_tflops"], "flops": flops,
                                     # the layer runs milliseconds back to back, under the
                                     # power cap: the sustained cuBLAS figure as well
                                     "peak_sustained": peaks["bf16_tflops_sustained"],
                                     "frac_sustained": tflops / peaks["bf16_tflops_sustained"]},
                "status": int(status.item())})
    del x
    return out


def config3(t: Timer, dev, peaks, steps, weights) -> list:
    """DeepSeek-style decode sweep, E=256: per (B, D) the transform (biased router + decode
    budget) and the step with the expert layer (router + decode fused with moe_align, gather,
    GEMMs and combine; H=4096, I=2048)."""
    import torch

    from exfold_b200 import ops
    from exfold_b200 import workloads as W

    cfg = W.WORKLOADS["dsv4_decode"]
    w13, w2 = weights
    rows = []
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(313)
    for batch in cfg["batches"]:
        lay = W.Layer(seed=cfg["seed"], tokens=batch, experts=256, top_k=8, kind="dsv4")
        c, l_, _ = _dsv4_tables(lay, dev)
        n = torch.from_numpy(lay.norms).to(dev)
        xl = torch.from_numpy(lay.logits).to(dev)
        b = torch.from_numpy(lay.bias).to(dev)
        x = torch.randn(batch, 4096, generator=gen, device=dev).to(torch.bfloat16)
        for budget in cfg["budgets"]:
            def transform():
                rw, ri = ops.router_topk(xl, 8, "sigmoid", b)
                ops.decode(rw, ri, n, c, l_, budget, variant="dsv4")

            def step():
                rw, ri = ops.router_topk(xl, 8, "sigmoid", b)
                ops.decode_fused_experts(x, rw, ri, n, c, l_, budget, w13, w2, variant="dsv4",
                                         status=status)

            us_t = t.flushed(transform, steps) * 1e3
            ms_s = t.replays(step, steps)
            rw, ri = ops.router_topk(xl, 8, "sigmoid", b)
            _, di = ops.decode(rw, ri, n, c, l_, budget, variant="dsv4")
            active = int(torch.unique(di).numel())
            tbytes = batch * 256 * 4 + 2 * 256 * 256 * 4 + 256 * 4 + batch * 8 * 8
            wbytes = active * 3 * 4096 * 2048 * 2
            rows.append({"batch": batch, "budget": budget, "transform_us": us_t,
                         "transform_gbs": tbytes / us_t / 1e3, "active_experts": active,
                         "step_us_router_decode_layer": ms_s * 1e3,
                         "layer_weights": _hbm(wbytes, ms_s, peaks)})
    torch.cuda.synchronize(dev)
    if int(status.item()) != 0:
        rows.append({"status": int(status.item())})
    return rows


def kernel_workload(name, t: Timer, dev, peaks, steps, tokens=None) -> dict:
    """One library kernel on a representative input (profiling commands for its summary):
    fold_kernel: the DeepSeek-V4 fold (mode 2) of given top-8 routes, T=65536, E=256;
    router_generic: router_kernel, sqrtsoftplus + bias top-8 over E=256 (the DeepSeek-V4
      model's scoring), T=65536;
    static_remap: the static decode table and the in-place remap of B=1024 x 8 routes, E=128;
    moe_align: the chunked moe_align of 196608 routes over 256 experts (block 64) and the
      one-CTA path on 2048 routes over 128 experts (block 16).
    The inputs fit in L2; the timings flush it between launches."""
    import torch

    from exfold_b200 import ops
    from exfold_b200 import workloads as W

    out: dict = {}
    if name in ("fold_kernel", "router_generic"):
        lay = W.layer("dsv4_prefill", tokens=tokens)
        x = torch.from_numpy(lay.logits).to(dev)
        b = torch.from_numpy(lay.bias).to(dev)
        if name == "router_generic":
            ms = t.flushed(lambda: ops.router_topk(x, 8, "sqrtsoftplus", b), steps)
            nbytes = lay.tokens * (256 * 4 + 8 * 8) + 256 * 4
        else:
            c, l_, cf = _dsv4_tables(lay, dev)
            w, ids = ops.router_topk(x, 8, "sigmoid", b)
            ms = t.flushed(lambda: ops.fold_prefill(w, ids, c, l_, 3, variant="dsv4",
                                                    renorm_mode=2, conf_loss=cf), steps)
            nbytes = lay.tokens * (8 * 8 + 3 * 8) + 3 * 256 * 256 * 4
        out.update(tokens=lay.tokens, us=ms * 1e3, **_hbm(nbytes, ms, peaks))
    elif name == "static_remap":
        lay = W.layer("qwen3_decode", tokens=1024)
        c, l_, n = _qwen3_tables(lay, dev)
        w, ids = ops.router_topk(torch.from_numpy(lay.logits).to(dev), 8)
        target, scale = ops.static_table(n, c, l_, 64)
        wc, ic = w.clone(), ids.clone()
        ms_t = t.flushed(lambda: ops.static_table(n, c, l_, 64), steps)
        ms_r = t.flushed(lambda: ops.static_remap_(wc, ic, target, scale), steps)
        out.update(batch=1024, table_us=ms_t * 1e3, remap_us=ms_r * 1e3,
                   remap=_hbm(2 * w.numel() * 8 + 128 * 8, ms_r, peaks))
    elif name == "moe_align":
        big = W.layer("dsv4_prefill", tokens=tokens)
        _, ids = ops.router_topk(torch.from_numpy(big.logits).to(dev), 8, "sigmoid",
                                 torch.from_numpy(big.bias).to(dev))
        ids3 = ids[:, :3].contiguous()
        ms_big = t.flushed(lambda: ops.moe_align_block_size(ids3, 64, 256), steps)
        small = W.layer("qwen3_decode")
        _, ids_s = ops.router_topk(torch.from_numpy(small.logits).to(dev), 8)
        ms_small = t.flushed(lambda: ops.moe_align_block_size(ids_s, 16, 128), steps)
        cap = ops.moe_align_capacity(ids3.numel(), 256, 64)
        out.update(routes=ids3.numel(), chunked_us=ms_big * 1e3,
                   chunked=_hbm(ids3.numel() * 4 * 2 + cap * 4, ms_big, peaks),
                   small_routes=ids_s.numel(), small_us=ms_small * 1e3)
    return out


def measure_configs(dev, stream, peaks, args) -> dict:
    t = Timer(dev, stream, max(3, args.warmup))
    steps = max(10, min(args.steps, 50))
    out = {"config0_qwen3_prefill_fold": config0(t, dev, peaks, steps),
           "config1_qwen3_decode": config1(t, dev, peaks, steps)}
    weights = _expert_weights(256, 4096, 2048, 222, dev)
    out["config2_dsv4_prefill"] = config2(t, dev, peaks, steps, weights)
    out["config3_dsv4_decode_sweep"] = config3(t, dev, peaks, steps, weights)
    del weights
    return out


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

    peaks = measured_peaks()
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            ms = timed(graph.replay, args.steps)
        ms_per_step = ms / args.steps
        tokens_per_step = LAYERS * TOKENS * world
        value = tokens_per_step / (ms_per_step / 1e3)
        launch_s = ms_per_step / 1e3 / LAYERS
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
        with near_gpu(dev):  # host pages on the GPU's NUMA node: the copies stay on its socket
            host_in = torch.empty((slots, TOKENS, EXPERTS), dtype=torch.float32).pin_memory()
            host_in.copy_(logits[:slots].cpu())
            host_w = torch.empty((slots, TOKENS, KEEP), dtype=torch.float32).pin_memory()
            host_i = torch.empty((slots, TOKENS, KEEP), dtype=torch.int32).pin_memory()
            host_w.zero_()
            host_i.zero_()
        dev_in = torch.empty((2, TOKENS, EXPERTS), dtype=torch.float32, device=dev)
        dev_w = torch.empty((2, TOKENS, KEEP), dtype=torch.float32, device=dev)
        dev_i = torch.empty((2, TOKENS, KEEP), dtype=torch.int32, device=dev)
        # Host->device copies, the router calls and device->host copies on three streams,
        # double buffered, so that layer l's results go back while layer l+1's logits come in
        # (PCIe runs both directions at once).  Every copy of the step is inside the timed region.
        copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event() for _ in range(2)]    # logits of buffer b are on the device
        ev_done = [torch.cuda.Event() for _ in range(2)]  # the call reading buffer b finished
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

        # the same step on bf16 logits (the gate output dtype of the served models)
        logits_bf16 = logits.to(torch.bfloat16)

        def step_bf16():
            for layer in range(LAYERS):
                ops.router_fold_prefill(logits_bf16[layer], TOP_K, KEEP, coeff[layer],
                                        loss[layer], out=(out_w[layer], out_ids[layer]))

        with torch.cuda.stream(stream):
            step_bf16()
            torch.cuda.synchronize(dev)
            g16 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g16, stream=stream):
                step_bf16()
            ms_16 = timed(g16.replay, args.steps) / args.steps
        del g16, logits_bf16
        bytes_16 = TOKENS * (EXPERTS * 2 + KEEP * 8) + 2 * EXPERTS * EXPERTS * 4
        launch_16 = ms_16 / 1e3 / LAYERS
        bf16 = {"value": tokens_per_step / (ms_16 / 1e3), "unit": UNIT, "ms_per_step": ms_16,
                "us_per_launch": launch_16 * 1e6, "bytes_per_launch": bytes_16,
                "achieved_gbs": bytes_16 / launch_16 / 1e9,
                "frac": bytes_16 / launch_16 / 1e9 / peaks["hbm_gbs"],
                "kernel": "exf::router_tpt_kernel<qwen3 fold, P=4, bf16>"}

        if args.workload == "prefill_only":  # profiling: the timed prefill step alone
            if rank == 0:
                print(json.dumps({"workload": "prefill_only", "layers": LAYERS,
                                  "tokens": TOKENS, "us_per_launch": launch_s * 1e6,
                                  "frac": achieved / peaks["hbm_gbs"],
                                  "batched_us_per_layer": 1e3 * ms_b / LAYERS,
                                  "bf16": bf16}), flush=True)
            del graph, gb
            if world > 1:
                dist.destroy_process_group()
            return

        e2e_steps = max(5, min(20, args.steps // 4))
        saved_warmup = args.warmup
        args.warmup = 1
        with torch.cuda.stream(stream):
            ms_e2e = timed(e2e_step, e2e_steps) / e2e_steps
        h2d = LAYERS * TOKENS * EXPERTS * 4
        d2h = LAYERS * TOKENS * KEEP * 8
        # the same with bf16 logits on the host (the served gate output dtype): half the H2D bytes
        with near_gpu(dev):
            host_in = host_in.to(torch.bfloat16).pin_memory()
        dev_in = torch.empty((2, TOKENS, EXPERTS), dtype=torch.bfloat16, device=dev)
        with torch.cuda.stream(stream):
            ms_e2e16 = timed(e2e_step, e2e_steps) / e2e_steps
        args.warmup = saved_warmup
        del host_in, host_w, host_i, dev_in, dev_w, dev_i

        with torch.cuda.stream(stream):
            decode = measure_decode(dev, world, rank, stream, coeff, loss, timed, args)

        configs = None
        if world == 1:
            configs = measure_configs(dev, stream, peaks, args)

    cpu = None
    if rank == 0 and world == 1:
        threads = host_threads()
        from exfold_b200 import workloads as W

        # 32768 tokens a pass (2048 per thread and layer): a call of the oracle on a few hundred
        # tokens spends most of its time outside the arithmetic, which would understate the CPU
        sample = W.logits(W.WORKLOADS["qwen3_layers"]["seed"], 32768, EXPERTS)
        with ThreadPoolExecutor(max_workers=threads) as pool:
            cpu_layers_pass(pool, threads, [sample[:256]] * LAYERS, coeff_np, loss_np)
            done, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < 15.0:
                done += cpu_layers_pass(pool, threads, [sample] * LAYERS, coeff_np, loss_np)
            rate = done / (time.perf_counter() - t0)
        cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{done} token-layers: {sample.shape[0]} tokens x all {LAYERS} layers' "
                         f"tables per pass, ~15 s on {threads} threads"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) logits, seeded calibration tables; expert "
                    "weights N(0, 0.02) bf16)",
            "config": {"workload": "qwen3_layers_prefill", "layers": LAYERS,
                       "tokens_per_gpu": TOKENS, "experts": EXPERTS, "top_k": TOP_K,
                       "keep": KEEP, "parallelism": f"token-sharded x{world}",
                       "l2": "inputs 3.2 GB/step per GPU > L2, no flush"},
            "tokens_per_s_per_forward": value / LAYERS,
            "gpu_launches": LAYERS * args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                         "traffic": profiled_traffic("router_fold_qwen3_layer"),
                         "peak_source": peaks["source"],
                         "kernel": "exf::router_tpt_kernel<qwen3 fold, P=4>",
                         "bytes_per_launch": bytes_per_launch(TOKENS),
                         "us_per_launch": launch_s * 1e6},
            "layer_batched": {"ms_per_step": ms_b, "value": tokens_per_step / (ms_b / 1e3),
                              "launches_per_step": 1},
            "bf16_logits": bf16,
            "e2e": {"value": tokens_per_step / (ms_e2e / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": ms_e2e, "steps": e2e_steps},
            "e2e_bf16_logits": {"value": tokens_per_step / (ms_e2e16 / 1e3), "unit": UNIT,
                                "h2d_bytes_per_step": h2d // 2, "d2h_bytes_per_step": d2h,
                                "ms_per_step": ms_e2e16},
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "decode": decode,
            "configs": configs,
        }
        print(json.dumps(line), flush=True)
    del graph, gb
    if world > 1:
        dist.destroy_process_group()


# ---- single workloads (--workload NAME), for profiling: one JSON line each -------------------
def run_extra(args) -> None:
    import torch

    from exfold_b200 import ops
    from exfold_b200 import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    peaks = measured_peaks()
    t = Timer(dev, stream, max(3, args.warmup))
    steps = max(5, min(args.steps, 200))
    out = {"workload": args.workload}
    if args.workload == "config0":
        out.update(config0(t, dev, peaks, steps))
    elif args.workload == "config1":
        out.update(config1(t, dev, peaks, steps))
    elif args.workload in ("config2", "config3"):
        weights = _expert_weights(256, 4096, 2048, 222, dev)
        fn = config2 if args.workload == "config2" else config3
        out["result"] = fn(t, dev, peaks, steps, weights)
    elif args.workload == "moe_dsv4_prefill":
        # the expert layer alone; --tokens / --experts shrink the case for profiling
        lay = W.layer("dsv4_prefill", tokens=args.tokens)
        c, l_, cf = _dsv4_tables(lay, dev)
        w, ids = ops.router_fold_prefill(
            torch.from_numpy(lay.logits).to(dev), 8, 3, c, l_, scoring="sigmoid",
            bias=torch.from_numpy(lay.bias).to(dev), variant="dsv4", renorm_mode=2,
            conf_loss=cf)
        experts = 256
        if args.experts and args.experts < experts:  # fold the routes onto fewer experts
            ids = (ids % args.experts).to(ids.dtype)
            experts = args.experts
        w13, w2 = _expert_weights(experts, 4096, 2048, 222, dev)
        gen = torch.Generator(device=dev)
        gen.manual_seed(11)
        x = torch.randn(lay.tokens, 4096, generator=gen, device=dev).to(torch.bfloat16)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        ms = t.replays(lambda: ops.fused_experts(x, w, ids, w13, w2, status=status), steps)
        flops = 6.0 * ids.numel() * 4096 * 2048
        out.update(tokens=lay.tokens, routes=ids.numel(), ms_per_layer=ms,
                   tflops=flops / ms / 1e9,
                   tensor_frac_of_measured_peak=flops / ms / 1e9 / peaks["bf16_tflops"],
                   status=int(status.item()))
    elif args.workload == "moe_qwen3_decode":
        out.update(config1(t, dev, peaks, steps))
    elif args.workload == "dsv4_fold":
        out.update(config2_fold(t, dev, peaks, steps, tokens=args.tokens)[0])
    elif args.workload in ("fold_kernel", "router_generic", "static_remap", "moe_align"):
        out.update(kernel_workload(args.workload, t, dev, peaks, steps, args.tokens))
    elif args.workload == "calibration_update":
        # PairwiseScalarStats.update (exfold/qwen3/calibration.py:49-95) at the Qwen3 layer shape:
        # 8 routes of 2048-wide bf16 expert outputs over 128 experts, 16384 tokens per call
        # (512 MiB of outputs > L2); the pass is bound by reading the outputs.
        from exfold_b200.calibration import PairwiseScalarStats

        gen = torch.Generator(device=dev)
        gen.manual_seed(11)
        T, K, H, E = (args.tokens or 16384), 8, 2048, 128
        outs = torch.randn((T, K, H), generator=gen, device=dev).to(torch.bfloat16)
        ids = torch.randint(0, E, (T, K), generator=gen, device=dev, dtype=torch.int32)
        stats = PairwiseScalarStats(E, device=dev)
        ms = t.replays(lambda: stats.update(ids, outs), steps)
        nbytes = T * K * H * 2 + T * K * 4
        out.update(tokens=T, top_k=K, hidden=H, experts=E, us_per_call=ms * 1e3,
                   tokens_per_s=T / ms * 1e3, **_hbm(nbytes, ms, peaks))
    print(json.dumps(out), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=LAYERS, help="smaller cases for profiling")
    ap.add_argument("--tokens", type=int, default=None, help="smaller cases for profiling")
    ap.add_argument("--experts", type=int, default=0, help="fewer experts (profiling cases)")
    ap.add_argument("--workload", default="qwen3_layers",
                    choices=["qwen3_layers", "prefill_only", "config0", "config1", "config2",
                             "config3", "dsv4_fold", "fold_kernel", "router_generic",
                             "static_remap", "moe_align", "moe_dsv4_prefill",
                             "moe_qwen3_decode", "calibration_update"])
    args = ap.parse_args()
    set_shape(args.layers, args.tokens or TOKENS)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload not in ("qwen3_layers", "prefill_only"):
        run_extra(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
