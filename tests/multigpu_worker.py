"""Worker of the multi-GPU tests (tests/test_gpu_multigpu.py): one process per GPU.

Each rank routes its shard of a decode batch and runs the sharded decode both ways (the
one-launch peer exchange and the importance / all-reduce / apply steps), eagerly and replayed
from a CUDA graph, and compares every layer with the single-GPU decode of the whole batch, which
every rank computes from the same seeded inputs.  The verdict goes to a JSON file per rank.
"""

from __future__ import annotations

import json
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "exfold-moe_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def run(rank: int, world: int, port: int, out_dir: str, layers: int = 6, batch: int = 1024,
        experts: int = 128, budget: int = 64) -> None:
    import torch
    import torch.distributed as dist

    from exfold_b200 import ops, parallel
    from exfold_b200 import workloads as W

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    result = {"rank": rank, "ok": True, "failures": []}
    try:
        start, end = parallel.shard_range(batch, world, rank)
        xch = parallel.DecodeExchange(experts, device=dev)
        cases = []
        for layer in range(layers):
            lay = W.layer("qwen3_decode", tokens=batch, layer_index=layer)
            x = torch.from_numpy(lay.logits).to(dev)
            fw, fi = ops.router_topk(x, 8)
            n, c, l_ = (torch.from_numpy(a).to(dev) for a in (lay.norms, lay.coeff, lay.loss))
            variant = "qwen3" if layer % 2 == 0 else "dsv4"
            ew, ei = ops.decode(fw, fi, n, c, l_, budget, variant=variant)
            cases.append((fw[start:end].contiguous(), fi[start:end].contiguous(), n, c, l_,
                          variant, ew[start:end], ei[start:end]))

        def check(tag, got):
            for layer, ((gw, gi), case) in enumerate(zip(got, cases)):
                if not (torch.equal(gi, case[7]) and torch.equal(gw, case[6])):
                    result["ok"] = False
                    result["failures"].append(f"{tag} layer {layer}")

        for rep in range(2):
            check(f"exchange eager {rep}", [
                xch.decode(w, i, n, c, l_, budget, variant=v) for w, i, n, c, l_, v, _, _ in cases])
        check("all-reduce", [parallel.sharded_decode(w, i, n, c, l_, budget, variant=v)
                             for w, i, n, c, l_, v, _, _ in cases])
        s = torch.cuda.Stream(dev)
        with torch.cuda.stream(s):
            g = torch.cuda.CUDAGraph()
            outs: list = []
            with torch.cuda.graph(g, stream=s):
                for w, i, n, c, l_, v, _, _ in cases:
                    outs.append(xch.decode(w, i, n, c, l_, budget, variant=v))
            for _ in range(4):
                g.replay()
        torch.cuda.synchronize(dev)
        check("exchange graph", outs)
        result["status"] = int(xch.status.item())
        result["calls"] = int(xch.buffer[0].item())
        if result["status"] != 0 or result["calls"] != 2 * layers + 4 * layers:
            result["ok"] = False
        dist.barrier()
        del g
        xch.close()
    except Exception as exc:  # noqa: BLE001 - reported to the parent test
        result["ok"] = False
        result["failures"].append(repr(exc))
    finally:
        Path(out_dir, f"rank{rank}.json").write_text(json.dumps(result))
        dist.destroy_process_group()
