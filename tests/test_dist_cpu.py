"""world_size-2 gloo tests of the sharded decode exchange, on CPU.

The per-rank compute is the CPU oracle (test infrastructure) standing in for the CUDA kernels;
what is under test is the host logic of exfold_b200.parallel: the token sharding, the int64
importance all-reduce, and that the sharded result equals the unsharded decode bit for bit.
A second test makes one rank fail before the collective and checks that the other rank's
all-reduce ends with an error (short process-group timeout) instead of hanging.
"""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _paths():
    for p in (str(ROOT), str(ROOT / "exfold-moe_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)


def oracle_importance(w, ids, norms, importance):
    from oracle import oracle as O

    importance += torch.from_numpy(O.importance(w.numpy(), ids.numpy(), norms.numpy()))


def oracle_apply(importance, w, ids, coeff, loss, budget, variant):
    from oracle import oracle as O

    ow, oi = O.decode_apply(importance.numpy(), w.numpy(), ids.numpy(), coeff.numpy(),
                            loss.numpy(), budget, variant)
    return torch.from_numpy(ow), torch.from_numpy(oi)


def _worker(rank, world, port, variant, out_dir):
    _paths()
    from exfold_b200 import parallel
    from exfold_b200 import workloads as W
    from oracle import oracle as O

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=30))
    lay = W.layer("qwen3_layers", tokens=1024, layer_index=5)
    w, ids = O.router_topk(lay.logits, 8, "softmax")
    start, end = parallel.shard_range(1024, world, rank)
    ow, oi = parallel.sharded_decode(
        torch.from_numpy(w[start:end]), torch.from_numpy(ids[start:end]),
        torch.from_numpy(lay.norms), torch.from_numpy(lay.coeff), torch.from_numpy(lay.loss), 64,
        variant=variant, importance_fn=oracle_importance, apply_fn=oracle_apply)
    np.save(os.path.join(out_dir, f"w{rank}.npy"), ow.numpy())
    np.save(os.path.join(out_dir, f"i{rank}.npy"), oi.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("variant", ["qwen3", "dsv4"])
def test_sharded_decode_equals_unsharded(tmp_path, variant):
    _paths()
    from exfold_b200 import workloads as W
    from oracle import oracle as O

    world = 2
    mp.start_processes(_worker, args=(world, free_port(), variant, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    lay = W.layer("qwen3_layers", tokens=1024, layer_index=5)
    w, ids = O.router_topk(lay.logits, 8, "softmax")
    if variant == "qwen3":
        ew, ei, _ = O.decode_qwen3(w, ids, lay.norms, lay.coeff, lay.loss, 64)
    else:
        ew, ei = O.decode_dsv4(w, ids, lay.norms, lay.coeff, lay.loss, 64)
    gw = np.concatenate([np.load(tmp_path / f"w{r}.npy") for r in range(world)])
    gi = np.concatenate([np.load(tmp_path / f"i{r}.npy") for r in range(world)])
    np.testing.assert_array_equal(gi, ei)
    np.testing.assert_array_equal(gw, ew)


def _failing_worker(rank, world, port, out_dir):
    _paths()
    from exfold_b200 import parallel

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        # this rank fails on the host before reaching the collective and leaves
        open(os.path.join(out_dir, "rank1_failed"), "w").close()
        os._exit(0)
    x = torch.ones(4, 8)
    ids = torch.zeros(4, 8, dtype=torch.int32)
    try:
        parallel.sharded_decode(x, ids, torch.ones(16), torch.ones(16, 16), torch.ones(16, 16),
                                4, importance_fn=oracle_importance, apply_fn=oracle_apply)
        result = "completed"
    except Exception as exc:  # noqa: BLE001 - the failure is the expected outcome
        result = f"error: {type(exc).__name__}"
    with open(os.path.join(out_dir, "rank0_result"), "w") as f:
        f.write(result)
    os._exit(0)


def test_peer_failure_surfaces_as_error_not_hang(tmp_path):
    world = 2
    ctx = mp.start_processes(_failing_worker, args=(world, free_port(), str(tmp_path)),
                             nprocs=world, start_method="spawn", join=False)
    for p in ctx.processes:
        p.join(timeout=60)
    alive = [p for p in ctx.processes if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung instead of failing"
    assert (tmp_path / "rank1_failed").exists()
    assert (tmp_path / "rank0_result").read_text().startswith("error")
