"""Multi-GPU parity of the sharded decode (2 GPUs of one node, one process per GPU).

Skipped with fewer than two GPUs.  Every rank's result of the one-launch peer exchange
(`DecodeExchange`, eager and replayed from a CUDA graph) and of the all-reduce path must equal
the single-GPU decode of the whole batch bit for bit (tests/multigpu_worker.py).
"""

from __future__ import annotations

import json
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_decode_two_gpus_equals_single_gpu(tmp_path):
    import torch.multiprocessing as mp

    import multigpu_worker

    world = 2
    ctx = mp.start_processes(multigpu_worker.run, args=(world, free_port(), str(tmp_path)),
                             nprocs=world, start_method="spawn", join=False)
    for _ in range(10):  # at most ~5 minutes, then the workers are ended
        if ctx.join(timeout=30):
            break
    else:
        for proc in ctx.processes:
            proc.terminate()
        pytest.fail("the two-GPU workers did not finish")
    for rank in range(world):
        res = json.loads((tmp_path / f"rank{rank}.json").read_text())
        assert res["ok"], res
