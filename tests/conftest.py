"""Test configuration: the `gpu` marker, import paths, and the router kernel choice fixture."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "exfold-moe_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(params=["by_size", "tile"])
def router_kernel_choice(request):
    """Run a router test twice: with the library's size-based choice (launches below its
    threshold take the generic kernel) and with the tile kernels (E = 128 softmax, E = 256
    biased sigmoid) taken at every size, so that both kernels meet every case."""
    if request.param == "by_size":
        yield request.param
        return
    from exfold_b200 import ops

    previous = ops.router_tile_min_rows(0)
    try:
        yield request.param
    finally:
        ops.router_tile_min_rows(previous)
