"""Seeded synthetic inputs for the routing-transform workloads.

The generator is a counter-based splitmix64 stream evaluated with numpy, so
the same (seed, stream) pair gives the same numbers on any host without
depending on numpy's or torch's generator implementations.  Normals come
from the Box-Muller transform in float64 and are rounded once to float32.

Workloads (all fp32 calibration tables, row-major [src][tgt]):

* ``qwen3_prefill``  T=4096 tokens, E=128, top-8, keep P=4.  Logits N(0,1);
  s ~ N(0.35, 0.15); L ~ U[0.2, 1.0) with +inf on the diagonal.
* ``qwen3_decode``   B=256, E=128, top-8, budget D=64; norms LogNormal(0, 0.5).
  Expert MLP: hidden 2048, intermediate 768, x ~ N(0,1), W ~ N(0, 0.02).
* ``dsv4_prefill``   T=65536, E=256, top-8, keep P=3, biased sigmoid router
  (bias ~ N(0, 0.1)); s ~ N(0.3, 0.2); L ~ U[0.1, 1.0) diagonal +inf.
  Expert MLP: hidden 4096, intermediate 2048.
* ``dsv4_decode``    E=256, B in {8, 32, 128, 512}, D in {64, 128}.
* ``qwen3_layers``   48 layers of the qwen3 shapes with per-layer seeds;
  prefill T=131072 at P=4, decode B=1024 at D=64.
"""

from __future__ import annotations

import numpy as np

_MASK64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def _stream_base(seed: int, stream: int) -> np.uint64:
    mixed = _splitmix64(np.array([(seed & 0xFFFFFFFF) << 20 ^ (stream & 0xFFFFF)], dtype=np.uint64))
    return mixed[0]


def uniform(seed: int, stream: int, n: int) -> np.ndarray:
    """n float64 values in [0, 1) from (seed, stream)."""
    base = _stream_base(seed, stream)
    with np.errstate(over="ignore"):
        counters = np.arange(n, dtype=np.uint64) * np.uint64(0xD1B54A32D192ED03) + base
    bits = _splitmix64(counters) >> np.uint64(11)
    return bits.astype(np.float64) * (1.0 / 9007199254740992.0)


def normal(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """n float32 normals (Box-Muller on two uniform streams)."""
    u1 = 1.0 - uniform(seed, stream * 2 + 1, n)
    u2 = uniform(seed, stream * 2 + 2, n)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return (mean + std * z).astype(np.float32)


def uniform_range(seed: int, stream: int, n: int, lo: float, hi: float) -> np.ndarray:
    """n float32 values in [lo, hi); uses a stream id disjoint from normal()'s."""
    return (lo + (hi - lo) * uniform(seed, 0x800 + stream, n)).astype(np.float32)


# stream ids: fixed per tensor role so that every workload is reproducible
_S_LOGITS, _S_BIAS, _S_COEFF, _S_LOSS, _S_NORMS, _S_CONF = 1, 2, 3, 4, 5, 6


def logits(seed: int, tokens: int, experts: int) -> np.ndarray:
    return normal(seed, _S_LOGITS, tokens * experts).reshape(tokens, experts)


def router_bias(seed: int, experts: int, std: float = 0.1) -> np.ndarray:
    return normal(seed, _S_BIAS, experts, 0.0, std)


def coefficient(seed: int, experts: int, mean: float, std: float) -> np.ndarray:
    return normal(seed, _S_COEFF, experts * experts, mean, std).reshape(experts, experts)


def loss_matrix(seed: int, experts: int, lo: float, hi: float, diag: float = np.inf) -> np.ndarray:
    m = uniform_range(seed, _S_LOSS, experts * experts, lo, hi).reshape(experts, experts)
    np.fill_diagonal(m, diag)
    return m


def expert_norms(seed: int, experts: int, sigma: float = 0.5) -> np.ndarray:
    return np.exp(normal(seed, _S_NORMS, experts, 0.0, sigma).astype(np.float64)).astype(np.float32)


class Layer:
    """Calibration tables and router inputs of one MoE layer."""

    def __init__(self, *, seed: int, tokens: int, experts: int, top_k: int, kind: str):
        self.seed, self.tokens, self.experts, self.top_k, self.kind = seed, tokens, experts, top_k, kind
        self.logits = logits(seed, tokens, experts)
        if kind == "qwen3":
            self.bias = None
            self.coeff = coefficient(seed, experts, 0.35, 0.15)
            self.loss = loss_matrix(seed, experts, 0.2, 1.0)
        elif kind == "dsv4":
            self.bias = router_bias(seed, experts)
            self.coeff = coefficient(seed, experts, 0.3, 0.2)
            self.loss = loss_matrix(seed, experts, 0.1, 1.0)
        else:
            raise ValueError(kind)
        self.norms = expert_norms(seed, experts)

    @property
    def scoring(self) -> str:
        return "softmax" if self.kind == "qwen3" else "sigmoid"


WORKLOADS = {
    "qwen3_prefill": dict(kind="qwen3", tokens=4096, experts=128, top_k=8, keep=4, seed=1000),
    "qwen3_decode": dict(kind="qwen3", tokens=256, experts=128, top_k=8, budget=64, seed=1100,
                         hidden=2048, intermediate=768),
    "dsv4_prefill": dict(kind="dsv4", tokens=65536, experts=256, top_k=8, keep=3, seed=2000,
                         hidden=4096, intermediate=2048),
    "dsv4_decode": dict(kind="dsv4", experts=256, top_k=8, batches=(8, 32, 128, 512),
                        budgets=(64, 128), seed=2100, hidden=4096, intermediate=2048),
    "qwen3_layers": dict(kind="qwen3", layers=48, experts=128, top_k=8, prefill_tokens=131072,
                         keep=4, decode_tokens=1024, budget=64, seed=4000),
}


def layer(name: str, *, tokens: int | None = None, layer_index: int = 0) -> Layer:
    cfg = WORKLOADS[name]
    t = tokens if tokens is not None else cfg.get("tokens", cfg.get("prefill_tokens"))
    return Layer(seed=cfg["seed"] + layer_index, tokens=t, experts=cfg["experts"],
                 top_k=cfg["top_k"], kind=cfg["kind"])
