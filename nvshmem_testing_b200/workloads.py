"""Seeded synthetic inputs for the benchmark configurations.

Shapes (tokens per rank T, hidden H, experts E, top-k K, expert GEMM width
N) follow the expert-layer configurations this package is measured on:

  cpu_gloo     T=128,  H=256,  E=4,   K=1, N=512,   fp32, uniform top-1
  mixtral      T=4096, H=4096, E=8,   K=2, N=14336, bf16, uniform distinct
  deepseek_v3  T=4096, H=7168, E=256, K=8, N=2048,  bf16, uniform distinct
  skewed_zipf  T=8192, H=2048, E=64,  K=6, N=1408,  bf16, Zipf(1.2)
  decode       T in {16..8192}, H=4096, E=64, K=8, N=1536, bf16, uniform

Activations are N(0, 1) seeded by (seed + rank); weights are 0.02 * N(0, 1)
seeded by (seed + 10086 + rank), mirroring benchmark.py:121 of the
reference.  Routing ids are generated directly (no router):

* uniform distinct top-k: ``rand(T, E).topk(K).indices``;
* uniform top-1: ``randint(0, E, (T, 1))``;
* Zipf(alpha) top-k without replacement (Efraimidis-Spirakis): expert of
  popularity rank i (over a seeded permutation of the ids that is identical
  on all ranks) has weight (i+1)^-alpha; key = log(u) / weight; take the K
  largest keys.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    T: int
    H: int
    E: int
    K: int
    N: int
    routing: str = "uniform"      # uniform | top1 | zipf
    alpha: float = 1.2
    dtype: torch.dtype = torch.bfloat16
    seed: int = 0

    def local_experts(self, world_size: int) -> int:
        if self.E % world_size:
            raise ValueError(f"{self.E} experts do not split over {world_size} ranks")
        return self.E // world_size


CONFIGS = {
    "cpu_gloo": Workload("cpu_gloo", 128, 256, 4, 1, 512, routing="top1", dtype=torch.float32),
    "mixtral": Workload("mixtral", 4096, 4096, 8, 2, 14336),
    "deepseek_v3": Workload("deepseek_v3", 4096, 7168, 256, 8, 2048),
    "skewed_zipf": Workload("skewed_zipf", 8192, 2048, 64, 6, 1408, routing="zipf"),
    "decode": Workload("decode", 1024, 4096, 64, 8, 1536),
}
DECODE_TOKENS = (16, 64, 256, 1024, 4096, 8192)


def get(name: str, **overrides) -> Workload:
    w = CONFIGS[name]
    return replace(w, **overrides) if overrides else w


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def top_idxs(w: Workload, rank: int, device="cpu") -> torch.Tensor:
    """[T, K] int64 expert ids for `rank`."""
    g = _gen(w.seed * 7919 + 17 + rank, device)
    if w.routing == "top1" or w.K == 1 and w.routing == "uniform":
        return torch.randint(0, w.E, (w.T, 1), generator=g, device=device)
    if w.routing == "uniform":
        return torch.rand(w.T, w.E, generator=g, device=device).topk(w.K, dim=-1).indices
    if w.routing == "zipf":
        order = torch.randperm(w.E, generator=_gen(w.seed * 7919 + 5, "cpu")).to(device)
        weight = torch.empty(w.E, dtype=torch.float64, device=device)
        weight[order] = torch.arange(1, w.E + 1, dtype=torch.float64, device=device).pow(-w.alpha)
        u = torch.rand(w.T, w.E, generator=g, device=device, dtype=torch.float64).clamp_min(1e-300)
        keys = torch.log(u) / weight
        return keys.topk(w.K, dim=-1).indices
    raise ValueError(f"unknown routing {w.routing}")


def tokens(w: Workload, rank: int, device="cpu") -> torch.Tensor:
    g = _gen(w.seed + rank, device)
    return torch.randn(w.T, w.H, generator=g, device=device, dtype=torch.float32).to(w.dtype)


def weights(w: Workload, rank: int, world_size: int, device="cpu") -> torch.Tensor:
    g = _gen(w.seed + 10086 + rank, device)
    El = w.local_experts(world_size)
    return (0.02 * torch.randn(El, w.H, w.N, generator=g, device=device, dtype=torch.float32)).to(w.dtype)


def top_vals(w: Workload, rank: int, device="cpu") -> torch.Tensor:
    """[T, K] float32 router weights for the combine step: a softmax over
    seeded N(0, 1) logits of the K chosen experts (the renormalised top-k
    weights of a softmax router); for top-1, the sigmoid of the logit."""
    g = _gen(w.seed * 7919 + 4242 + rank, device)
    K = 1 if (w.routing == "top1" or w.K == 1) else w.K
    logits = torch.randn(w.T, K, generator=g, device=device, dtype=torch.float32)
    return logits.softmax(dim=-1) if K > 1 else logits.sigmoid()
