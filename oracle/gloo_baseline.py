"""The reference's CPU/gloo path, restated for timing on the host cores.

The reference runs its NCCL baseline (baseline.py:8-56) on CPU under gloo
at world_size=2 in fp32 (T=128 tokens per rank, H=256, 4 experts, top-1,
expert GEMM [tokens_e, 256] x [256, 512]).  ``gloo_layer`` is one rank's
step of that path with this package's routing restatement in front:

* utils.py:28-75: per-expert buckets in ascending token order, padded to the
  largest bucket (all-reduced MAX over the group, the deliberate fix of the
  rank-local max at utils.py:45-49) and concatenated expert-major;
* benchmark.py:95-118: the per-expert counts exchanged with an
  all_to_all_single into ``recv_counts[W, El]``;
* baseline.py:18-50: the equal-split all_to_all_single of the padded send
  buffer, the view [W, El, gm, H] permuted to [El, W*gm, H], and a bmm with
  the local weights [El, H, N].

Test infrastructure and the CPU baseline only: the library never imports it.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from .routing import bucketize, local_max, pad_coalesce


def gloo_layer(tokens: torch.Tensor, top_idxs: np.ndarray, num_experts: int, weights: torch.Tensor,
               group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """One rank's step on CPU tensors under an initialised (gloo) group.
    Returns ``(out [El, W*gm, N], recv_counts [W, El])``."""
    W = dist.get_world_size(group)
    El = num_experts // W
    counts, offsets, perm = bucketize(top_idxs, num_experts)
    m = torch.tensor([local_max(counts)], dtype=torch.int64)
    dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
    gm = int(m[0])
    send = torch.from_numpy(pad_coalesce(tokens.numpy(), counts, offsets, perm, gm))
    sent = torch.from_numpy(counts.astype(np.int32)).view(W, El).contiguous()
    recv_counts = torch.empty_like(sent)
    dist.all_to_all_single(recv_counts, sent, group=group)
    chunk = El * gm
    recv = torch.zeros(chunk * W, tokens.shape[1], dtype=tokens.dtype)
    dist.all_to_all_single(recv, send, group=group)
    x = recv.view(W, El, gm, tokens.shape[1]).permute(1, 0, 2, 3).flatten(1, 2)
    return torch.bmm(x, weights), recv_counts
