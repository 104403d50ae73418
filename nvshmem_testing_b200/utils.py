"""Routing post-processing on the device: counts, offsets, permutation, pad.

Reference: utils.py:7-75 (``gen_tensor``) and utils.py:78-80
(``gen_weights``).  The reference buckets tokens on the host with one boolean
mask per expert (``(top_idxs == ex).any(-1)``, :30-41), pads every bucket to
the largest bucket with zero rows (:45-64), concatenates them expert-major
(:69) and returns ``(coalesced [E*gm, H], chunk_size = gm*El, lengths [E])``.

``route`` and ``dispatch`` do the same on the device with the sm_100a
kernels ``moe_route`` (one pass for counts/offsets, one stable bitmap pass
for the permutation) and ``moe_pack_padded``.  One deliberate deviation:
the reference's "global" max is the rank-local max (:45-49), so
``chunk_size`` can differ between ranks; ``dispatch`` all-reduces it with
MAX over the process group so the equal-split exchange is consistent.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _native as N


@dataclass
class Routing:
    counts: torch.Tensor     # [E] int32: tokens per expert
    offsets: torch.Tensor    # [E+1] int32: exclusive scan of counts
    perm: torch.Tensor       # [T*K] int32: first offsets[E] entries are token ids grouped by expert
    max_count: torch.Tensor  # [1] int32: local max bucket
    slots: torch.Tensor | None = None  # [T, K] int32: row of (t, k) inside its bucket, -1 if not routed


def _stream_ptr(dev: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def route(top_idxs: torch.Tensor, num_experts: int, with_slots: bool = False) -> Routing:
    """Per-expert counts, offsets and stable token permutation (no host sync).

    ``with_slots`` also returns, per (token, k), the token's row inside the
    bucket of ``top_idxs[t, k]`` (the key the combine step gathers with)."""
    if not top_idxs.is_cuda:
        raise ValueError("top_idxs must be a CUDA tensor")
    if top_idxs.dim() == 1:
        top_idxs = top_idxs[:, None]
    if top_idxs.dtype not in (torch.int32, torch.int64):
        raise TypeError("top_idxs must be int32 or int64")
    ids = top_idxs.contiguous()
    T, K = ids.shape
    dev = ids.device
    counts = torch.empty(num_experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    perm = torch.empty(max(T * K, 1), dtype=torch.int32, device=dev)
    maxc = torch.empty(1, dtype=torch.int32, device=dev)
    if with_slots:
        slots = torch.empty((T, K), dtype=torch.int32, device=dev)
        N.check(N.lib().moe_route_slots(ids.data_ptr(), int(ids.dtype == torch.int64), T, K, num_experts,
                                        counts.data_ptr(), offsets.data_ptr(), perm.data_ptr(), slots.data_ptr(),
                                        maxc.data_ptr(), _stream_ptr(dev)), "moe_route_slots")
        return Routing(counts, offsets, perm, maxc, slots)
    N.check(N.lib().moe_route(ids.data_ptr(), int(ids.dtype == torch.int64), T, K, num_experts, counts.data_ptr(),
                              offsets.data_ptr(), perm.data_ptr(), maxc.data_ptr(), _stream_ptr(dev)), "moe_route")
    return Routing(counts, offsets, perm, maxc)


def pack_padded(tokens: torch.Tensor, r: Routing, gm: int) -> torch.Tensor:
    """``[E*gm, H]``: bucket e in rows [e*gm, e*gm + counts[e]), zero rows after."""
    tokens = tokens.contiguous()
    E = r.counts.numel()
    H = tokens.shape[1]
    out = torch.empty((E * gm, H), dtype=tokens.dtype, device=tokens.device)
    N.check(N.lib().moe_pack_padded(tokens.data_ptr(), H, tokens.element_size(), r.counts.data_ptr(),
                                    r.offsets.data_ptr(), r.perm.data_ptr(), E, gm, out.data_ptr(),
                                    _stream_ptr(tokens.device)), "moe_pack_padded")
    return out


def pack_compact(tokens: torch.Tensor, r: Routing, rows: int | None = None) -> torch.Tensor:
    """``[offsets[E], H]``: every bucket back to back in expert order, no
    padding (the general all-to-all's send buffer).  ``rows`` = offsets[E]
    if known (otherwise read from the device)."""
    tokens = tokens.contiguous()
    n = int(r.offsets[-1].item()) if rows is None else int(rows)
    H = tokens.shape[1]
    out = torch.empty((n, H), dtype=tokens.dtype, device=tokens.device)
    N.check(N.lib().moe_pack_compact(tokens.data_ptr(), H, tokens.element_size(), r.perm.data_ptr(), n,
                                     out.data_ptr(), _stream_ptr(tokens.device)), "moe_pack_compact")
    return out


def global_max_count(r: Routing, group=None) -> int:
    """All-reduced (MAX) largest bucket; at least 1 like the reference, whose
    empty buckets carry a one-row placeholder (utils.py:36-41).

    The one host read of the routing: a kernel writes the value into pinned
    host memory (``moe_publish_i32``) and the host waits for an event after
    it, i.e. for this stream's work only — not behind a bulk device-to-host
    copy that another stream may have queued on the copy engines."""
    m = r.max_count.clone()
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
    host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    N.check(N.lib().moe_publish_i32(m.data_ptr(), 1, host.data_ptr(), _stream_ptr(m.device)), "moe_publish_i32")
    done = torch.cuda.Event()
    done.record(torch.cuda.current_stream(m.device))
    done.synchronize()
    return max(int(host[0]), 1)


def dispatch(tokens: torch.Tensor, top_idxs: torch.Tensor, num_experts: int, world_size: int, group=None,
             gm: int | None = None, general_a2a: bool = False) -> tuple[torch.Tensor, int, list[int]]:
    """Device restatement of utils.py:28-75 for given routing ids.

    Returns ``(coalesced [E*gm, H], chunk_size, lengths)`` with the
    reference's conventions; ``gm`` (if given) overrides the all-reduced max.
    With ``general_a2a`` the send buffer is compact instead — ``[sum(lengths),
    H]``, buckets back to back in expert order — and the second value is its
    row count (the input of ``run(..., general_a2a=True)``).
    """
    assert num_experts % world_size == 0, "Incorrect EP_SIZE, world_size should evenly divide num_experts."
    r = route(top_idxs, num_experts)
    if general_a2a:
        lengths = r.counts.tolist()
        total = sum(lengths)
        return pack_compact(tokens, r, total), total, lengths
    g = global_max_count(r, group) if gm is None else int(gm)
    coalesced = pack_padded(tokens, r, g)
    return coalesced, g * (num_experts // world_size), r.counts.tolist()


def recv_counts_from(counts: torch.Tensor, world_size: int, group=None) -> torch.Tensor:
    """``recv_counts[j, k]``: rows rank j sends to this rank's local expert k
    (the count all-to-all of benchmark.py:95-118)."""
    sent = counts.to(torch.int32).view(world_size, -1).contiguous()
    if world_size == 1:
        return sent.clone()
    recv = torch.empty_like(sent)
    dist.all_to_all_single(recv, sent, group=group)
    return recv


def router(x: torch.Tensor, router_w: torch.Tensor, topk: int, ids_dtype=torch.int64,
           logits: torch.Tensor | None = None, status: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """The router of utils.py:17-25 on the device (``moe_router``):
    ``softmax(einsum('bh,he->be', x, router_w))`` and its top-k.

    x [T, H] and router_w [H, E] bf16.  Returns ``(top_vals [T, K] float32,
    top_idxs [T, K])``, probabilities descending (bf16 values), equal ones by
    ascending expert id.  ``logits`` optionally supplies the [T, E] bf16
    buffer; ``status`` (a pinned int32 host tensor of one element) receives
    a device-side error word, if any."""
    if x.dtype != torch.bfloat16 or router_w.dtype != torch.bfloat16:
        raise TypeError("x and router_w must be bfloat16")
    if not x.is_cuda or router_w.device != x.device:
        raise ValueError("x and router_w must be CUDA tensors on one device")
    if ids_dtype not in (torch.int32, torch.int64):
        raise TypeError("ids_dtype must be int32 or int64")
    x = x.contiguous()
    router_w = router_w.contiguous()
    T, H = x.shape
    E = router_w.shape[1]
    if router_w.shape[0] != H:
        raise ValueError(f"router_w {tuple(router_w.shape)} does not match x {tuple(x.shape)}")
    if logits is None:
        logits = torch.empty((max(T, 1), E), dtype=torch.bfloat16, device=x.device)
    vals = torch.empty((max(T, 1), topk), dtype=torch.float32, device=x.device)
    ids = torch.empty((max(T, 1), topk), dtype=ids_dtype, device=x.device)
    N.check(N.lib().moe_router(x.data_ptr(), T, H, router_w.data_ptr(), E, topk, logits.data_ptr(), ids.data_ptr(),
                               int(ids_dtype == torch.int64), vals.data_ptr(),
                               None if status is None else status.data_ptr(), _stream_ptr(x.device)), "moe_router")
    return vals[:T], ids[:T]


def gen_weights(num_experts: int, hidden_dim: int, out_dim: int, dtype=torch.bfloat16, device="cuda"):
    """``[E, H, out]`` standard-normal expert weights (utils.py:78-80)."""
    return torch.randn(num_experts, hidden_dim, out_dim, dtype=dtype, device=device)


def gen_tensor(batch: int, seq: int, hidden_dim: int, world_size: int, num_experts: int, rank: int, topk: int,
               group=None):
    """The reference's synthetic inputs (utils.py:12-22), its router
    (utils.py:23-25: einsum, softmax, top-k) on the device through
    ``router`` where E and H are multiples of 8 (torch otherwise), and the
    device dispatch."""
    torch.manual_seed(rank)
    assert num_experts % world_size == 0, "Incorrect EP_SIZE, world_size should evenly divide num_experts."
    tokens = torch.rand(batch * seq, hidden_dim, dtype=torch.bfloat16).to("cuda")
    rw = torch.zeros(hidden_dim, num_experts, dtype=torch.bfloat16).to("cuda")
    rw = rw + torch.randn_like(rw) * 0.001
    if num_experts % 8 == 0 and hidden_dim % 8 == 0:
        _, top_idxs = router(tokens, rw, topk)
    else:
        _, top_idxs = torch.topk(F.softmax(torch.einsum("bh, he -> be", tokens, rw), dim=-1), topk)
    return dispatch(tokens, top_idxs, num_experts, world_size, group)
