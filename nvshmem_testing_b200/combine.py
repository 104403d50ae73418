"""The layer with its return path: dispatch, expert GEMM, return, combine.

The reference's path ends at the expert outputs ``[El, W*gm, N]`` on each
expert's rank (alltoall_persistent_gemm.py:207-309, baseline.py:8-56); its
router computes top-k weights (utils.py:24-25, ``top_vals``) that nothing
uses.  The step after the path is the reverse exchange of every output row to
the rank that sent the token, followed by the top-k weighted sum per token:

    y[t, :] = sum_k top_vals[t, k] * (x_t @ W_{top_idxs[t, k]})

over the distinct ids of the row that lie in [0, E) (the routing's own rule,
utils.py:31 ``.any(-1)``); a token with no such id gets a zero row.

``run`` takes the send buffer and counts of ``alltoall_persistent_gemm.run``
plus the token-level routing (``top_idxs``, ``top_vals`` and the ``slots`` of
``utils.route(..., with_slots=True)``) and returns ``y [T, N]`` bf16 on the
token's own rank.  One C call, ``moe_ep_run_combine``, launches the fused
kernel in return mode — its epilogue stores each output row straight into
the source rank's return region over NVLink, at the row of that rank's padded
send buffer that held the token — and then the combine kernel, which waits
for every peer's "returned" flag and forms ``y`` in fp32.  Nothing is
synchronised on the host.

``moe_layer`` is the whole layer from activations and router output.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native as N
from . import utils
from .alltoall_persistent_gemm import _group_info, _launch_params, raise_if_device_error


def run(rank: int, tokens: torch.Tensor, transmit_size: int, world_size: int, local_weights: torch.Tensor,
        recv_counts: torch.Tensor, top_idxs: torch.Tensor, top_vals: torch.Tensor, slots: torch.Tensor, *,
        group=None, timeout_s: float | None = None, push_rows: int | None = None, num_ctas: int = 0,
        check: bool = False, trace: torch.Tensor | None = None) -> torch.Tensor:
    """Dispatch + expert GEMM + return + top-k combine.

    tokens        [W*transmit_size, H] bf16: this rank's padded send buffer
                  (``utils.pack_padded`` of the routing below)
    local_weights [El, H, N] bf16
    recv_counts   [W, El] int32: rows this rank receives per (source, expert)
    top_idxs      [T, K] int32/int64: this rank's expert ids (E = El * W)
    top_vals      [T, K] float32 or bf16: router weights
    slots         [T, K] int32: ``utils.route(top_idxs, E, with_slots=True).slots``
    Returns ``y [T, N]`` bf16.  Collective over the process group.
    """
    if world_size > 1 and not (dist.is_available() and dist.is_initialized()):
        raise RuntimeError("world_size > 1 needs an initialised process group")
    if not tokens.is_cuda:
        raise ValueError("tokens must be a CUDA tensor")
    if tokens.shape[0] != transmit_size * world_size:
        raise ValueError(f"tokens has {tokens.shape[0]} rows, expected transmit_size * world_size")
    me, W = _group_info(group, world_size, rank)
    if W != world_size or me != rank:
        raise ValueError(f"rank/world_size ({rank}/{world_size}) disagree with the process group ({me}/{W})")
    if top_idxs.dim() == 1:
        top_idxs = top_idxs[:, None]
    if top_vals.dim() == 1:
        top_vals = top_vals[:, None]
    if slots.dim() == 1:
        slots = slots[:, None]
    T, K = top_idxs.shape
    if tuple(top_vals.shape) != (T, K) or tuple(slots.shape) != (T, K):
        raise ValueError(f"top_vals {tuple(top_vals.shape)} and slots {tuple(slots.shape)} must match top_idxs {(T, K)}")
    if top_idxs.dtype not in (torch.int32, torch.int64) or slots.dtype != torch.int32:
        raise TypeError("top_idxs must be int32/int64 and slots int32")
    if top_vals.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("top_vals must be float32 or bfloat16")
    for name, t in (("top_idxs", top_idxs), ("top_vals", top_vals), ("slots", slots)):
        if t.device != tokens.device:
            raise ValueError(f"{name} must be on {tokens.device}")
    if local_weights is None or local_weights.dim() != 3:
        raise ValueError("local_weights [El, H, N] is required")
    Nout = local_weights.shape[2]
    ws, p, (El, gm, Nout), keep = _launch_params(me, W, tokens, None, transmit_size, tokens.shape[1], local_weights,
                                                 recv_counts, group, timeout_s, push_rows, num_ctas, trace,
                                                 ret_cols=Nout)
    ids, vals, sl = top_idxs.contiguous(), top_vals.contiguous(), slots.contiguous()
    y = torch.empty((T, Nout), dtype=torch.bfloat16, device=tokens.device)
    c = N.CombineParams()
    c.top_idxs, c.top_vals, c.slots, c.y = ids.data_ptr(), vals.data_ptr(), sl.data_ptr(), y.data_ptr()
    c.T, c.K, c.ret_rows = T, K, ws.key.ret_rows
    c.ids_are_int64 = int(ids.dtype == torch.int64)
    c.vals_are_bf16 = int(vals.dtype == torch.bfloat16)
    stream = torch.cuda.current_stream(tokens.device)
    N.check(N.lib().moe_ep_run_combine(ctypes.byref(p), ctypes.byref(c), ctypes.c_void_p(stream.cuda_stream)),
            "moe_ep_run_combine")
    if check:
        stream.synchronize()
        raise_if_device_error(ws)
    return y


def moe_layer(x: torch.Tensor, top_idxs: torch.Tensor, top_vals: torch.Tensor, local_weights: torch.Tensor, *,
              group=None, **kwargs) -> torch.Tensor:
    """``y [T, N]`` of the whole expert-parallel layer for this rank's tokens.

    Routes on the device (counts, permutation, slots), all-reduces the
    padded bucket size (one host read, like ``utils.dispatch``), packs the
    padded send buffer, exchanges the count matrix row (NCCL all-to-all of
    W*El ints) and calls ``run``.  Extra keywords go to ``run``.
    """
    initialised = dist.is_available() and dist.is_initialized()
    W = dist.get_world_size(group) if initialised else 1
    rank = dist.get_rank(group) if initialised else 0
    El = local_weights.shape[0]
    r = utils.route(top_idxs, El * W, with_slots=True)
    gm = utils.global_max_count(r, group)
    send = utils.pack_padded(x, r, gm)
    rc = utils.recv_counts_from(r.counts, W, group)
    return run(rank, send, El * gm, W, local_weights, rc, top_idxs, top_vals, r.slots, group=group, **kwargs)
