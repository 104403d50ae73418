"""Drop-in ``run`` of the reference's fused all-to-all + grouped GEMM path.

Same positional signature, tensor layouts and preconditions as
alltoall_persistent_gemm.py:207-226 of the reference:

    run(rank, tokens, transmit_size, batch, seq, hidden_dim, num_experts,
        world_size, shmem=None, general_a2a=False, local_weights=None,
        recv_counts=None) -> Tensor[El, world_size*gm, out_dim]

with ``tokens`` the padded, expert-major send buffer ``[W*transmit_size, H]``
(rank d's chunk is rows ``[d*transmit_size, (d+1)*transmit_size)``, itself
``[El, gm, H]``), ``gm = transmit_size // El``, ``local_weights [El, H, N]``
and ``recv_counts [W, El]`` int32 (rows received from each source for each
local expert; all ``gm`` when omitted, alltoall_persistent_gemm.py:286-288).
Output row ``src*gm + i`` of expert ``le`` is ``recv_tokens @ W[le]`` for
``i < recv_counts[src, le]`` and exactly zero otherwise
(alltoall_persistent_gemm.py:257-258, 273-291).

``general_a2a=True`` (a stub in the reference, :221-222) runs the
unpadded exchange instead: compact send buffer in, compact output out
(``moe_ep_run_compact``; see ``run``).

The work runs in one launch of the sm_100a kernel ``moe_ep_run``
(libmoe_ep.so): counts are exchanged through the symmetric workspace, only
valid rows cross NVLink, and each GEMM tile starts when its rows have
landed.  The call is collective over the process group, is stream-ordered on
the caller's current stream, and does not synchronise the host (the
reference synchronises twice per call, :237-240).
"""
from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

from . import _native as N
from .symm import get_workspace

DEFAULT_PUSH_ROWS = int(os.environ.get("MOE_EP_PUSH_ROWS", "32"))
DEFAULT_TIMEOUT_S = float(os.environ.get("MOE_EP_TIMEOUT_S", "20"))
# Dispatch placement with more than one rank: CTAs that only push rows (0 =
# two push warps in every CTA), and experts whose local tiles run first.
DEFAULT_PUSH_CTAS = int(os.environ.get("MOE_EP_PUSH_CTAS", "0"))
# None: local tiles first at 8 ranks and more (the layer is tensor-bound
# there and the local tiles cover the first NVLink transfers; measured 1022
# against 1080 us at N=8), expert-major below (HBM-bound: the local tiles'
# weight slices would be read a second time by the remote tiles).
DEFAULT_LOCAL_FIRST = int(os.environ["MOE_EP_LOCAL_FIRST"]) if os.environ.get("MOE_EP_LOCAL_FIRST") else None
DEFAULT_PUSH_WARPS = int(os.environ.get("MOE_EP_PUSH_WARPS", "2"))
DEFAULT_PUSH_MODE = int(os.environ.get("MOE_EP_PUSH_MODE", "0"))
DEFAULT_READY_FIRST = os.environ.get("MOE_EP_READY_FIRST", "0") not in ("", "0")
# Merged tiles for small experts (decode shapes) unless switched off.
DEFAULT_MERGED = os.environ.get("MOE_EP_MERGED", "1") not in ("", "0")
# Remote row groups per expert (MOE_EP_SCHED_ROW_GROUPS bits; 0 lets the
# kernel choose W-1 groups for large experts).  1, plain feature-major, by
# default: at N=8 on Mixtral's shapes 1, 2, 3 and 7 groups measured alike
# (818-880 us, the pairs' waits for rows unchanged at about 115 us), and each
# group reads the expert's weights once more.
DEFAULT_ROW_GROUPS = int(os.environ.get("MOE_EP_ROW_GROUPS", "1"))


def placement(W: int, El: int, push_ctas: int | None = None, local_first: int | None = None) -> tuple[int, int]:
    """(push_ctas, local_first) for a launch: one rank has no rows to push
    and no remote tiles, so both are 0 there; otherwise the given values or
    the defaults, local_first clamped to the local experts."""
    if W == 1:
        return 0, 0
    pc = DEFAULT_PUSH_CTAS if push_ctas is None else int(push_ctas)
    lf = DEFAULT_LOCAL_FIRST if local_first is None else int(local_first)
    if lf is None:
        lf = El if W >= 8 else 0
    if pc < 0 or pc % 2:
        raise ValueError(f"push_ctas must be even and >= 0, got {pc}")
    return pc, max(0, min(lf, El))


def push_setup(push_warps: int | None = None, push_mode: int | None = None) -> tuple[int, int]:
    """(push_warps, push_mode): warps per CTA that move rows when no push
    CTAs are used, and the MOE_EP_PUSH_* bits (1: bulk copies in push CTAs,
    2: destination-major order, 4: computing CTAs push beside the push
    CTAs, 8: send-buffer loads and output stores evict-first in L2)."""
    pw = DEFAULT_PUSH_WARPS if push_warps is None else int(push_warps)
    pm = DEFAULT_PUSH_MODE if push_mode is None else int(push_mode)
    if not 1 <= pw <= 6 or pm & ~15:
        raise ValueError(f"push_warps must be 1..6 and push_mode a combination of the MOE_EP_PUSH_* bits 1, 2, 4, 8, "
                         f"got {pw}, {pm}")
    return pw, pm


def sched_setup(W: int, ready_first: bool | None = None, merged: bool | None = None,
                row_groups: int | None = None) -> int:
    """The MOE_EP_SCHED_* word of a launch: ready-first and merged tiles
    (only with more than one rank: one rank has no remote tiles) and the
    remote row groups in bits 4-7 (0..15; 0 lets the kernel choose)."""
    rf = DEFAULT_READY_FIRST if ready_first is None else bool(ready_first)
    mg = DEFAULT_MERGED if merged is None else bool(merged)
    rg = DEFAULT_ROW_GROUPS if row_groups is None else int(row_groups)
    if not 0 <= rg <= 15:
        raise ValueError(f"row_groups must be 0..15 (0: chosen by the kernel), got {rg}")
    return ((N.SCHED_READY_FIRST if (rf and W > 1) else 0) | (N.SCHED_MERGED if (mg and W > 1) else 0) |
            (rg << N.SCHED_ROW_GROUPS_SHIFT))


def _group_info(group, world_size: int, rank: int) -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return rank, world_size


def raise_if_device_error(ws) -> None:
    """Raise if an earlier launch on this workspace latched a device error."""
    w = ws.host_status()
    if w:
        code, site, detail = N.decode_status_word(w)
        raise N.MoeEpError(code, "moe_ep_run (device)", f"site={site} detail={detail}; the workspace is unusable")


def _launch_params(me: int, W: int, tokens: torch.Tensor, gm: int | None, transmit_size: int, hidden_dim: int,
                   local_weights: torch.Tensor, recv_counts, group, timeout_s, push_rows, num_ctas, trace,
                   ret_cols: int = 0, push_ctas: int | None = None, local_first: int | None = None,
                   send_counts: torch.Tensor | None = None, push_warps: int | None = None,
                   push_mode: int | None = None, ready_first: bool | None = None, merged: bool | None = None,
                   row_groups: int | None = None):
    """Validate the fused layer's inputs and fill ``moe_ep_run_params``.

    ``gm`` is the bound on every (rank, expert) count; ``None`` means the
    padded layout's ``transmit_size // El``.  Returns
    ``(workspace, params, (El, gm, N), keepalive)``; ``ret_cols`` > 0 selects
    a workspace with a return region (the combine path)."""
    if local_weights is None:
        raise ValueError("local_weights [El, H, N] is required")
    El, H, Nout = local_weights.shape
    if tokens.dim() != 2 or tokens.shape[1] != H or H != hidden_dim:
        raise ValueError(f"tokens {tuple(tokens.shape)} / hidden_dim {hidden_dim} do not match weights {tuple(local_weights.shape)}")
    if gm is None:
        if transmit_size % El:
            raise ValueError(f"transmit_size {transmit_size} is not a multiple of the {El} local experts")
        gm = transmit_size // El
    if tokens.dtype != torch.bfloat16 or local_weights.dtype != torch.bfloat16:
        raise TypeError("tokens and local_weights must be bfloat16")
    if local_weights.device != tokens.device:
        raise ValueError("tokens and local_weights must be on the same device")
    dev = tokens.device.index if tokens.device.index is not None else torch.cuda.current_device()
    tokens = tokens.contiguous()
    local_weights = local_weights.contiguous()
    if send_counts is not None:
        # This rank's per-expert send counts; the kernel's count exchange
        # gives every rank the whole matrix.
        if send_counts.numel() != W * El:
            raise ValueError(f"send_counts must hold {W}x{El} counts, got {tuple(send_counts.shape)}")
        recv_counts = send_counts.to(device=tokens.device, dtype=torch.int32).reshape(W, El).contiguous()
    elif recv_counts is None:
        recv_counts = torch.full((W, El), gm, dtype=torch.int32, device=tokens.device)
    else:
        if tuple(recv_counts.shape) != (W, El):
            raise ValueError(f"recv_counts must be [{W}, {El}], got {tuple(recv_counts.shape)}")
        recv_counts = recv_counts.to(device=tokens.device, dtype=torch.int32).contiguous()

    rows = push_rows or DEFAULT_PUSH_ROWS
    ws = get_workspace(W, El, H, gm, dev, group, me, rows, ret_cols)
    raise_if_device_error(ws)

    p = N.RunParams()
    p.world_size, p.rank, p.local_experts = W, me, El
    p.hidden, p.out_dim, p.elem_bytes, p.gm = H, Nout, 2, gm
    p.tokens, p.weights = tokens.data_ptr(), local_weights.data_ptr()
    p.recv_counts = recv_counts.data_ptr()
    p.peer_bases, p.local_base = ws.peer_bases.data_ptr(), ws.base
    p.cap_rows, p.push_rows, p.max_chunks = ws.key.cap_rows, ws.push_rows, ws.key.max_chunks
    p.epoch = ws.next_epoch()
    p.num_ctas = num_ctas
    p.push_ctas, p.local_first = placement(W, El, push_ctas, local_first)
    p.push_warps, p.push_mode = push_setup(push_warps, push_mode)
    p.sched_mode = sched_setup(W, ready_first, merged, row_groups)
    p.counts_are_send = int(send_counts is not None)
    p.timeout_ns = int((timeout_s if timeout_s is not None else DEFAULT_TIMEOUT_S) * 1e9)
    p.status_host = ws.status_host.data_ptr()
    if trace is not None:
        if trace.dtype != torch.int64 or not trace.is_cuda:
            raise TypeError("trace must be an int64 CUDA tensor")
        p.trace = trace.data_ptr()
    return ws, p, (El, gm, Nout), (tokens, local_weights, recv_counts)


def _general_bound(recv_counts: torch.Tensor, group) -> tuple[int, int]:
    """(rows this rank receives, MAX over the group of every count): one
    read of the W x El counts and, with more than one rank, one all-reduce."""
    rc = recv_counts.to(torch.int64)
    local = torch.stack([rc.sum(), rc.max() if rc.numel() else torch.zeros((), dtype=torch.int64,
                                                                         device=rc.device)])
    host = local.cpu()
    m = torch.tensor([int(host[1])], dtype=torch.int64, device=recv_counts.device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
    return int(host[0]), max(int(m.item()), 1)


def run(rank: int, tokens: torch.Tensor, transmit_size: int, batch: int, seq: int, hidden_dim: int,
        num_experts: int, world_size: int, shmem=None, general_a2a: bool = False,
        local_weights: torch.Tensor = None, recv_counts: torch.Tensor = None, *, group=None,
        timeout_s: float | None = None, push_rows: int | None = None, num_ctas: int = 0,
        check: bool = False, trace: torch.Tensor | None = None, max_count: int | None = None,
        recv_rows: int | None = None, push_ctas: int | None = None, local_first: int | None = None,
        send_counts: torch.Tensor | None = None, push_warps: int | None = None,
        push_mode: int | None = None, ready_first: bool | None = None, merged: bool | None = None,
        row_groups: int | None = None) -> torch.Tensor:
    """Fused dispatch + grouped GEMM; see the module docstring.

    ``general_a2a=True`` (a stub in the reference, alltoall_persistent_gemm.py:221-222)
    runs the unpadded exchange: ``tokens`` is the compact send buffer
    ``[transmit_size, H]`` of ``utils.dispatch(..., general_a2a=True)`` —
    the cells (d, le) back to back in (d, le) order — ``recv_counts`` is
    required, and the result is compact, ``[recv_counts.sum(), N]``: the
    cells (le, src) back to back in (le, src) order, ``recv_counts[src, le]``
    rows each.  Its buffers are sized by the largest count over the group
    and the output by the rows this rank receives: pass ``max_count`` (the
    same on every rank, at least every count) and ``recv_rows``
    (``recv_counts.sum()``) to keep the call free of host synchronisation;
    otherwise both are read from ``recv_counts`` (the maximum all-reduced).

    Keyword-only extensions: ``group`` (process group, default WORLD),
    ``timeout_s`` (bound on every device wait for a peer), ``push_rows``
    (rows per NVLink chunk and arrival flag), ``num_ctas`` (0 = one per SM),
    ``check`` (synchronise and raise on a device error before returning),
    ``trace`` (int64 device tensor of at least ``num_sms * 24`` words that
    receives the per-CTA device timeline, ``_native.TRACE_FIELDS``),
    ``push_ctas`` / ``local_first`` (dispatch placement, see ``placement``),
    ``push_warps`` / ``push_mode`` (how rows move, see ``push_setup``),
    ``ready_first`` (more than one rank: remote tiles whose rows have landed
    first, local tiles while none has; ``local_first`` is then ignored),
    ``merged`` (more than one rank: an expert whose local and remote rows
    together fit 128 rows gets one tile per weight slice instead of two),
    ``row_groups`` (more than one rank: an expert's remote row tiles taken in
    that many contiguous groups, each feature-major, so rows that land first
    are computed first; 0 lets the kernel choose, 1 is plain feature-major),
    ``send_counts`` (padded path only: this rank's ``[W*El]`` per-expert
    counts, i.e. the routing's ``lengths``, in place of ``recv_counts``; the
    kernel's count exchange then replaces the count all-to-all of
    benchmark.py:114-118, so no collective or host read precedes the call).
    """
    assert dist.is_initialized()
    assert tokens.is_cuda
    me, W = _group_info(group, world_size, rank)
    if W != world_size or me != rank:
        raise ValueError(f"rank/world_size ({rank}/{world_size}) disagree with the process group ({me}/{W})")
    if send_counts is not None and (general_a2a or recv_counts is not None):
        raise ValueError("send_counts replaces recv_counts and needs the padded layout (general_a2a=False)")
    if general_a2a:
        if recv_counts is None:
            raise ValueError("general_a2a needs recv_counts [W, El]")
        if tokens.shape[0] != transmit_size:
            raise ValueError(f"general_a2a: tokens has {tokens.shape[0]} rows, transmit_size is {transmit_size}")
        if max_count is None or recv_rows is None:
            rows_h, bound = _general_bound(recv_counts, group)
        out_rows = int(recv_rows) if recv_rows is not None else rows_h
        gm = max(int(max_count), 1) if max_count is not None else bound
        send_rows = tokens.shape[0]
        if send_rows == 0:  # nothing to send: any valid 16-byte-aligned row serves as the (unread) buffer
            tokens = torch.zeros((1, tokens.shape[1]), dtype=tokens.dtype, device=tokens.device)
        ws, p, (El, gm, Nout), keep = _launch_params(me, W, tokens, gm, transmit_size, hidden_dim, local_weights,
                                                     recv_counts, group, timeout_s, push_rows, num_ctas, trace,
                                                     push_ctas=push_ctas, local_first=local_first,
                                                     push_warps=push_warps, push_mode=push_mode,
                                                     ready_first=ready_first, merged=merged,
                                                     row_groups=row_groups)
        # A zero-row view has a null data_ptr; the kernel wants a real buffer.
        buf = torch.empty((max(out_rows, 1), Nout), dtype=torch.bfloat16, device=tokens.device)
        out = buf[:out_rows]
        p.out = buf.data_ptr()
        stream = torch.cuda.current_stream(tokens.device)
        N.check(N.lib().moe_ep_run_compact(ctypes.byref(p), send_rows, out_rows,
                                           ctypes.c_void_p(stream.cuda_stream)), "moe_ep_run_compact")
    else:
        assert tokens.shape[0] == transmit_size * world_size
        ws, p, (El, gm, Nout), keep = _launch_params(me, W, tokens, None, transmit_size, hidden_dim, local_weights,
                                                     recv_counts, group, timeout_s, push_rows, num_ctas, trace,
                                                     push_ctas=push_ctas, local_first=local_first,
                                                     send_counts=send_counts, push_warps=push_warps,
                                                     push_mode=push_mode, ready_first=ready_first,
                                                     merged=merged, row_groups=row_groups)
        out = torch.empty((El, W * gm, Nout), dtype=torch.bfloat16, device=tokens.device)
        p.out = out.data_ptr()
        stream = torch.cuda.current_stream(tokens.device)
        N.check(N.lib().moe_ep_run(ctypes.byref(p), ctypes.c_void_p(stream.cuda_stream)), "moe_ep_run")
    if check:
        stream.synchronize()
        raise_if_device_error(ws)
    return out


def layer(tokens: torch.Tensor, top_idxs: torch.Tensor, num_experts: int, local_weights: torch.Tensor, *,
          group=None, gm: int | None = None, **kw) -> torch.Tensor:
    """The whole path from token rows and routing ids: device routing
    (utils.py:28-41), the padded expert-major send buffer (utils.py:45-69)
    and the fused exchange + grouped GEMM (``run``), returning
    ``[El, W*gm, N]`` like ``run``.

    The only host read is the group's largest bucket, ``gm`` (an all-reduced
    MAX of the device routing's local maxima; it sizes the padded buffers, as
    ``chunk_size`` does in the reference); pass ``gm`` to skip it.  Counts
    are not exchanged on the host: ``run`` receives this rank's send counts
    and exchanges them inside the kernel.  Keyword arguments go to ``run``.
    """
    from . import utils
    me, W = _group_info(group, 1, 0)
    if num_experts % W:
        raise ValueError(f"{num_experts} experts do not split over {W} ranks")
    El = num_experts // W
    r = utils.route(top_idxs, num_experts)
    g = utils.global_max_count(r, group) if gm is None else max(int(gm), 1)
    coalesced = utils.pack_padded(tokens, r, g)
    T = int(top_idxs.shape[0])
    return run(me, coalesced, El * g, 1, T, tokens.shape[1], num_experts, W, None, False, local_weights, None,
               group=group, send_counts=r.counts, **kw)
