"""The full expert MLP behind the exchange: gate/up GEMM, SwiGLU, down GEMM.

The reference's expert is one GEMM (``tokens @ W[e]``, baseline.py:50;
alltoall_persistent_gemm.py:16-157) whose ``out_dim`` is the FFN width of the
configurations.  An MoE layer's expert is the gated MLP
``(silu(x @ W_gate) * (x @ W_up)) @ W_down``.  ``run`` computes it for the
rows this rank receives, with three launches and no padding anywhere:

1. the fused exchange + grouped GEMM in compact mode (``moe_ep_run_compact``,
   as ``alltoall_persistent_gemm.run(..., general_a2a=True)``) with
   ``w13 [El, H, 2F]`` = [W_gate | W_up] per expert: its output is
   ``a [rows_in, 2F]``, the cells (le, src) back to back;
2. ``moe_swiglu``: ``h = silu(a[:, :F]) * a[:, F:]`` in fp32, bf16 out;
3. one rank's compact grouped GEMM (``moe_ep_run_compact`` with W=1) over the
   same rows with ``w2 [El, F, H]``: each expert's rows are already
   contiguous in ``h`` (its cells for every source), so the output keeps the
   row order of step 1.

Returns ``y [rows_in, H]`` bf16 in the compact (le, src) order of
``run(..., general_a2a=True)``.

With ``w13_fused=True`` steps 1 and 2 are one launch
(``moe_ep_run_compact_swiglu``): ``w13`` is then in the layout of
``fuse_gate_up`` and the GEMM's epilogue writes ``h`` directly, so the
[gate | up] rows never reach memory.  The values are the same.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native as N
from . import alltoall_persistent_gemm as apg
from . import utils


def fuse_gate_up(w13: torch.Tensor) -> torch.Tensor:
    """[El, H, 2F] with gate columns [0, F) and up columns [F, 2F) -> the
    layout of the SwiGLU epilogue: per 256 columns (one CTA pair's tile),
    gate j..j+63, up j..j+63, gate j+64..j+127, up j+64..j+127, so that each
    CTA holds a gate feature and its up feature.  Needs F % 128 == 0."""
    El, H, F2 = w13.shape
    F = F2 // 2
    if F2 % 2 or F % 128:
        raise ValueError(f"w13 {tuple(w13.shape)}: the fused layout needs an FFN width that is a multiple of 128")
    gate = w13[..., :F].reshape(El, H, F // 128, 2, 1, 64)
    up = w13[..., F:].reshape(El, H, F // 128, 2, 1, 64)
    return torch.cat([gate, up], dim=4).reshape(El, H, F2).contiguous()


def _exchange_swiglu(rank, W, tokens, transmit_size, H, F, w13f, recv_counts, group, max_count, rows, timeout_s,
                     push_rows, num_ctas, stream):
    """Step 1 and 2 in one launch: h [rows, F] (w13f in the fused layout)."""
    send_rows = tokens.shape[0]
    if send_rows == 0:  # nothing to send: any valid 16-byte-aligned row serves as the (unread) buffer
        tokens = torch.zeros((1, H), dtype=tokens.dtype, device=tokens.device)
    ws, p, _, keep = apg._launch_params(rank, W, tokens, max(int(max_count), 1), transmit_size, H, w13f, recv_counts,
                                        group, timeout_s, push_rows, num_ctas, None)
    h = torch.empty((max(rows, 1), F), dtype=torch.bfloat16, device=tokens.device)
    p.out = h.data_ptr()
    N.check(N.lib().moe_ep_run_compact_swiglu(ctypes.byref(p), send_rows, rows, ctypes.c_void_p(stream.cuda_stream)),
            "moe_ep_run_compact_swiglu")
    return ws, h


def run(rank: int, tokens: torch.Tensor, transmit_size: int, world_size: int, w13: torch.Tensor,
        w2: torch.Tensor, recv_counts: torch.Tensor, *, group=None, max_count: int | None = None,
        recv_rows: int | None = None, timeout_s: float | None = None, push_rows: int | None = None,
        num_ctas: int = 0, check: bool = False, w13_fused: bool = False) -> torch.Tensor:
    """Exchange + expert MLP for the rows this rank receives.

    tokens  [transmit_size, H] bf16: the compact send buffer of
            ``utils.dispatch(..., general_a2a=True)``
    w13     [El, H, 2F] bf16: gate columns [0, F), up columns [F, 2F)
    w2      [El, F, H] bf16
    recv_counts [W, El] int32.  ``max_count`` (a bound on every count, equal
    on all ranks) and ``recv_rows`` (``recv_counts.sum()``) keep the call free
    of host synchronisation; otherwise they are read from ``recv_counts``.
    """
    if w13.dim() != 3 or w2.dim() != 3:
        raise ValueError("w13 [El, H, 2F] and w2 [El, F, H] are required")
    El, H, F2 = w13.shape
    F = F2 // 2
    if F2 % 2 or tuple(w2.shape) != (El, F, H):
        raise ValueError(f"w13 {tuple(w13.shape)} and w2 {tuple(w2.shape)} do not form an MLP")
    if w2.dtype != torch.bfloat16 or w2.device != tokens.device:
        raise TypeError("w2 must be bfloat16 on the tokens' device")
    if max_count is None or recv_rows is None:
        rows_h, bound = apg._general_bound(recv_counts, group)
        max_count = bound if max_count is None else max_count
        recv_rows = rows_h if recv_rows is None else recv_rows
    stream = torch.cuda.current_stream(tokens.device)
    rows = int(recv_rows)
    if w13_fused:
        # 1+2. exchange + [gate | up] GEMM with the activation in its epilogue
        if not (dist.is_available() and dist.is_initialized()) and world_size > 1:
            raise RuntimeError("world_size > 1 needs an initialised process group")
        me, W = apg._group_info(group, world_size, rank)
        ws1, h = _exchange_swiglu(me, W, tokens, transmit_size, H, F, w13, recv_counts, group, max_count, rows,
                                  timeout_s, push_rows, num_ctas, stream)
        if check:
            stream.synchronize()
            apg.raise_if_device_error(ws1)
    else:
        kw = dict(group=group, timeout_s=timeout_s, push_rows=push_rows, num_ctas=num_ctas, check=check)
        # 1. exchange + [gate | up]
        a = apg.run(rank, tokens, transmit_size, 1, 1, H, El * world_size, world_size, None, True, w13,
                    recv_counts, max_count=max_count, recv_rows=recv_rows, **kw)
        # 2. activation
        h = torch.empty((max(rows, 1), F), dtype=torch.bfloat16, device=tokens.device)
        N.check(N.lib().moe_swiglu(a.data_ptr() if rows else h.data_ptr(), rows, F, h.data_ptr(),
                                   ctypes.c_void_p(stream.cuda_stream)), "moe_swiglu")
    # 3. down projection: one rank, expert le's rows = its cells from every source
    local_counts = recv_counts.to(torch.int32).sum(dim=0, dtype=torch.int32).view(1, El)
    gm_local = max(int(max_count), 1) * world_size
    ws, p, _, keep = apg._launch_params(0, 1, h, gm_local, rows, F, w2, local_counts, None, timeout_s, push_rows,
                                        num_ctas, None)
    y = torch.empty((max(rows, 1), H), dtype=torch.bfloat16, device=tokens.device)
    p.out = y.data_ptr()
    N.check(N.lib().moe_ep_run_compact(ctypes.byref(p), rows, rows, ctypes.c_void_p(stream.cuda_stream)),
            "moe_ep_run_compact")
    if check:
        stream.synchronize()
        apg.raise_if_device_error(ws)
    return y[:rows]


def moe_mlp(x: torch.Tensor, top_idxs: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, *, group=None,
            **kwargs) -> tuple[torch.Tensor, torch.Tensor]:
    """Route, pack (compact), exchange the counts and run the expert MLP.

    Returns ``(y [rows_in, H], recv_counts [W, El])``: y in the compact
    (le, src) order, recv_counts saying how many rows each cell holds."""
    initialised = dist.is_available() and dist.is_initialized()
    W = dist.get_world_size(group) if initialised else 1
    rank = dist.get_rank(group) if initialised else 0
    El = w13.shape[0]
    send, total, lengths = utils.dispatch(x, top_idxs, El * W, W, group, general_a2a=True)
    rc = utils.recv_counts_from(torch.tensor(lengths, dtype=torch.int32, device=x.device), W, group)
    return run(rank, send, total, W, w13, w2, rc, group=group, **kwargs), rc
