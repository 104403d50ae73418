"""The expert-parallel layer, restated from the reference's NCCL baseline
(baseline.py:18-50) with the exchange done in-process.

Floating-point work: fp32 accumulation of bf16 (or fp32) inputs, compared
against the device result within the stated tolerance.
"""
from __future__ import annotations

import numpy as np


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32, exactly."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns with round-to-nearest-even (finite inputs)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def alltoall_equal(send: list[np.ndarray], chunk: int) -> list[np.ndarray]:
    """dist.all_to_all_single with equal splits (baseline.py:23): rank r
    receives rank j's rows [r*chunk, (r+1)*chunk) at [j*chunk, (j+1)*chunk)."""
    W = len(send)
    return [np.concatenate([send[j][r * chunk:(r + 1) * chunk] for j in range(W)]) for r in range(W)]


def baseline_run(recv: np.ndarray, chunk: int, world_size: int, weights: np.ndarray) -> np.ndarray:
    """baseline.py:33-50 on one rank: view [W, El, gm, H], permute to
    [El, W, gm, H], flatten to [El, W*gm, H], bmm with [El, H, N] in fp32."""
    El = weights.shape[0]
    gm = chunk // El
    H = recv.shape[-1]
    x = recv.reshape(world_size, El, gm, H).transpose(1, 0, 2, 3).reshape(El, world_size * gm, H)
    return np.matmul(x.astype(np.float32), weights.astype(np.float32))


def expert_cell(tokens: np.ndarray, routing: tuple, expert: int, weights: np.ndarray,
                rows: np.ndarray | None = None) -> np.ndarray:
    """One (source rank, expert) cell of the layer output, in fp32: the
    source's tokens routed to ``expert`` in ascending token order
    (utils.py:30-32; ``routing`` = ``bucketize`` of the source's ids) times
    the expert's weights [H, N] (baseline.py:50).  ``rows`` selects rows of
    the cell by their index inside the bucket."""
    counts, offsets, perm = routing
    idx = perm[offsets[expert]:offsets[expert] + counts[expert]]
    if rows is not None:
        idx = idx[np.asarray(rows, np.int64)]
    return np.asarray(tokens[idx], np.float32) @ np.asarray(weights, np.float32)


def ep_layer(send: list[np.ndarray], chunk: int, weights: list[np.ndarray]) -> list[np.ndarray]:
    """Whole layer for all ranks: exchange, regroup, per-expert GEMM."""
    W = len(send)
    recv = alltoall_equal(send, chunk)
    return [baseline_run(recv[r], chunk, W, weights[r]) for r in range(W)]


# ---------------------------------------------------------------- return path
# The step after the reference's path: expert outputs go back to the rank
# that sent each token and are summed with the router's top-k weights
# (top_vals, computed at utils.py:24-25 and unused by the reference).  The
# selection rule is the routing's (utils.py:31): a repeated id counts once,
# ids outside [0, E) are skipped.  The expert output is rounded to bf16 (the
# dtype the layer stores it in) before the fp32 weighted sum.

def route_slots(top_idxs: np.ndarray, num_experts: int) -> np.ndarray:
    """[T, K] int32: the row of token t inside bucket top_idxs[t, k] (its
    index in the ascending token list of that expert), -1 for a repeated or
    out-of-range id."""
    from .routing import bucketize
    ids = np.asarray(top_idxs)
    if ids.ndim == 1:
        ids = ids[:, None]
    counts, offsets, perm = bucketize(ids, num_experts)
    T, K = ids.shape
    slots = np.full((T, K), -1, np.int32)
    for t in range(T):
        seen = set()
        for k in range(K):
            e = int(ids[t, k])
            if e < 0 or e >= num_experts or e in seen:
                continue
            seen.add(e)
            bucket = perm[offsets[e]:offsets[e + 1]]
            slots[t, k] = int(np.searchsorted(bucket, t))
    return slots


def _bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def combine_layer(x: list[np.ndarray], ids: list[np.ndarray], vals: list[np.ndarray],
                  weights: list[np.ndarray]) -> list[np.ndarray]:
    """y[r] [T_r, N] fp32 (before the final bf16 rounding) for every rank r:
    y[t] = sum over distinct valid ids e of row t of vals[t, k] * bf16(x[t] @ W_e),
    with expert e held by rank e // El as weights[e // El][e % El]."""
    W = len(x)
    El = weights[0].shape[0]
    E = El * W
    out = []
    for r in range(W):
        xr = np.asarray(x[r], np.float32)
        idr = np.asarray(ids[r])
        if idr.ndim == 1:
            idr = idr[:, None]
        vr = np.asarray(vals[r], np.float32).reshape(idr.shape)
        T, K = idr.shape
        y = np.zeros((T, weights[0].shape[2]), np.float32)
        first = np.ones((T, K), bool)
        for k in range(K):
            for j in range(k):
                first[:, k] &= idr[:, j] != idr[:, k]
        for e in range(E):
            for k in range(K):
                sel = np.nonzero((idr[:, k] == e) & first[:, k])[0]
                if sel.size == 0:
                    continue
                rows = _bf16_round(xr[sel] @ weights[e // El][e % El].astype(np.float32))
                y[sel] += vr[sel, k][:, None] * rows
        out.append(y)
    return out


def combine_from_outputs(outs: list[np.ndarray], ids: list[np.ndarray], vals: list[np.ndarray],
                         gm: int) -> list[np.ndarray]:
    """The same combine read from the layer's own outputs: outs[o] is rank o's
    [El, W*gm, N] result of ``ep_layer`` (row src*gm + j of expert le is the
    j-th token that rank src routed to expert o*El + le)."""
    W = len(outs)
    El = outs[0].shape[0]
    E = El * W
    res = []
    for r in range(W):
        idr = np.asarray(ids[r])
        if idr.ndim == 1:
            idr = idr[:, None]
        vr = np.asarray(vals[r], np.float32).reshape(idr.shape)
        slots = route_slots(idr, E)
        T, K = idr.shape
        y = np.zeros((T, outs[0].shape[2]), np.float32)
        for t in range(T):
            for k in range(K):
                if slots[t, k] < 0:
                    continue
                e = int(idr[t, k])
                y[t] += vr[t, k] * _bf16_round(outs[e // El][e % El, r * gm + slots[t, k]])
        res.append(y)
    return res


# ---------------------------------------------------------------- general (unpadded) all-to-all

def compact_layer(send: list[np.ndarray], all_counts: list[np.ndarray], weights: list[np.ndarray]) -> list[np.ndarray]:
    """The layer on compact buffers.  send[r] is rank r's compact send buffer
    (cells (d, le) back to back in (d, le) order, all_counts[r][d*El + le]
    rows each); the result for rank r is [sum of its received rows, N] with
    the cells (le, src) back to back in (le, src) order: cell (le, src) is
    send[src]'s cell (r, le) @ weights[r][le], in fp32."""
    W = len(send)
    El = weights[0].shape[0]
    starts = [np.concatenate([[0], np.cumsum(np.asarray(c, np.int64))]) for c in all_counts]
    outs = []
    for r in range(W):
        parts = []
        for le in range(El):
            w = weights[r][le].astype(np.float32)
            for src in range(W):
                cell = r * El + le
                rows = send[src][starts[src][cell]:starts[src][cell + 1]].astype(np.float32)
                parts.append(rows @ w)
        outs.append(np.concatenate(parts) if parts else np.zeros((0, weights[r].shape[2]), np.float32))
    return outs


def compact_from_padded(out: np.ndarray, recv_counts: np.ndarray) -> np.ndarray:
    """[El, W*gm, N] padded layer output -> compact [(le, src) cells, N]."""
    El, rows, N = out.shape
    W = recv_counts.shape[0]
    gm = rows // W
    return np.concatenate([out[le, src * gm:src * gm + int(recv_counts[src, le])]
                           for le in range(El) for src in range(W)])


# ---------------------------------------------------------------- router
# utils.py:17-25: logits = einsum('bh,he->be', tokens, router) in bf16,
# softmax over experts (bf16 result), top-k.  Restated with fp32
# accumulation rounded once to bf16 for the logits, an fp32 softmax rounded
# to bf16, and top-k ordered by (probability descending, expert ascending);
# the reference's torch.topk leaves the order of equal values unspecified,
# so ``topk_mismatches`` compares selections tie-aware.

def router(tokens: np.ndarray, router_w: np.ndarray, k: int):
    """Returns (logits, probs, top_vals, top_idxs): logits and probs are
    bf16-valued float32 [T, E]; top_vals [T, k] float32, top_idxs [T, k] int64."""
    x = np.asarray(tokens, np.float32)
    r = np.asarray(router_w, np.float32)
    logits = _bf16_round(x @ r)
    return (logits,) + softmax_topk(logits, k)


def softmax_topk(logits: np.ndarray, k: int):
    """The router after its GEMM: (probs, top_vals, top_idxs) of bf16-valued logits."""
    logits = np.asarray(logits, np.float32)
    T, E = logits.shape
    if T == 0:
        return logits.copy(), np.zeros((0, k), np.float32), np.zeros((0, k), np.int64)
    e = np.exp(logits - logits.max(axis=-1, keepdims=True))
    probs = _bf16_round(e / e.sum(axis=-1, keepdims=True))
    order = np.lexsort((np.broadcast_to(np.arange(E), probs.shape), -probs), axis=-1)
    ids = order[:, :k].astype(np.int64)
    return probs, np.take_along_axis(probs, ids, axis=-1), ids


def topk_mismatches(ids: np.ndarray, vals: np.ndarray, probs: np.ndarray, ref_vals: np.ndarray,
                    ulps: int = 0) -> int:
    """Tokens whose selection is not a valid top-k of ``probs``: the ids
    must be distinct, ``vals`` must equal the reference's sorted top values
    and the probabilities the ids point at (both within ``ulps`` bf16 ulps)."""
    ids = np.asarray(ids, np.int64)
    tol = np.abs(ref_vals) * (ulps * 2.0 ** -7) if ulps else 0.0  # a bf16 ulp is 2^-8..2^-7 of the value
    picked = np.take_along_axis(probs, ids, axis=-1)
    ok = (np.abs(vals - ref_vals) <= tol) & (np.abs(picked - ref_vals) <= tol)
    s = np.sort(ids, axis=-1)
    distinct = (s[:, 1:] != s[:, :-1]).all(axis=-1) if ids.shape[1] > 1 else np.ones(ids.shape[0], bool)
    return int((~(ok.all(axis=-1) & distinct)).sum())


# ---------------------------------------------------------------- expert MLP
# The gated expert MLP around the exchange (the reference's expert is the
# single GEMM of baseline.py:50): a = x @ [W_gate | W_up] (bf16 out),
# h = silu(gate) * up (fp32, bf16 out), y = h @ W_down (fp32).

def mlp_compact(send: list[np.ndarray], all_counts: list[np.ndarray], w13: list[np.ndarray],
                w2: list[np.ndarray]) -> list[np.ndarray]:
    """Per rank r: [rows received, H] in the compact (le, src) cell order of
    ``compact_layer``; w13[r] [El, H, 2F], w2[r] [El, F, H]."""
    from .routing import recv_counts_matrix
    W = len(send)
    El = w13[0].shape[0]
    F = w13[0].shape[2] // 2
    first = compact_layer(send, all_counts, w13)
    outs = []
    for r in range(W):
        a = _bf16_round(first[r])
        g, u = a[:, :F], a[:, F:]
        h = _bf16_round((g / (1.0 + np.exp(-g))) * u)
        rcm = recv_counts_matrix(all_counts, r, W)
        per_expert = rcm.sum(axis=0)
        starts = np.concatenate([[0], np.cumsum(per_expert)])
        y = np.zeros((h.shape[0], w2[r].shape[2]), np.float32)
        for le in range(El):
            y[starts[le]:starts[le + 1]] = h[starts[le]:starts[le + 1]] @ w2[r][le].astype(np.float32)
        outs.append(y)
    return outs
