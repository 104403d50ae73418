"""Routing post-processing, restated from the reference (utils.py:28-75,
benchmark.py:95-118).  Integer work: results must match bit for bit.

Rows are handled as opaque bit patterns (bf16 as uint16, fp32 as float32
or uint32), so padding and gathering are exact copies.
"""
from __future__ import annotations

import numpy as np


def bucketize(top_idxs: np.ndarray, num_experts: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """utils.py:28-41: for each expert, the ascending token ids whose top-k
    row contains it (``(top_idxs == ex).any(-1)``; a repeated id counts once,
    ids outside [0, E) match nothing).

    Returns (counts [E] int32, offsets [E+1] int32, perm [offsets[E]] int32).
    """
    ids = np.asarray(top_idxs)
    if ids.ndim == 1:
        ids = ids[:, None]
    lists = []
    for ex in range(num_experts):
        mask = (ids == ex).any(axis=-1)                        # utils.py:31
        lists.append(np.nonzero(mask)[0].astype(np.int32))     # tokens[mask]: ascending (utils.py:32)
    counts = np.array([len(x) for x in lists], dtype=np.int32)
    offsets = np.zeros(num_experts + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    perm = np.concatenate(lists) if lists else np.zeros(0, np.int32)
    return counts, offsets, perm.astype(np.int32)


def local_max(counts: np.ndarray) -> int:
    """utils.py:45: largest bucket; an empty bucket is a one-row placeholder
    (utils.py:36-41), so the result is at least 1."""
    return max(int(np.max(counts)) if counts.size else 0, 1)


def pad_coalesce(tokens: np.ndarray, counts: np.ndarray, offsets: np.ndarray, perm: np.ndarray,
                 gm: int) -> np.ndarray:
    """utils.py:54-69: bucket e in rows [e*gm, e*gm + counts[e]), zero rows
    up to (e+1)*gm, buckets concatenated expert-major."""
    E = counts.size
    out = np.zeros((E * gm,) + tokens.shape[1:], dtype=tokens.dtype)
    for e in range(E):
        c = int(counts[e])
        if c > gm:
            raise ValueError(f"bucket {e} has {c} rows > gm {gm}")
        out[e * gm:e * gm + c] = tokens[perm[offsets[e]:offsets[e] + c]]
    return out


def gen_tensor_restated(tokens: np.ndarray, top_idxs: np.ndarray, num_experts: int, world_size: int,
                        gm: int | None = None) -> tuple[np.ndarray, int, list[int]]:
    """utils.py:28-75 for given tokens and routing ids: (coalesced,
    chunk_size, lengths).  ``gm`` defaults to the local max, as the
    reference computes it; pass the all-ranks max for a consistent exchange."""
    assert num_experts % world_size == 0
    counts, offsets, perm = bucketize(top_idxs, num_experts)
    g = local_max(counts) if gm is None else int(gm)
    return pad_coalesce(tokens, counts, offsets, perm, g), g * (num_experts // world_size), counts.tolist()


def recv_counts_matrix(all_counts: list[np.ndarray], rank: int, world_size: int) -> np.ndarray:
    """benchmark.py:95-118: recv_counts[j, k] = rows rank j sends to local
    expert k of `rank` (expert e lives on rank e // El)."""
    E = int(np.asarray(all_counts[0]).size)
    El = E // world_size
    return np.stack([np.asarray(all_counts[j], np.int32)[rank * El:(rank + 1) * El]
                     for j in range(world_size)]).astype(np.int32)


# ---------------------------------------------------------------- general (unpadded) all-to-all
# The reference leaves general_a2a unimplemented (alltoall_persistent_gemm.py:221-222,
# baseline.py:15-16); the unpadded layout restated here is the padded one of
# utils.py:54-69 with the zero rows removed.

def compact_coalesce(tokens: np.ndarray, counts: np.ndarray, offsets: np.ndarray, perm: np.ndarray) -> np.ndarray:
    """Every bucket back to back in expert order, no padding:
    rows [offsets[e], offsets[e] + counts[e]) hold bucket e."""
    n = int(offsets[-1]) if len(offsets) else 0
    return tokens[perm[:n]]


def uncompact_padded(padded: np.ndarray, counts: np.ndarray, gm: int) -> np.ndarray:
    """The compact form of a padded expert-major buffer (drop rows >= counts[e])."""
    return np.concatenate([padded[e * gm:e * gm + int(c)] for e, c in enumerate(counts)]) if len(counts) else padded[:0]
