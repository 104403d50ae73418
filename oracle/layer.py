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


def ep_layer(send: list[np.ndarray], chunk: int, weights: list[np.ndarray]) -> list[np.ndarray]:
    """Whole layer for all ranks: exchange, regroup, per-expert GEMM."""
    W = len(send)
    recv = alltoall_equal(send, chunk)
    return [baseline_run(recv[r], chunk, W, weights[r]) for r in range(W)]
