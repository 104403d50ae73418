"""Fused layer on one rank (W=1: local tiles only) against the oracle.

Tolerance: bf16 inputs, fp32 accumulation, bf16 output; the kernel must
satisfy the reference's own check, allclose(rtol=1e-2, atol=1e-2)
(benchmark.py:143), and a maximum error of at most 1e-2 relative to the
largest reference magnitude.  Padded rows must be exactly zero.
"""
import numpy as np
import pytest
import torch

import oracle
from nvshmem_testing_b200 import alltoall_persistent_gemm as apg
from nvshmem_testing_b200 import baseline as bl

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2
MAX_REL = 1e-2


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _make(El, H, N, gm, counts, seed):
    g = torch.Generator().manual_seed(seed)
    tok = torch.zeros(El * gm, H)
    for e, c in enumerate(counts):
        tok[e * gm:e * gm + c] = torch.randn(c, H, generator=g)
    tok = tok.to(torch.bfloat16)
    w = (0.02 * torch.randn(El, H, N, generator=g)).to(torch.bfloat16)
    return tok, w


def _oracle(tok, w, gm, counts, W=1):
    x = oracle.bf16_bits_to_f32(_bits(tok))
    wt = oracle.bf16_bits_to_f32(_bits(w))
    ref = oracle.baseline_run(x, gm * w.shape[0], W, wt)
    return ref


def _assert_close(out, ref, counts_rows):
    o = out.float().cpu().numpy()
    valid = counts_rows  # boolean [El, rows]
    np.testing.assert_allclose(o[valid], ref[valid], rtol=RTOL, atol=ATOL)
    scale = max(float(np.abs(ref[valid]).max()) if valid.any() else 1.0, 1e-6)
    assert float(np.abs(o[valid] - ref[valid]).max(initial=0.0)) <= MAX_REL * scale
    assert not o[~valid].any(), "padded rows must be exactly zero"


CASES = [
    # El, H, N, gm, counts
    (2, 64, 256, 128, [128, 128]),
    (3, 72, 200, 200, [0, 131, 200]),
    (5, 256, 520, 300, [1, 299, 128, 129, 0]),
    (4, 1024, 1024, 512, [512, 7, 385, 256]),
    (1, 4096, 256, 130, [130]),
]


@pytest.mark.parametrize("El,H,N,gm,counts", CASES)
def test_run_single_rank_matches_oracle(single_rank_group, El, H, N, gm, counts):
    tok, w = _make(El, H, N, gm, counts, seed=El * 1000 + H)
    rc = torch.tensor([counts], dtype=torch.int32)
    out = apg.run(0, tok.cuda(), El * gm, 1, El * gm, H, El, 1, None, False, w.cuda(), rc.cuda(), check=True)
    assert out.shape == (El, gm, N) and out.dtype == torch.bfloat16
    ref = _oracle(tok, w, gm, counts)
    valid = np.zeros((El, gm), bool)
    for e, c in enumerate(counts):
        valid[e, :c] = True
    _assert_close(out, ref, valid)


def test_run_repeated_calls_are_stable(single_rank_group):
    El, H, N, gm, counts = 3, 128, 256, 160, [160, 33, 97]
    tok, w = _make(El, H, N, gm, counts, seed=7)
    rc = torch.tensor([counts], dtype=torch.int32).cuda()
    first = apg.run(0, tok.cuda(), El * gm, 1, El * gm, H, El, 1, None, False, w.cuda(), rc)
    for _ in range(5):
        again = apg.run(0, tok.cuda(), El * gm, 1, El * gm, H, El, 1, None, False, w.cuda(), rc)
    torch.cuda.synchronize()
    assert torch.equal(first, again)


def test_l2_stream_hints_give_the_same_output(single_rank_group):
    """push_mode=8 (evict-first L2 hints on the output's stores) changes
    no bit of the output."""
    El, H, N, gm, counts = 5, 256, 520, 300, [1, 299, 128, 129, 0]
    tok, w = _make(El, H, N, gm, counts, seed=21)
    rc = torch.tensor([counts], dtype=torch.int32).cuda()
    plain = apg.run(0, tok.cuda(), El * gm, 1, El * gm, H, El, 1, None, False, w.cuda(), rc, check=True)
    hinted = apg.run(0, tok.cuda(), El * gm, 1, El * gm, H, El, 1, None, False, w.cuda(), rc, check=True,
                     push_mode=8)
    assert torch.equal(plain, hinted)


def test_baseline_entry_point_treats_all_rows_valid(single_rank_group):
    El, H, N, gm = 2, 128, 128, 64
    tok, w = _make(El, H, N, gm, [64, 64], seed=11)
    out = bl.run(0, tok.cuda(), El * gm, 1, El * gm, H, El, 1, False, None, w.cuda())
    ref = _oracle(tok, w, gm, [64, 64])
    _assert_close(out, ref, np.ones((El, gm), bool))
    assert bl.run(0, tok.cuda(), El * gm, 1, El * gm, H, El, 1, True, None, w.cuda()) is None


@pytest.mark.parametrize("El,H,N,gm,counts", CASES + [(3, 64, 128, 8, [0, 0, 0])])
def test_general_a2a_single_rank_matches_oracle(single_rank_group, El, H, N, gm, counts):
    """general_a2a=True: compact send buffer in, compact [(le, src) cells]
    out, no padding anywhere."""
    g = torch.Generator().manual_seed(El * 77 + H)
    total = sum(counts)
    tok = torch.randn(total, H, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(El, H, N, generator=g)).to(torch.bfloat16)
    rc = torch.tensor([counts], dtype=torch.int32)
    out = apg.run(0, tok.cuda(), total, 1, total, H, El, 1, None, True, w.cuda(), rc.cuda(), check=True)
    assert out.shape == (total, N) and out.dtype == torch.bfloat16
    ref = oracle.compact_layer([oracle.bf16_bits_to_f32(_bits(tok))], [np.array(counts)],
                               [oracle.bf16_bits_to_f32(_bits(w))])[0]
    if total:
        o = out.float().cpu().numpy()
        np.testing.assert_allclose(o, ref, rtol=RTOL, atol=ATOL)
        assert float(np.abs(o - ref).max()) <= MAX_REL * max(float(np.abs(ref).max()), 1e-6)


def test_general_a2a_requires_counts(single_rank_group):
    with pytest.raises(ValueError):
        apg.run(0, torch.zeros(2, 8, device="cuda", dtype=torch.bfloat16), 2, 1, 2, 8, 1, 1, None, True,
                torch.zeros(1, 8, 8, device="cuda", dtype=torch.bfloat16))
