"""The fused layer at the full per-rank shapes of the benchmark
configurations, on one GPU, against the oracle.

* DeepSeek-V3 receiver shape: H=7168, N=2048, 32 local experts with about
  1024 rows each (the per-rank GEMM of the 8-GPU layer: 4096 tokens x top-8
  over 32 experts) — the 4-D weight map, 56 k-blocks, every CTA pair;
* one Mixtral-8x7B rank: H=4096, N=14336 (56 feature slices), 8 experts;
* the skewed Zipf(1.2) workload through the unpadded exchange
  (general_a2a=True): 64 experts whose buckets differ tenfold;
* the whole path from token rows and ids (``alltoall_persistent_gemm.layer``,
  counts exchanged in the kernel) equal to ``run`` with host-exchanged
  counts.

Routing and the send buffer must match the oracle bit for bit; expert
outputs (sampled experts, every row or evenly spaced rows) within the
layer tests' tolerance: allclose(rtol=1e-2, atol=1e-2) (the reference's own
check, benchmark.py:143) and max |err| <= 1e-2 x max |ref|; padded rows
exactly zero.
"""
import numpy as np
import pytest
import torch

import oracle
from nvshmem_testing_b200 import alltoall_persistent_gemm as apg
from nvshmem_testing_b200 import utils, workloads

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2
MAX_REL = 1e-2


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _check_cells(out, tok_bits, routed, w_dev, experts, rows_per_cell, cell_rows):
    """out rows of every sampled expert against oracle.expert_cell;
    ``cell_rows(le, rows)`` maps bucket rows to output rows."""
    counts = routed[0]
    x = oracle.bf16_bits_to_f32(tok_bits)
    err = scale = 0.0
    for le in experts:
        c = int(counts[le])
        if c == 0:
            continue
        rows = np.arange(c) if rows_per_cell is None else \
            np.unique(np.linspace(0, c - 1, min(rows_per_cell, c)).round().astype(np.int64))
        w = oracle.bf16_bits_to_f32(_bits(w_dev[le]))
        ref = oracle.expert_cell(x, routed, le, w, rows)
        got = out[cell_rows(le, torch.as_tensor(rows, device="cuda"))].float().cpu().numpy()
        np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)
        err = max(err, float(np.abs(got - ref).max()))
        scale = max(scale, float(np.abs(ref).max()))
    assert err <= MAX_REL * scale, (err, scale)


def _padded_case(single_rank_group, name, over, experts, rows_per_cell):
    wl = workloads.get(name, **over)
    tok = workloads.tokens(wl, 0)
    ids = workloads.top_idxs(wl, 0)
    w = workloads.weights(wl, 0, 1, device="cuda")
    coal, chunk, lengths = utils.dispatch(tok.cuda(), ids.cuda(), wl.E, 1)
    routed = oracle.bucketize(ids.numpy(), wl.E)
    gm = chunk // wl.E
    assert lengths == routed[0].tolist() and gm == oracle.local_max(routed[0])
    tb = _bits(tok)
    assert np.array_equal(_bits(coal), oracle.pad_coalesce(tb, *routed, gm)), "send buffer differs from the oracle"
    rc = torch.tensor([lengths], dtype=torch.int32, device="cuda")
    out = apg.run(0, coal, chunk, 1, wl.T, wl.H, wl.E, 1, None, False, w, rc, check=True)
    assert out.shape == (wl.E, gm, wl.N)
    _check_cells(out, tb, routed, w, experts, rows_per_cell, lambda le, r: (le, r))
    i = torch.arange(gm, device="cuda")
    valid = i[None, :] < rc[0][:, None]
    assert out.masked_fill(valid[..., None], 0).abs().amax().item() == 0, "padded rows must be zero"
    return wl, tok, ids, w, out


def test_deepseek_v3_receiver_shape(single_rank_group):
    _padded_case(single_rank_group, "deepseek_v3", {"E": 32}, [0, 13, 31], None)


def test_mixtral_rank(single_rank_group):
    _padded_case(single_rank_group, "mixtral", {}, [0, 7], 128)


def test_skewed_zipf_general(single_rank_group):
    wl = workloads.get("skewed_zipf")
    tok = workloads.tokens(wl, 0)
    ids = workloads.top_idxs(wl, 0)
    w = workloads.weights(wl, 0, 1, device="cuda")
    compact, total, lengths = utils.dispatch(tok.cuda(), ids.cuda(), wl.E, 1, general_a2a=True)
    routed = oracle.bucketize(ids.numpy(), wl.E)
    assert lengths == routed[0].tolist()
    assert max(lengths) > 5 * (sum(lengths) / len(lengths)), "the Zipf workload should be skewed"
    tb = _bits(tok)
    assert np.array_equal(_bits(compact), oracle.compact_coalesce(tb, *routed))
    rc = torch.tensor([lengths], dtype=torch.int32, device="cuda")
    out = apg.run(0, compact, total, 1, wl.T, wl.H, wl.E, 1, None, True, w, rc, check=True)
    assert out.shape == (total, wl.N)
    starts = np.concatenate([[0], np.cumsum(lengths)])
    _check_cells(out, tb, routed, w, list(range(wl.E)), 32, lambda le, r: int(starts[le]) + r)


def test_layer_with_counts_exchanged_in_the_kernel(single_rank_group):
    """``layer`` (send counts, exchanged by the kernel) gives exactly the
    output of ``run`` with host-exchanged receive counts."""
    wl = workloads.get("deepseek_v3", E=32, T=1024)
    tok = workloads.tokens(wl, 0).cuda()
    ids = workloads.top_idxs(wl, 0).cuda()
    w = workloads.weights(wl, 0, 1, device="cuda")
    coal, chunk, lengths = utils.dispatch(tok, ids, wl.E, 1)
    rc = utils.recv_counts_from(torch.tensor(lengths, dtype=torch.int32, device="cuda"), 1)
    ref = apg.run(0, coal, chunk, 1, wl.T, wl.H, wl.E, 1, None, False, w, rc, check=True)
    for _ in range(2):
        got = apg.layer(tok, ids, wl.E, w, check=True)
        assert torch.equal(got, ref)
