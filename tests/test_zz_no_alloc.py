"""moe_ep_run_noalloc, the entry point for callers that cannot allocate
device memory (a host that only has this C ABI and no CUDA allocator, a
process whose device memory is fixed after start-up, a single-GPU user who
does not want the exportable cuMem workspace).  It keeps the kernel's control
words in a fixed array inside the library instead of a caller-allocated
workspace.

Checked through the C ABI against the regular entry point (the drop-in
``run``, whose workspace is allocated) on the same inputs, on two calls in a
row with different routing, within the layer tests' tolerance.  Kept in its
own file so that it is collected after every other test."""
import ctypes

import numpy as np
import pytest
import torch

from nvshmem_testing_b200 import _native as N
from nvshmem_testing_b200 import alltoall_persistent_gemm as apg

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2


def _inputs(El, H, Nn, gm, counts, seed):
    g = torch.Generator().manual_seed(seed)
    tok = torch.zeros(El * gm, H)
    for e, c in enumerate(counts):
        tok[e * gm:e * gm + c] = torch.randn(c, H, generator=g)
    w = 0.02 * torch.randn(El, H, Nn, generator=g)
    rc = torch.tensor([counts], dtype=torch.int32)
    return tok.to(torch.bfloat16).cuda(), w.to(torch.bfloat16).cuda(), rc.cuda()


def _noalloc(tok, w, rc, El, H, Nn, gm, status, out=None):
    if out is None:
        out = torch.full((El, gm, Nn), 7.0, dtype=torch.bfloat16, device="cuda")  # stale values must be overwritten
    p = N.RunParams()
    p.world_size, p.rank, p.local_experts = 1, 0, El
    p.hidden, p.out_dim, p.elem_bytes, p.gm = H, Nn, 2, gm
    p.tokens, p.weights, p.recv_counts, p.out = tok.data_ptr(), w.data_ptr(), rc.data_ptr(), out.data_ptr()
    p.timeout_ns = 10_000_000_000
    p.status_host = status.data_ptr()
    rc_code = N.lib().moe_ep_run_noalloc(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc_code == N.OK, N.STATUS_NAMES.get(rc_code, rc_code)
    return out


def test_noalloc_matches_the_allocating_entry_point(single_rank_group):
    El, H, Nn, gm = 5, 384, 520, 200
    status = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    for call, counts in enumerate(([200, 0, 131, 17, 64], [3, 199, 0, 128, 200])):
        tok, w, rc = _inputs(El, H, Nn, gm, counts, seed=100 + call)
        got = _noalloc(tok, w, rc, El, H, Nn, gm, status)
        ref = apg.run(0, tok, El * gm, 1, El * gm, H, El, 1, None, False, w, rc, check=True)
        torch.cuda.synchronize()
        assert int(status[0]) == 0, hex(int(status[0]))
        g, r = got.float().cpu().numpy(), ref.float().cpu().numpy()
        valid = np.zeros((El, gm), bool)
        for e, c in enumerate(counts):
            valid[e, :c] = True
        np.testing.assert_allclose(g[valid], r[valid], rtol=RTOL, atol=ATOL)
        scale = max(float(np.abs(r[valid]).max()), 1e-6)
        assert float(np.abs(g[valid] - r[valid]).max()) <= 1e-2 * scale
        assert not g[~valid].any(), "padded rows must be zero"


def _check(got, ref, counts, El, gm):
    g, r = got.float().cpu().numpy(), ref.float().cpu().numpy()
    valid = np.zeros((El, gm), bool)
    for e, c in enumerate(counts):
        valid[e, :c] = True
    np.testing.assert_allclose(g[valid], r[valid], rtol=RTOL, atol=ATOL)
    scale = max(float(np.abs(r[valid]).max()), 1e-6)
    assert float(np.abs(g[valid] - r[valid]).max()) <= 1e-2 * scale
    assert not g[~valid].any(), "padded rows must be zero"


def test_noalloc_calls_queued_back_to_back(single_rank_group):
    """Two calls with different counts queued on one stream with no
    synchronisation between them: the second call's preparation of the shared
    array runs after the first kernel, in stream order."""
    El, H, Nn, gm = 4, 256, 384, 160
    status = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    cases = ([160, 3, 0, 77], [1, 159, 160, 40])
    ins = [_inputs(El, H, Nn, gm, c, seed=300 + i) for i, c in enumerate(cases)]
    outs = [_noalloc(tok, w, rc, El, H, Nn, gm, status) for tok, w, rc in ins]
    torch.cuda.synchronize()
    assert int(status[0]) == 0, hex(int(status[0]))
    for (tok, w, rc), got, counts in zip(ins, outs, cases):
        ref = apg.run(0, tok, El * gm, 1, El * gm, H, El, 1, None, False, w, rc, check=True)
        _check(got, ref, counts, El, gm)


def test_noalloc_reports_a_device_error_then_recovers(single_rank_group):
    """A count above gm is caught by the kernel's own check of the count
    table before it touches memory: MOE_EP_BAD_ARG (site: the count table)
    appears in the caller's status word.  The next valid call starts from a
    cleared array and succeeds."""
    El, H, Nn, gm = 3, 128, 256, 64
    status = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    tok, w, _ = _inputs(El, H, Nn, gm, [64, 64, 64], seed=9)
    bad = torch.tensor([[10, gm + 1, 5]], dtype=torch.int32, device="cuda")
    _noalloc(tok, w, bad, El, H, Nn, gm, status)
    torch.cuda.synchronize()
    code, site, detail = N.decode_status_word(int(status[0]) & 0xFFFFFFFF)
    assert code == N.BAD_ARG and site == 2, (code, site, detail)
    status[0] = 0
    counts = [64, 17, 0]
    tok, w, rc = _inputs(El, H, Nn, gm, counts, seed=10)
    got = _noalloc(tok, w, rc, El, H, Nn, gm, status)
    torch.cuda.synchronize()
    assert int(status[0]) == 0, hex(int(status[0]))
    ref = apg.run(0, tok, El * gm, 1, El * gm, H, El, 1, None, False, w, rc, check=True)
    _check(got, ref, counts, El, gm)


def test_noalloc_requires_a_status_word():
    p = N.RunParams()
    p.world_size, p.rank, p.local_experts = 1, 0, 2
    p.hidden, p.out_dim, p.elem_bytes, p.gm = 64, 64, 2, 16
    assert N.lib().moe_ep_run_noalloc(ctypes.byref(p), None) == N.BAD_ARG


def test_noalloc_rejects_sizes_beyond_its_scratch():
    p = N.RunParams()
    p.world_size, p.rank, p.local_experts = 1, 0, N.NOALLOC_MAX_EXPERTS + 1
    p.hidden, p.out_dim, p.elem_bytes, p.gm = 64, 64, 2, 16
    assert N.lib().moe_ep_run_noalloc(ctypes.byref(p), None) == N.SCRATCH_LIMIT
    assert N.lib().moe_ep_status_string(N.SCRATCH_LIMIT) == b"size exceeds the fixed scratch of moe_ep_run_noalloc"
    p.local_experts, p.world_size = 4, 2  # one rank only
    assert N.lib().moe_ep_run_noalloc(ctypes.byref(p), None) == N.BAD_ARG
