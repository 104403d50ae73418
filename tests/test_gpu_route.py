"""Routing kernels against the oracle and the reference's golden vectors:
counts, offsets, permutation and the padded pack must match bit for bit."""
import hashlib

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN
from nvshmem_testing_b200 import utils, workloads

pytestmark = pytest.mark.gpu


def _check(ids_cpu: torch.Tensor, E: int, dtype=torch.int64):
    ids = ids_cpu.to(dtype).cuda()
    r = utils.route(ids, E)
    c, o, p = oracle.bucketize(ids_cpu.numpy(), E)
    assert np.array_equal(r.counts.cpu().numpy(), c)
    assert np.array_equal(r.offsets.cpu().numpy(), o)
    assert np.array_equal(r.perm[: int(o[-1])].cpu().numpy(), p)
    assert int(r.max_count.item()) == (int(c.max()) if c.size else 0)
    return r, c, o, p


def test_route_and_pack_match_reference_golden():
    g = np.load(GOLDEN / "routing_golden.npz")
    for ci in range(int(g["num_cases"][0])):
        pre = f"c{ci}_"
        b, s, h, e, k, w, rk = (int(x) for x in g[pre + "shape"])
        ids = torch.from_numpy(g[pre + "top_idxs"].astype(np.int64))
        r, c, o, p = _check(ids, e)
        tok = torch.from_numpy(g[pre + "tokens"].view(np.int16)).view(torch.bfloat16).cuda()
        gm = max(int(c.max()), 1)
        coal = utils.pack_padded(tok, r, gm)
        bits = coal.cpu().view(torch.int16).numpy().view(np.uint16)
        assert hashlib.sha256(bits.tobytes()).digest() == g[pre + "coalesced_sha256"].tobytes(), ci


@pytest.mark.parametrize("name", ["cpu_gloo", "mixtral", "deepseek_v3", "skewed_zipf", "decode"])
@pytest.mark.parametrize("rank", [0, 3])
def test_route_full_size_configs(name, rank):
    wl = workloads.get(name)
    ids = workloads.top_idxs(wl, rank)
    _check(ids, wl.E)
    _check(ids, wl.E, torch.int32)


@pytest.mark.parametrize("T", [16, 64, 256, 1024, 4096, 8192])
def test_route_decode_sweep(T):
    wl = workloads.get("decode", T=T)
    _check(workloads.top_idxs(wl, 1), wl.E)


def test_route_edge_cases():
    # duplicates within a row count once; ids outside [0, E) are dropped
    _check(torch.tensor([[1, 1], [0, 3], [7, -1], [3, 0], [2, 2]]), 4)
    # single token, single expert
    _check(torch.tensor([[0]]), 1)
    # many tokens spanning several bitmap chunks, all on one expert
    _check(torch.zeros(5000, 2, dtype=torch.int64), 3)
    # E at its maximum
    g = torch.Generator().manual_seed(3)
    _check(torch.randint(0, 1024, (3000, 4), generator=g), 1024)
    # ragged: T not a multiple of the chunk, many empty experts
    _check(torch.randint(0, 5, (1031, 3), generator=g), 700)


def test_pack_zero_fills_and_matches_oracle_fp32():
    g = torch.Generator().manual_seed(5)
    T, H, E, K = 300, 96, 12, 3
    ids = torch.rand(T, E, generator=g).topk(K).indices
    tok = torch.randn(T, H, generator=g)
    r, c, o, p = _check(ids, E)
    gm = int(c.max()) + 7
    out = utils.pack_padded(tok.cuda(), r, gm).cpu().numpy()
    ref = oracle.pad_coalesce(tok.numpy(), c, o, p, gm)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_dispatch_matches_gen_tensor_restated(single_rank_group):
    wl = workloads.get("deepseek_v3", T=1024, H=256)
    tok = workloads.tokens(wl, 0)
    ids = workloads.top_idxs(wl, 0)
    coal, chunk, lengths = utils.dispatch(tok.cuda(), ids.cuda(), wl.E, 1)
    ref, rchunk, rlen = oracle.gen_tensor_restated(tok.view(torch.int16).numpy(), ids.numpy(), wl.E, 1)
    assert chunk == rchunk and lengths == rlen
    assert np.array_equal(coal.cpu().view(torch.int16).numpy(), ref)


def test_route_spans_every_cta_of_the_cluster():
    """Token counts below, at and above the cluster's CTA count and chunk
    size: each CTA routes a contiguous token range, so ranks inside a bucket
    must continue across CTA boundaries."""
    g = torch.Generator().manual_seed(5)
    for T in (1, 7, 8, 9, 511, 512, 513, 4095, 4097, 40000):
        _check(torch.randint(0, 37, (T, 3), generator=g), 37)
        _check(torch.randint(0, 1024, (T, 2), generator=g), 1024, dtype=torch.int32)


def test_publish_reaches_pinned_host_memory():
    """moe_publish_i32: a device word copied by a kernel into pinned host
    memory, read after an event (the routing's one host read)."""
    import ctypes
    from nvshmem_testing_b200 import _native as N
    src = torch.tensor([7, -3, 123456], dtype=torch.int32, device="cuda")
    host = torch.zeros(3, dtype=torch.int32, pin_memory=True)
    N.check(N.lib().moe_publish_i32(src.data_ptr(), 3, host.data_ptr(),
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "moe_publish_i32")
    ev = torch.cuda.Event()
    ev.record()
    ev.synchronize()
    assert host.tolist() == [7, -3, 123456]
