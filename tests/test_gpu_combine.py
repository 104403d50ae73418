"""Return path (combine) on the GPU against the oracle.

* route slots: bit-exact against the oracle's restatement;
* one rank: ``combine.moe_layer`` (route, pack, fused kernel in return
  mode, combine kernel) against ``oracle.combine_layer``;
* several ranks (spawned, one per GPU): every rank's y against the oracle
  over all ranks' inputs;
* a peer that never runs: the call ends with MOE_EP_TIMEOUT in the status
  word and the context stays usable.

Tolerance: bf16 inputs and expert outputs, fp32 accumulation, bf16 y; the
reference's own check allclose(rtol=1e-2, atol=1e-2) (benchmark.py:143) and
a maximum error of at most 1e-2 relative to the largest reference value.
Tokens without a valid expert id must give exactly zero rows.
"""
import ctypes
import os
import traceback

import numpy as np
import pytest
import torch

import oracle
from conftest import free_port
from nvshmem_testing_b200 import combine, utils, workloads

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2
MAX_REL = 1e-2


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _compare(y: torch.Tensor, ref: np.ndarray, ids: np.ndarray, E: int) -> list[str]:
    errs = []
    o = _f32(y)
    if o.shape != ref.shape:
        return [f"shape {o.shape} != {ref.shape}"]
    routed = ((ids >= 0) & (ids < E)).any(axis=1) if ids.size else np.zeros(0, bool)
    if o.size:
        if not np.allclose(o, ref, rtol=RTOL, atol=ATOL):
            errs.append(f"allclose failed: max abs err {np.abs(o - ref).max():.3e}")
        scale = max(float(np.abs(ref).max()), 1e-6)
        rel = float(np.abs(o - ref).max()) / scale
        if rel > MAX_REL:
            errs.append(f"max rel err {rel:.3e}")
        if o[~routed].any():
            errs.append("unrouted tokens must give zero rows")
    return errs


@pytest.mark.parametrize("E,K", [(8, 2), (5, 3), (64, 8), (4, 1)])
@pytest.mark.parametrize("dtype", [torch.int64, torch.int32])
def test_route_slots_match_oracle(E, K, dtype):
    g = torch.Generator().manual_seed(E * 31 + K)
    T = 3000
    ids = torch.rand(T, E, generator=g).topk(K, dim=-1).indices
    if K > 1:  # plant repeats and out-of-range ids
        ids[::7, 1] = ids[::7, 0]
        ids[3::11, 0] = E + 3
        ids[5::13, K - 1] = -1
    r = utils.route(ids.to(dtype).cuda(), E, with_slots=True)
    assert np.array_equal(r.slots.cpu().numpy(), oracle.route_slots(ids.numpy(), E))
    r0 = utils.route(ids.to(dtype).cuda(), E)
    n = int(r0.offsets[-1])  # perm holds offsets[E] valid entries
    assert torch.equal(r0.perm[:n], r.perm[:n]) and torch.equal(r0.counts, r.counts)


CASES = [
    # T, H, N, E, K, vals dtype, id pattern
    (300, 256, 384, 8, 2, torch.float32, "uniform"),
    (257, 128, 136, 5, 3, torch.bfloat16, "planted"),
    (64, 512, 256, 4, 1, torch.float32, "uniform"),
    (1000, 1024, 1024, 16, 4, torch.float32, "uniform"),
    (96, 256, 256, 6, 2, torch.float32, "none"),
    (0, 256, 256, 4, 2, torch.float32, "uniform"),
]


def _ids(T, E, K, pattern, seed):
    g = torch.Generator().manual_seed(seed)
    if T == 0:
        return torch.zeros(0, K, dtype=torch.int64)
    ids = torch.rand(T, E, generator=g).topk(K, dim=-1).indices
    if pattern == "planted":
        ids[::5, 1] = ids[::5, 0]      # repeated id: counts once
        ids[2::9, 2] = E + 1           # out of range: skipped
        ids[4::17, :] = -1             # no valid id: zero row
    elif pattern == "none":
        ids[:] = -1
    return ids


@pytest.mark.parametrize("T,H,N,E,K,vdt,pattern", CASES)
def test_single_rank_combine_matches_oracle(single_rank_group, T, H, N, E, K, vdt, pattern):
    g = torch.Generator().manual_seed(T + H + N)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(E, H, N, generator=g)).to(torch.bfloat16)
    ids = _ids(T, E, K, pattern, seed=E + K)
    vals = torch.rand(T, K, generator=g).to(vdt)
    y = combine.moe_layer(x.cuda(), ids.cuda(), vals.cuda(), w.cuda(), check=True)
    assert y.shape == (T, N) and y.dtype == torch.bfloat16
    ref = oracle.combine_layer([_f32(x)], [ids.numpy()], [_f32(vals)], [_f32(w)])[0]
    errs = _compare(y, ref, ids.numpy(), E)
    assert not errs, errs


def test_combine_repeated_and_mixed_with_run(single_rank_group):
    """Epochs advance across calls; the return-mode workspace is separate
    from the plain one, so alternating entry points stays correct."""
    from nvshmem_testing_b200 import alltoall_persistent_gemm as apg
    T, H, N, E, K = 512, 256, 256, 4, 2
    g = torch.Generator().manual_seed(5)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    w = (0.02 * torch.randn(E, H, N, generator=g)).to(torch.bfloat16).cuda()
    ids = torch.rand(T, E, generator=g).topk(K, dim=-1).indices.cuda()
    vals = torch.rand(T, K, generator=g).cuda()
    first = combine.moe_layer(x, ids, vals, w)
    for _ in range(4):
        coal, chunk, lengths = utils.dispatch(x, ids, E, 1)
        apg.run(0, coal, chunk, 1, T, H, E, 1, None, False, w, torch.tensor([lengths], dtype=torch.int32).cuda())
        again = combine.moe_layer(x, ids, vals, w)
    torch.cuda.synchronize()
    assert torch.equal(first, again)


def _worker(rank, world, port, cases, q):
    try:
        import torch.distributed as dist
        from nvshmem_testing_b200 import symm

        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                device_id=torch.device("cuda", rank))
        results = []
        for name, over in cases:
            wl = workloads.get(name, **over)
            xs = [workloads.tokens(wl, r) for r in range(world)]
            ids = [workloads.top_idxs(wl, r) for r in range(world)]
            vals = [workloads.top_vals(wl, r) for r in range(world)]
            wts = [workloads.weights(wl, r, world) for r in range(world)]
            ys = [combine.moe_layer(xs[rank].cuda(), ids[rank].cuda(), vals[rank].cuda(), wts[rank].cuda(),
                                    timeout_s=10.0) for _ in range(3)]
            torch.cuda.synchronize()
            ref = oracle.combine_layer([_f32(a) for a in xs], [a.numpy() for a in ids], [a.numpy() for a in vals],
                                       [_f32(a) for a in wts])[rank]
            errs = []
            for k, y in enumerate(ys):
                errs += [f"call {k}: {e}" for e in _compare(y, ref, ids[rank].numpy(), wl.E)]
            results.append((name, errs))
        dist.barrier()
        symm.release_all()
        dist.destroy_process_group()
        q.put((rank, "ok", results))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def _spawn(world, cases):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cases, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, kind, payload = q.get(timeout=600)
        out[rank] = (kind, payload)
    for p in procs:
        p.join(timeout=120)
    for r, (kind, payload) in sorted(out.items()):
        assert kind == "ok", f"rank {r}:\n{payload}"
        for name, errs in payload:
            assert not errs, f"rank {r} {name}: {errs}"


MULTI_CASES = [
    ("deepseek_v3", {"T": 256, "H": 256, "N": 384, "E": 16}),
    ("skewed_zipf", {"T": 512, "H": 128, "N": 136, "E": 8}),
    ("decode", {"T": 16, "H": 256, "N": 256}),
]


def test_two_ranks_combine_match_oracle():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _spawn(2, MULTI_CASES)


def test_all_visible_ranks_combine_match_oracle():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 3:
        pytest.skip("needs 3+ GPUs")
    n = 8 if n >= 8 else (4 if n >= 4 else 2)
    _spawn(n, [("deepseek_v3", {"T": 128, "H": 256, "N": 256, "E": 32})])


def test_missing_peer_times_out_in_combine(single_rank_group):
    """W=2 return-mode launch on one GPU where rank 1 never runs: the count
    wait expires, MOE_EP_TIMEOUT is latched, the combine kernel sees the
    error and returns at once, and the context keeps working."""
    from nvshmem_testing_b200 import _native as N

    W, El, H, Nn, gm, T, K = 2, 2, 64, 64, 16, 8, 2
    L = N.lib()
    ret_rows = W * El * gm
    layout = N.workspace_layout(W, El, H, 2, (W - 1) * El * gm, 1, ret_rows, Nn)
    mapped, base, fd, handle = ctypes.c_size_t(), ctypes.c_uint64(), ctypes.c_int(), ctypes.c_uint64()
    N.check(L.moe_symm_alloc(0, layout.total_bytes, ctypes.byref(mapped), ctypes.byref(base), ctypes.byref(fd),
                             ctypes.byref(handle)), "alloc")
    os.close(fd.value)
    try:
        N.check(L.moe_ep_workspace_reset(base.value, ctypes.byref(layout), None), "reset")
        torch.cuda.synchronize()
        peers = torch.tensor([base.value, base.value], dtype=torch.int64, device="cuda")
        tok = torch.zeros(W * El * gm, H, dtype=torch.bfloat16, device="cuda")
        w = torch.zeros(El, H, Nn, dtype=torch.bfloat16, device="cuda")
        rc = torch.full((W, El), 3, dtype=torch.int32, device="cuda")
        ids = torch.zeros(T, K, dtype=torch.int64, device="cuda")
        vals = torch.ones(T, K, dtype=torch.float32, device="cuda")
        slots = torch.zeros(T, K, dtype=torch.int32, device="cuda")
        y = torch.empty(T, Nn, dtype=torch.bfloat16, device="cuda")
        status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        p = N.RunParams()
        p.world_size, p.rank, p.local_experts, p.hidden, p.out_dim, p.elem_bytes, p.gm = W, 0, El, H, Nn, 2, gm
        p.tokens, p.weights, p.recv_counts, p.out = tok.data_ptr(), w.data_ptr(), rc.data_ptr(), None
        p.peer_bases, p.local_base = peers.data_ptr(), base.value
        p.cap_rows, p.push_rows, p.max_chunks, p.epoch = (W - 1) * El * gm, 16, 1, 1
        p.num_ctas, p.timeout_ns, p.status_host = 4, 200_000_000, status_host.data_ptr()
        c = N.CombineParams()
        c.top_idxs, c.top_vals, c.slots, c.y = ids.data_ptr(), vals.data_ptr(), slots.data_ptr(), y.data_ptr()
        c.T, c.K, c.ret_rows, c.ids_are_int64, c.vals_are_bf16 = T, K, ret_rows, 1, 0
        N.check(L.moe_ep_run_combine(ctypes.byref(p), ctypes.byref(c), None), "launch")
        torch.cuda.synchronize()  # returns: every wait is bounded
        word = ctypes.c_uint32()
        N.check(L.moe_ep_read_status(base.value, ctypes.byref(layout), ctypes.byref(word)), "status")
        code, site, detail = N.decode_status_word(word.value)
        assert code == N.TIMEOUT, hex(word.value)
        assert site == 1 and detail == 1  # count exchange, waiting for rank 1
        x = torch.randn(64, 64, device="cuda")
        assert torch.allclose(x @ torch.eye(64, device="cuda"), x)
    finally:
        torch.cuda.synchronize()
        L.moe_symm_free(base.value, mapped.value, handle.value)
