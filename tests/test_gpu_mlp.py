"""The full expert MLP (exchange + gate/up GEMM, SwiGLU, down GEMM) on the
GPU against the oracle's restatement.

Tolerance: bf16 inputs, two GEMMs with fp32 accumulation and a bf16
intermediate; the reference's allclose(rtol=1e-2, atol=1e-2)
(benchmark.py:143) scaled to the output's magnitude, and a maximum error of
at most 1e-2 relative to the largest reference value.
"""
import traceback

import numpy as np
import pytest
import torch

import oracle
from conftest import free_port
from nvshmem_testing_b200 import _native as N
from nvshmem_testing_b200 import mlp, utils, workloads

pytestmark = pytest.mark.gpu


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def _errs(y: torch.Tensor, ref: np.ndarray) -> list[str]:
    o = _f32(y)
    if o.shape != ref.shape:
        return [f"shape {o.shape} != {ref.shape}"]
    if not o.size:
        return []
    scale = max(float(np.abs(ref).max()), 1e-6)
    errs = []
    if not np.allclose(o, ref, rtol=1e-2, atol=1e-2 * scale):
        errs.append(f"allclose failed: max abs err {np.abs(o - ref).max():.3e} (scale {scale:.3e})")
    if float(np.abs(o - ref).max()) > 1e-2 * scale:
        errs.append(f"max rel err {float(np.abs(o - ref).max()) / scale:.3e}")
    return errs


def test_swiglu_matches_oracle():
    g = torch.Generator().manual_seed(1)
    rows, F = 3001, 136
    a = (2 * torch.randn(rows, 2 * F, generator=g)).to(torch.bfloat16)
    ad = a.cuda()
    h = torch.empty(rows, F, dtype=torch.bfloat16, device="cuda")
    N.check(N.lib().moe_swiglu(ad.data_ptr(), rows, F, h.data_ptr(), None), "moe_swiglu")
    af = _f32(a)
    gate, up = af[:, :F], af[:, F:]
    ref = oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(gate / (1 + np.exp(-gate)) * up))
    o = _f32(h)
    assert np.all(np.abs(o - ref) <= np.abs(ref) * 2.0 ** -7 + 1e-30)  # within one bf16 ulp
    assert (o == ref).mean() > 0.99


CASES = [
    # El, H, F, counts (one rank)
    (2, 256, 128, [130, 77]),
    (3, 512, 256, [0, 300, 17]),
    (4, 1024, 512, [256, 1, 128, 511]),
    (2, 128, 64, [0, 0]),
]


@pytest.mark.parametrize("El,H,F,counts", CASES)
def test_single_rank_mlp_matches_oracle(single_rank_group, El, H, F, counts):
    g = torch.Generator().manual_seed(El * 13 + H + F)
    total = sum(counts)
    tok = torch.randn(total, H, generator=g).to(torch.bfloat16)
    w13 = (0.05 * torch.randn(El, H, 2 * F, generator=g)).to(torch.bfloat16)
    w2 = (0.05 * torch.randn(El, F, H, generator=g)).to(torch.bfloat16)
    rc = torch.tensor([counts], dtype=torch.int32)
    y = mlp.run(0, tok.cuda(), total, 1, w13.cuda(), w2.cuda(), rc.cuda(), check=True)
    assert y.shape == (total, H) and y.dtype == torch.bfloat16
    ref = oracle.mlp_compact([_f32(tok)], [np.array(counts)], [_f32(w13)], [_f32(w2)])[0]
    errs = _errs(y, ref)
    assert not errs, errs
    again = mlp.run(0, tok.cuda(), total, 1, w13.cuda(), w2.cuda(), rc.cuda(), max_count=max(counts + [1]),
                    recv_rows=total)
    torch.cuda.synchronize()
    assert torch.equal(y, again)


@pytest.mark.parametrize("El,H,F,counts", [c for c in CASES if c[2] % 128 == 0])
def test_fused_swiglu_matches_separate_activation(single_rank_group, El, H, F, counts):
    """The activation in the first GEMM's epilogue (moe_ep_run_compact_swiglu)
    gives the values of the separate moe_swiglu pass: the same bf16 gate and
    up values and the same fp32 arithmetic."""
    g = torch.Generator().manual_seed(El * 7 + H + F)
    total = sum(counts)
    tok = torch.randn(total, H, generator=g).to(torch.bfloat16).cuda()
    w13 = (0.05 * torch.randn(El, H, 2 * F, generator=g)).to(torch.bfloat16).cuda()
    w2 = (0.05 * torch.randn(El, F, H, generator=g)).to(torch.bfloat16).cuda()
    rc = torch.tensor([counts], dtype=torch.int32).cuda()
    y_sep = mlp.run(0, tok, total, 1, w13, w2, rc, check=True)
    w13f = mlp.fuse_gate_up(w13)
    y_fused = mlp.run(0, tok, total, 1, w13f, w2, rc, check=True, w13_fused=True)
    y_again = mlp.run(0, tok, total, 1, w13f, w2, rc, w13_fused=True)
    torch.cuda.synchronize()
    assert y_fused.shape == y_sep.shape
    if total:
        assert (y_fused == y_sep).float().mean().item() > 0.99
        ref = oracle.mlp_compact([_f32(tok)], [np.array(counts)], [_f32(w13)], [_f32(w2)])[0]
        errs = _errs(y_fused, ref)
        assert not errs, errs
    assert torch.equal(y_fused, y_again)


def test_moe_mlp_from_routing(single_rank_group):
    wl = workloads.get("deepseek_v3", T=512, H=256, N=256, E=8)
    x = workloads.tokens(wl, 0).cuda()
    ids = workloads.top_idxs(wl, 0)
    g = torch.Generator().manual_seed(3)
    F = 128
    w13 = (0.05 * torch.randn(wl.E, wl.H, 2 * F, generator=g)).to(torch.bfloat16)
    w2 = (0.05 * torch.randn(wl.E, F, wl.H, generator=g)).to(torch.bfloat16)
    y, rc = mlp.moe_mlp(x, ids.cuda(), w13.cuda(), w2.cuda())
    c, o, p = oracle.bucketize(ids.numpy(), wl.E)
    send = oracle.compact_coalesce(_f32(x.cpu()), c, o, p)
    ref = oracle.mlp_compact([send], [c], [_f32(w13)], [_f32(w2)])[0]
    assert np.array_equal(rc.cpu().numpy(), c[None, :])
    errs = _errs(y, ref)
    assert not errs, errs


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        from nvshmem_testing_b200 import symm

        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                device_id=torch.device("cuda", rank))
        wl = workloads.get("skewed_zipf", T=512, H=256, N=256, E=8)
        El, F = wl.local_experts(world), 128
        xs = [workloads.tokens(wl, r) for r in range(world)]
        ids = [workloads.top_idxs(wl, r) for r in range(world)]
        w13s, w2s = [], []
        for r in range(world):
            g = torch.Generator().manual_seed(100 + r)
            w13s.append((0.05 * torch.randn(El, wl.H, 2 * F, generator=g)).to(torch.bfloat16))
            w2s.append((0.05 * torch.randn(El, F, wl.H, generator=g)).to(torch.bfloat16))
        errs = []
        for k in range(3):
            w13 = w13s[rank].cuda()
            fused = k == 2  # the third call with the activation in the GEMM epilogue
            y, rc = mlp.moe_mlp(xs[rank].cuda(), ids[rank].cuda(), mlp.fuse_gate_up(w13) if fused else w13,
                                w2s[rank].cuda(), timeout_s=10.0, w13_fused=fused)
            torch.cuda.synchronize()
            send, counts = [], []
            for r in range(world):
                c, o, p = oracle.bucketize(ids[r].numpy(), wl.E)
                send.append(oracle.compact_coalesce(_f32(xs[r]), c, o, p))
                counts.append(c)
            ref = oracle.mlp_compact(send, counts, [_f32(a) for a in w13s], [_f32(a) for a in w2s])[rank]
            errs += [f"call {k}: {e}" for e in _errs(y, ref)]
        dist.barrier()
        symm.release_all()
        dist.destroy_process_group()
        q.put((rank, "ok", errs))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def test_two_ranks_mlp_match_oracle():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict((r, (k, v)) for r, k, v in (q.get(timeout=600) for _ in range(2)))
    for p in procs:
        p.join(timeout=120)
    for r, (kind, payload) in sorted(out.items()):
        assert kind == "ok", f"rank {r}:\n{payload}"
        assert not payload, f"rank {r}: {payload}"
