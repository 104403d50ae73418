"""Router (moe_router: logits GEMM on tcgen05, softmax, top-k) on the GPU.

* against the reference's own router (golden vectors of utils.py:17-25 run
  on CPU): logits within one bf16 ulp, top-k values within one ulp, and
  every selection a valid top-k of the reference's probabilities — the
  reference's 0.001-scale router makes many probabilities equal, and
  torch.topk orders equal values arbitrarily, so ids are compared tie-aware;
* against the oracle on larger, untied routers at the configurations'
  shapes (DeepSeek-V3 T=4096, H=7168, E=256, top-8; Mixtral E=8, top-2);
* the routing it feeds (counts, permutation) equals routing the oracle's ids.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN
from nvshmem_testing_b200 import _native as N
from nvshmem_testing_b200 import utils

pytestmark = pytest.mark.gpu


def _bits_to_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def _close_bf16(a: np.ndarray, b: np.ndarray, noise=1e-6) -> np.ndarray:
    """Elementwise: equal within one bf16 ulp plus ``noise`` (the fp32
    summation-order noise of the logits GEMM)."""
    return np.abs(a - b) <= np.maximum(np.abs(a), np.abs(b)) * 2.0 ** -7 + noise


def _gemm_noise(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Per-logit bound on the difference two fp32 summation orders make:
    a few fp32 ulps of sum |x_h w_h|, growing like sqrt(H)."""
    return 2.0 ** -22 * np.sqrt(x.shape[1]) * (np.abs(x) @ np.abs(w))


@pytest.mark.parametrize("ids_dtype", [torch.int64, torch.int32])
def test_router_matches_reference_golden(ids_dtype):
    g = np.load(GOLDEN / "router_golden.npz")
    f = oracle.bf16_bits_to_f32
    for ci in range(int(g["num_cases"][0])):
        p = f"c{ci}_"
        b, s, h, e, k, w, r = (int(x) for x in g[p + "shape"])
        x = _bits_to_bf16(g[p + "tokens"]).cuda()
        rw = _bits_to_bf16(g[p + "router"]).cuda()
        logits = torch.empty((b * s, e), dtype=torch.bfloat16, device="cuda")
        vals, ids = utils.router(x, rw, k, ids_dtype=ids_dtype, logits=logits)
        assert vals.shape == (b * s, k) and ids.dtype == ids_dtype
        ref_logits, ref_probs, ref_vals = f(g[p + "logits"]), f(g[p + "probs"]), f(g[p + "top_vals"])
        lg = _f32(logits)
        assert _close_bf16(lg, ref_logits).all(), ci
        assert (lg == ref_logits).mean() > 0.99, ci
        v = _f32(vals)
        assert np.all(np.diff(v, axis=-1) <= 0), ci
        assert oracle.topk_mismatches(ids.cpu().numpy(), v, ref_probs, ref_vals, ulps=1) == 0, ci


CASES = [
    # T, H, E, K, router scale
    (4096, 7168, 256, 8, 0.05),   # DeepSeek-V3 router shape
    (1000, 4096, 8, 2, 0.05),     # Mixtral router shape
    (777, 512, 64, 6, 0.1),
    (33, 256, 1024, 32, 0.1),
    (5, 64, 16, 16, 0.1),
]


@pytest.mark.parametrize("T,H,E,K,scale", CASES)
def test_router_matches_oracle(T, H, E, K, scale):
    gen = torch.Generator().manual_seed(T + E)
    x = torch.randn(T, H, generator=gen).to(torch.bfloat16)
    rw = (scale * torch.randn(H, E, generator=gen)).to(torch.bfloat16)
    logits = torch.empty((T, E), dtype=torch.bfloat16, device="cuda")
    vals, ids = utils.router(x.cuda(), rw.cuda(), K, logits=logits)
    # The GEMM: logits within one bf16 ulp plus summation-order noise.
    ref_logits = oracle.router(_f32(x), _f32(rw), K)[0]
    lg = _f32(logits)
    assert _close_bf16(lg, ref_logits, _gemm_noise(_f32(x), _f32(rw))).all()
    assert (lg == ref_logits).mean() > 0.99
    # Softmax and top-k, on the device's own logits (with logits near 8 one
    # bf16 ulp of a logit is 0.0625, i.e. 6 % of its probability, so the
    # probabilities are compared from the same logits).
    ref_probs, ref_vals, ref_ids = oracle.softmax_topk(lg, K)
    v = _f32(vals)
    assert _close_bf16(v, ref_vals).all()
    assert oracle.topk_mismatches(ids.cpu().numpy(), v, ref_probs, ref_vals, ulps=1) == 0
    # with a router this wide, equal or near-equal probabilities are rare: the
    # ids themselves agree almost everywhere
    assert (ids.cpu().numpy() == ref_ids).mean() > 0.99


def test_router_feeds_routing():
    """Routing the router's ids gives the oracle's buckets of those ids."""
    gen = torch.Generator().manual_seed(9)
    T, H, E, K = 2048, 1024, 64, 6
    x = torch.randn(T, H, generator=gen).to(torch.bfloat16).cuda()
    rw = (0.05 * torch.randn(H, E, generator=gen)).to(torch.bfloat16).cuda()
    _, ids = utils.router(x, rw, K)
    r = utils.route(ids, E)
    c, o, p = oracle.bucketize(ids.cpu().numpy(), E)
    assert np.array_equal(r.counts.cpu().numpy(), c)
    assert np.array_equal(r.perm[: int(o[-1])].cpu().numpy(), p)


def test_router_edge_cases():
    x = torch.zeros(0, 64, dtype=torch.bfloat16, device="cuda")
    rw = torch.zeros(64, 16, dtype=torch.bfloat16, device="cuda")
    vals, ids = utils.router(x, rw, 4)
    assert vals.shape == (0, 4) and ids.shape == (0, 4)
    # all-equal logits: probabilities 1/E, ids ascending
    x1 = torch.ones(3, 64, dtype=torch.bfloat16, device="cuda")
    vals, ids = utils.router(x1, rw, 4)
    assert ids.cpu().tolist() == [[0, 1, 2, 3]] * 3
    assert torch.allclose(vals.cpu(), torch.full((3, 4), 1 / 16))
    with pytest.raises(N.MoeEpError):  # E must be a multiple of 8
        utils.router(x1, torch.zeros(64, 12, dtype=torch.bfloat16, device="cuda"), 2)
    with pytest.raises(N.MoeEpError):  # K > E
        utils.router(x1, rw, 17)
