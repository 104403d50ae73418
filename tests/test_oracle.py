"""The oracle against the reference's own outputs (golden fixtures) and its
own edge cases.  CPU only."""
import hashlib

import numpy as np
import pytest
import torch

import oracle
from nvshmem_testing_b200 import workloads
from conftest import GOLDEN


def _routing_cases():
    g = np.load(GOLDEN / "routing_golden.npz")
    return g, int(g["num_cases"][0])


def test_routing_matches_reference_gen_tensor():
    """utils.gen_tensor of the reference, bit for bit: lengths, chunk_size and
    the coalesced tensor (SHA-256), with the reference's local max as gm."""
    g, n = _routing_cases()
    assert n >= 10
    for ci in range(n):
        p = f"c{ci}_"
        b, s, h, e, k, w, r = (int(x) for x in g[p + "shape"])
        tokens = g[p + "tokens"]
        ids = g[p + "top_idxs"].astype(np.int64)
        assert tokens.shape == (b * s, h) and ids.shape == (b * s, k)
        coalesced, chunk, lengths = oracle.gen_tensor_restated(tokens, ids, e, w)
        assert lengths == g[p + "lengths"].tolist(), ci
        assert chunk == int(g[p + "chunk"][0]), ci
        assert coalesced.shape[0] == int(g[p + "coalesced_rows"][0]), ci
        digest = hashlib.sha256(np.ascontiguousarray(coalesced).tobytes()).digest()
        assert digest == g[p + "coalesced_sha256"].tobytes(), ci
        if p + "coalesced" in g:
            assert np.array_equal(coalesced, g[p + "coalesced"])


def test_layer_matches_reference_baseline_run():
    """baseline.run of the reference under gloo (2 CPU ranks, fp32)."""
    g = np.load(GOLDEN / "layer_golden.npz")
    W = int(g["world"][0])
    gm = int(g["gm"][0])
    wl = workloads.get("cpu_gloo")
    El = wl.E // W
    send, wts = [], []
    for r in range(W):
        tok = workloads.tokens(wl, r).numpy()
        wt = workloads.weights(wl, r, W).numpy()
        assert hashlib.sha256(tok.tobytes()).digest() == g[f"r{r}_tokens_sha256"].tobytes()
        assert hashlib.sha256(wt.tobytes()).digest() == g[f"r{r}_weights_sha256"].tobytes()
        ids = workloads.top_idxs(wl, r).numpy()
        assert np.array_equal(ids, g[f"r{r}_top_idxs"].astype(np.int64))
        counts, offsets, perm = oracle.bucketize(ids, wl.E)
        assert np.array_equal(counts, g[f"r{r}_counts"])
        send.append(oracle.pad_coalesce(tok, counts, offsets, perm, gm))
        wts.append(wt)
    outs = oracle.ep_layer(send, gm * El, wts)
    for r in range(W):
        ref = g[f"r{r}_out"]
        assert outs[r].shape == ref.shape
        np.testing.assert_allclose(outs[r], ref, rtol=1e-5, atol=1e-5)


def test_bucketize_dedup_and_out_of_range():
    ids = np.array([[1, 1], [0, 3], [7, -1], [3, 0], [2, 2]])
    counts, offsets, perm = oracle.bucketize(ids, 4)
    assert counts.tolist() == [2, 1, 1, 2]
    assert offsets.tolist() == [0, 2, 3, 4, 6]
    assert perm.tolist() == [1, 3, 0, 4, 1, 3]


def test_bucketize_empty_and_ragged():
    counts, offsets, perm = oracle.bucketize(np.zeros((0, 2), np.int64), 3)
    assert counts.tolist() == [0, 0, 0] and perm.size == 0
    assert oracle.local_max(counts) == 1
    tok = np.arange(10, dtype=np.uint16).reshape(5, 2)
    ids = np.array([[0], [0], [2], [0], [2]])
    c, o, p = oracle.bucketize(ids, 3)
    out = oracle.pad_coalesce(tok, c, o, p, 3)
    assert out.shape == (9, 2)
    assert out[:3].tolist() == [[0, 1], [2, 3], [6, 7]]
    assert not out[3:6].any()
    assert out[6:8].tolist() == [[4, 5], [8, 9]] and not out[8].any()


def test_pad_rejects_small_gm():
    ids = np.array([[0], [0]])
    c, o, p = oracle.bucketize(ids, 1)
    with pytest.raises(ValueError):
        oracle.pad_coalesce(np.zeros((2, 4), np.uint16), c, o, p, 1)


def test_recv_counts_matrix():
    a = [np.array([1, 2, 3, 4]), np.array([5, 6, 7, 8])]
    assert oracle.recv_counts_matrix(a, 0, 2).tolist() == [[1, 2], [5, 6]]
    assert oracle.recv_counts_matrix(a, 1, 2).tolist() == [[3, 4], [7, 8]]


def test_bf16_round_trip():
    x = np.array([1.0, -2.5, 3.140625, 1e-3, 65504.0], np.float32)
    bits = oracle.f32_to_bf16_bits(x)
    t = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bits, t)
    back = oracle.bf16_bits_to_f32(bits)
    assert np.array_equal(back, torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).float().numpy())


@pytest.mark.parametrize("name", ["mixtral", "deepseek_v3", "skewed_zipf", "decode", "cpu_gloo"])
def test_workload_routing_properties(name):
    wl = workloads.get(name, T=min(workloads.get(name).T, 512))
    ids = workloads.top_idxs(wl, 0)
    assert ids.shape == (wl.T, wl.K)
    assert int(ids.min()) >= 0 and int(ids.max()) < wl.E
    if wl.K > 1:  # distinct experts per token
        s = torch.sort(ids, dim=1).values
        assert bool((s[:, 1:] != s[:, :-1]).all())


def test_zipf_is_skewed_and_shared_across_ranks():
    wl = workloads.get("skewed_zipf", T=2048)
    c0 = np.bincount(workloads.top_idxs(wl, 0).flatten().numpy(), minlength=wl.E)
    c1 = np.bincount(workloads.top_idxs(wl, 1).flatten().numpy(), minlength=wl.E)
    assert c0.max() > 4 * np.median(c0)
    assert np.argmax(c0) == np.argmax(c1)  # same popularity order on every rank


def test_route_slots_known_answer():
    ids = np.array([[1, 1], [0, 3], [7, -1], [3, 0], [2, 2]])
    assert oracle.route_slots(ids, 4).tolist() == [[0, -1], [0, 0], [-1, -1], [1, 1], [0, -1]]
    assert oracle.route_slots(np.zeros((0, 3), np.int64), 5).shape == (0, 3)


def test_combine_matches_reference_layer_outputs():
    """The combine restatement against the reference's own baseline.run
    outputs (golden): gathering each token's rows out of the reference's
    [El, W*gm, N] results and weighting them gives the same y as the direct
    per-token formula of the oracle."""
    g = np.load(GOLDEN / "layer_golden.npz")
    W = int(g["world"][0])
    gm = int(g["gm"][0])
    wl = workloads.get("cpu_gloo")
    xs, ids, vals, wts = [], [], [], []
    for r in range(W):
        xs.append(workloads.tokens(wl, r).numpy())
        ids.append(workloads.top_idxs(wl, r).numpy())
        vals.append(workloads.top_vals(wl, r).numpy())
        wts.append(workloads.weights(wl, r, W).numpy())
    outs = [g[f"r{r}_out"] for r in range(W)]
    via_ref = oracle.combine_from_outputs(outs, ids, vals, gm)
    direct = oracle.combine_layer(xs, ids, vals, wts)
    for r in range(W):
        assert direct[r].shape == (wl.T, wl.N)
        np.testing.assert_allclose(direct[r], via_ref[r], rtol=1e-2, atol=1e-3)
        assert np.abs(direct[r]).max() > 0


def test_combine_edge_cases():
    """Repeated ids count once, out-of-range ids and unrouted tokens give
    zero contributions, top-k weights scale linearly."""
    rng = np.random.default_rng(3)
    H, N, El, W = 16, 24, 2, 2
    x = [rng.standard_normal((5, H)).astype(np.float32) for _ in range(W)]
    w = [rng.standard_normal((El, H, N)).astype(np.float32) for _ in range(W)]
    ids = [np.array([[0, 0], [3, -1], [9, 7], [1, 2], [2, 3]]), np.array([[1, 3], [0, 0], [2, 1], [3, 3], [-5, 0]])]
    v = [rng.random((5, 2)).astype(np.float32) for _ in range(W)]
    y = oracle.combine_layer(x, ids, v, w)
    bf = lambda a: oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(a))
    np.testing.assert_allclose(y[0][0], v[0][0, 0] * bf(x[0][0] @ w[0][0]), rtol=1e-6)
    np.testing.assert_allclose(y[0][1], v[0][1, 0] * bf(x[0][1] @ w[1][1]), rtol=1e-6)
    assert not y[0][2].any()
    y2 = oracle.combine_layer(x, ids, [2 * a for a in v], w)
    np.testing.assert_allclose(y2[1], 2 * y[1], rtol=1e-6)


def test_compact_layer_matches_reference_layer_outputs():
    """The unpadded (general all-to-all) restatement against the reference's
    own baseline.run outputs (golden): removing the padding from the
    reference's [El, W*gm, N] results gives the compact layer's rows."""
    g = np.load(GOLDEN / "layer_golden.npz")
    W = int(g["world"][0])
    gm = int(g["gm"][0])
    wl = workloads.get("cpu_gloo")
    send, counts, wts = [], [], []
    for r in range(W):
        tok = workloads.tokens(wl, r).numpy()
        c, o, p = oracle.bucketize(workloads.top_idxs(wl, r).numpy(), wl.E)
        compact = oracle.compact_coalesce(tok, c, o, p)
        assert np.array_equal(compact, oracle.uncompact_padded(oracle.pad_coalesce(tok, c, o, p, gm), c, gm))
        send.append(compact)
        counts.append(c)
        wts.append(workloads.weights(wl, r, W).numpy())
    outs = oracle.compact_layer(send, counts, wts)
    for r in range(W):
        rcm = oracle.recv_counts_matrix(counts, r, W)
        ref = oracle.compact_from_padded(g[f"r{r}_out"], rcm)
        assert outs[r].shape == (int(rcm.sum()), wl.N)
        np.testing.assert_allclose(outs[r], ref, rtol=1e-5, atol=1e-5)


def test_router_matches_reference_router():
    """The router restatement against the reference's own router
    (utils.py:17-25, run on CPU; golden): logits and probabilities bit for
    bit (a rare logit may differ by one bf16 ulp through the summation
    order), top-k values equal, and every selection a valid top-k of the
    reference's probabilities (the reference's tiny router makes many
    probabilities equal, and torch.topk orders equal values arbitrarily)."""
    g = np.load(GOLDEN / "router_golden.npz")
    f = oracle.bf16_bits_to_f32
    for ci in range(int(g["num_cases"][0])):
        p = f"c{ci}_"
        b, s, h, e, k, w, r = (int(x) for x in g[p + "shape"])
        logits, probs, vals, ids = oracle.router(f(g[p + "tokens"]), f(g[p + "router"]), k)
        ref_logits, ref_probs, ref_vals = f(g[p + "logits"]), f(g[p + "probs"]), f(g[p + "top_vals"])
        assert ids.shape == (b * s, k)
        assert (logits == ref_logits).mean() > 0.999, ci
        assert np.all(np.abs(logits - ref_logits) <= np.abs(ref_logits) * 2.0 ** -7), ci
        assert np.array_equal(probs, ref_probs), ci
        assert np.array_equal(vals, ref_vals), ci
        assert oracle.topk_mismatches(ids, vals, ref_probs, ref_vals) == 0, ci
        # and the reference's own selection passes the same check
        assert oracle.topk_mismatches(g[p + "top_idxs"], ref_vals, ref_probs, ref_vals) == 0, ci


def test_router_topk_order_and_ties():
    x = np.eye(4, dtype=np.float32)
    rw = np.array([[0, 1, 1, 0], [2, 0, 0, 0], [0, 0, 0, 0], [0, 0, 3, 1]], np.float32)
    _, probs, vals, ids = oracle.router(x, rw, 2)
    assert ids[0].tolist() == [1, 2]          # equal probabilities: ascending id
    assert ids[1].tolist() == [0, 1]
    assert ids[3].tolist() == [2, 3]
    assert np.all(np.diff(vals, axis=-1) <= 0)


def test_mlp_oracle_reduces_to_the_reference_layer():
    """The MLP restatement is the compact layer (pinned to the reference's
    outputs above) followed by SwiGLU and a per-expert GEMM: with an
    identity-like W_down its output is the activation h itself."""
    rng = np.random.default_rng(5)
    W, El, H, F = 2, 2, 16, 8
    counts = [np.array([3, 0, 2, 4]), np.array([1, 5, 0, 2])]
    send = [rng.standard_normal((int(c.sum()), H)).astype(np.float32) for c in counts]
    w13 = [rng.standard_normal((El, H, 2 * F)).astype(np.float32) * 0.3 for _ in range(W)]
    eye = [np.stack([np.eye(F, H, dtype=np.float32)] * El) for _ in range(W)]
    y = oracle.mlp_compact(send, counts, w13, eye)
    a = oracle.compact_layer(send, counts, w13)
    bf = lambda z: oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(z))
    for r in range(W):
        ab = bf(a[r])
        h = bf(ab[:, :F] / (1 + np.exp(-ab[:, :F])) * ab[:, F:])
        np.testing.assert_allclose(y[r][:, :F], h, rtol=1e-6, atol=1e-6)
        assert not y[r][:, F:].any()
        assert y[r].shape[0] == int(oracle.recv_counts_matrix(counts, r, W).sum())
