"""Generate the golden fixtures from the reference's own code.

Run where the reference is importable (its directory given by
``--reference``); writes ``routing_golden.npz`` and ``layer_golden.npz`` next
to this script.  The fixtures travel with the repository; tests never import
the reference.

1. routing_golden.npz — ``utils.gen_tensor`` (utils.py:7-75) run on CPU for
   small shapes whose buckets are all non-empty (an empty bucket makes the
   reference allocate on "cuda", utils.py:40).  ``torch.rand`` and
   ``torch.topk`` are observed (wrapped, not altered) to record the exact
   tokens and routing ids the reference drew; the fixture stores them with
   the reference's lengths, chunk_size and the SHA-256 of its coalesced
   tensor (plus the full tensor for two cases).
2. layer_golden.npz — ``baseline.run`` (baseline.py:8-56) under gloo with two
   CPU ranks for the fp32 CPU configuration (T=128, H=256, E=4, top-1,
   N=512), with ``torch.cuda.synchronize`` replaced by a no-op in the
   harness (baseline.py:53 calls it unconditionally).  Inputs come from
   ``nvshmem_testing_b200.workloads`` seeds and are padded with the
   all-ranks max (the oracle's convention); the fixture stores the routing
   ids, counts, the reference's fp32 output and SHA-256 digests of the
   regenerated tokens and weights.
3. router_golden.npz — the router of ``utils.gen_tensor`` (utils.py:17-25:
   bf16 einsum of tokens and router matrix, softmax, top-k) run on CPU for
   shapes whose expert count is a multiple of 8.  ``torch.einsum`` and
   ``torch.topk`` are observed to record their operands and results: the
   tokens, the router matrix, the bf16 logits, the bf16 probabilities and
   the top-k values and ids.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent

ROUTING_CASES = [  # (batch, seq, hidden, experts, topk, world, rank)
    (1, 64, 32, 4, 2, 2, 0), (1, 64, 32, 4, 2, 2, 1), (1, 64, 32, 4, 2, 2, 3),
    (1, 128, 64, 4, 2, 2, 0), (1, 128, 64, 4, 2, 2, 2),
    (1, 256, 128, 8, 4, 2, 0), (1, 256, 128, 8, 4, 4, 1),
    (2, 64, 64, 4, 3, 2, 0), (2, 64, 64, 4, 3, 4, 3),
    (1, 512, 16, 4, 2, 2, 2),
    (1, 64, 8, 8, 8, 2, 0),
    (1, 128, 32, 8, 6, 2, 0), (1, 128, 32, 8, 6, 2, 3),
    (1, 96, 24, 6, 3, 2, 2), (1, 96, 24, 6, 3, 3, 3),
]
FULL_COALESCED = {0, 10}


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def make_routing(ref: Path) -> dict:
    sys.path.insert(0, str(ref))
    import utils as ref_utils  # the reference's utils.py

    out = {}
    real_rand, real_topk = torch.rand, torch.topk
    for ci, (b, s, h, e, k, w, r) in enumerate(ROUTING_CASES):
        seen = {}

        def rand_spy(*a, **kw):
            t = real_rand(*a, **kw)
            seen.setdefault("tokens", t)
            return t

        def topk_spy(*a, **kw):
            res = real_topk(*a, **kw)
            seen["top_idxs"] = res[1]
            return res

        torch.rand, torch.topk = rand_spy, topk_spy
        try:
            coalesced, chunk, lengths = ref_utils.gen_tensor(b, s, h, w, e, r, k)
        finally:
            torch.rand, torch.topk = real_rand, real_topk
        p = f"c{ci}_"
        out[p + "shape"] = np.array([b, s, h, e, k, w, r], np.int64)
        out[p + "tokens"] = bf16_bits(seen["tokens"])
        out[p + "top_idxs"] = seen["top_idxs"].numpy().astype(np.int16)
        out[p + "chunk"] = np.array([chunk], np.int64)
        out[p + "lengths"] = np.array(lengths, np.int32)
        cb = bf16_bits(coalesced)
        out[p + "coalesced_sha256"] = np.frombuffer(hashlib.sha256(cb.tobytes()).digest(), np.uint8)
        out[p + "coalesced_rows"] = np.array([cb.shape[0]], np.int64)
        if ci in FULL_COALESCED:
            out[p + "coalesced"] = cb
    out["num_cases"] = np.array([len(ROUTING_CASES)], np.int64)
    return out


ROUTER_CASES = [  # (batch, seq, hidden, experts, topk, world, rank)
    (1, 256, 64, 8, 2, 2, 0), (1, 128, 256, 16, 4, 2, 1), (1, 512, 128, 64, 6, 2, 0),
    (1, 64, 512, 256, 8, 8, 3), (2, 64, 32, 8, 1, 1, 0),
]


def make_router(ref: Path) -> dict:
    sys.path.insert(0, str(ref))
    import utils as ref_utils  # the reference's utils.py

    out = {}
    real_einsum, real_topk = torch.einsum, torch.topk
    for ci, (b, s, h, e, k, w, r) in enumerate(ROUTER_CASES):
        seen = {}

        def einsum_spy(eq, *ops, **kw):
            res = real_einsum(eq, *ops, **kw)
            seen.setdefault("einsum", (ops[0], ops[1], res))
            return res

        def topk_spy(x, *a, **kw):
            res = real_topk(x, *a, **kw)
            seen.setdefault("topk", (x, res[0], res[1]))
            return res

        torch.einsum, torch.topk = einsum_spy, topk_spy
        try:
            try:
                ref_utils.gen_tensor(b, s, h, w, e, r, k)
            except (RuntimeError, AssertionError):
                pass  # bucketing after the router may need a GPU; the router ran first
        finally:
            torch.einsum, torch.topk = real_einsum, real_topk
        tok, rmat, logits = seen["einsum"]
        probs, vals, ids = seen["topk"]
        p = f"c{ci}_"
        out[p + "shape"] = np.array([b, s, h, e, k, w, r], np.int64)
        out[p + "tokens"] = bf16_bits(tok)
        out[p + "router"] = bf16_bits(rmat)
        out[p + "logits"] = bf16_bits(logits)
        out[p + "probs"] = bf16_bits(probs)
        out[p + "top_vals"] = bf16_bits(vals)
        out[p + "top_idxs"] = ids.numpy().astype(np.int16)
    out["num_cases"] = np.array([len(ROUTER_CASES)], np.int64)
    return out


def _layer_rank(rank: int, world: int, port: int, ref: str, q) -> None:
    import torch.distributed as dist
    sys.path.insert(0, ref)
    sys.path.insert(0, str(ROOT))
    import baseline as ref_baseline  # the reference's baseline.py
    from nvshmem_testing_b200 import workloads
    import oracle

    torch.cuda.synchronize = lambda *a, **k: None  # harness shim: CPU ranks have no device
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    wl = workloads.get("cpu_gloo")
    tok = workloads.tokens(wl, rank)
    ids = workloads.top_idxs(wl, rank)
    wts = workloads.weights(wl, rank, world)
    counts, offsets, perm = oracle.bucketize(ids.numpy(), wl.E)
    m = torch.tensor([oracle.local_max(counts)], dtype=torch.int64)
    dist.all_reduce(m, op=dist.ReduceOp.MAX)
    gm = int(m.item())
    coalesced = torch.from_numpy(oracle.pad_coalesce(tok.numpy(), counts, offsets, perm, gm))
    El = wl.E // world
    out = ref_baseline.run(rank, coalesced, gm * El, 1, wl.T, wl.H, wl.E, world, False, None, wts)
    q.put((rank, gm, tok.numpy(), ids.numpy(), wts.numpy(), counts, out.numpy()))
    dist.barrier()
    dist.destroy_process_group()


def make_layer(ref: Path) -> dict:
    import socket
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 2
    procs = [ctx.Process(target=_layer_rank, args=(r, world, port, str(ref), q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    out = {}
    for rank, gm, tok, ids, wts, counts, o in sorted(res, key=lambda x: x[0]):
        p = f"r{rank}_"
        # Inputs are regenerated from workload seeds by the tests; their
        # SHA-256 pins the generator.
        out[p + "tokens_sha256"] = np.frombuffer(hashlib.sha256(tok.astype(np.float32).tobytes()).digest(), np.uint8)
        out[p + "weights_sha256"] = np.frombuffer(hashlib.sha256(wts.astype(np.float32).tobytes()).digest(), np.uint8)
        out[p + "top_idxs"] = ids.astype(np.int16)
        out[p + "counts"] = counts.astype(np.int32)
        out[p + "out"] = o.astype(np.float32)
        out["gm"] = np.array([gm], np.int64)
    out["world"] = np.array([world], np.int64)
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="directory of the reference checkout (its utils.py, baseline.py)")
    a = ap.parse_args()
    ref = Path(a.reference)
    np.savez_compressed(HERE / "routing_golden.npz", **make_routing(ref))
    np.savez_compressed(HERE / "layer_golden.npz", **make_layer(ref))
    np.savez_compressed(HERE / "router_golden.npz", **make_router(ref))
    for f in ("routing_golden.npz", "layer_golden.npz", "router_golden.npz"):
        print(f, os.path.getsize(HERE / f), "bytes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
