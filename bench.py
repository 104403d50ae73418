"""Benchmark: fused MoE expert-parallel layer (dispatch + grouped GEMM).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]
                    [--path dispatch_gemm|combine]

One process per GPU (torchrun for N > 1).  A step is one call of the fused
layer ``alltoall_persistent_gemm.run`` on this rank's padded, expert-major
token buffer (inputs resident in HBM): count exchange, NVLink dispatch of the
valid rows, and the grouped GEMM over the local experts.  Weak scaling: the
tokens per rank are fixed; experts split E/N per rank.

Printed (rank 0, one JSON line): whole-job TFLOP/s over valid rows (``value``),
µs per layer, the roofline of the fused kernel, the same metric end to end
through the public API from pinned host buffers (``e2e``), the reference's
NCCL all_to_all_single + bmm on the same inputs, and the oracle's CPU time on
the host cores (``cpu_baseline``).  ``--impl reference`` times the oracle (the
CPU restatement of the reference path) on the host cores instead.

``--path combine`` times the layer with its return path instead: the fused
kernel in return mode (each output row stored into its source rank's return
region over NVLink) plus the top-k combine kernel (``combine.run``), against
NCCL all_to_all_single + bmm + the reverse all_to_all_single + a torch
gather/weighted sum on the same inputs.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from nvshmem_testing_b200 import alltoall_persistent_gemm as apg  # noqa: E402
from nvshmem_testing_b200 import utils, workloads  # noqa: E402

METRIC = "fused dispatch+grouped-GEMM µs/layer & TFLOP/s, 1/2/4/8 B200 vs NCCL a2a+GEMM"
METRIC_COMBINE = "fused dispatch+grouped-GEMM+return+top-k combine µs/layer & TFLOP/s vs NCCL a2a+GEMM+a2a+combine"
NVLINK_GBS = 770.0          # measured peer copy per direction on this pool (nominal 900)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(workload: str, world: int):
    """Per-launch DRAM bytes of the fused kernel from a committed ncu summary
    (profiles/traffic.txt: lines "workload world bytes"), or None."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        f = line.split()
        if len(f) >= 3 and not line.startswith("#") and f[0] == workload and f[1] == str(world):
            return int(float(f[2]))
    return None


class ClockSampler:
    """nvidia-smi clock/throttle samples for one GPU while running."""

    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        """Start sampling; call ``mark_start``/``mark_end`` around the timed
        region, then ``stop``; only samples inside the window count."""
        self.proc = None
        self.t0 = self.t1 = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            gid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", gid, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(1.0)  # let nvidia-smi start emitting before the window opens
        except Exception:
            self.proc = None

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self) -> dict:
        from datetime import datetime
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.2)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            out = ""
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                ts = datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                clk, cmax = float(f[1]), float(f[2])
            except ValueError:
                continue
            if self.t0 is not None and not (self.t0 - 0.05 <= ts <= (self.t1 or ts) + 0.05):
                continue
            sm.append(clk)
            smax.append(cmax)
            try:
                power.append(float(f[3]))
            except ValueError:
                pass
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


def init_dist(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29531")
    dist.init_process_group("nccl", init_method="env://", rank=rank, world_size=world,
                            timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(x: float) -> float:
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float) -> float:
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def nccl_a2a_bmm(tokens, chunk, world, weights):
    """The reference's NCCL baseline (baseline.py:18-50) restated for timing:
    equal-split all_to_all_single, view/permute/flatten, bmm over padded rows."""
    recv = torch.zeros(chunk * world, tokens.shape[1], dtype=tokens.dtype, device=tokens.device)
    dist.all_to_all_single(recv, tokens)
    El = weights.shape[0]
    x = recv.view(world, El, chunk // El, tokens.shape[1]).permute(1, 0, 2, 3).flatten(1, 2)
    return torch.bmm(x, weights)


def nccl_layer_combine(tokens, chunk, world, weights, ids, vals, slots):
    """The same layer with the return path done the NCCL way: the baseline's
    a2a + bmm, the reverse all_to_all_single of the [El, W*gm, N] outputs
    back to the senders' padded layout, and a torch gather + top-k weighted
    sum (fp32) per token."""
    out = nccl_a2a_bmm(tokens, chunk, world, weights)
    El, N = weights.shape[0], weights.shape[2]
    gm = chunk // El
    send = out.view(El, world, gm, N).permute(1, 0, 2, 3).reshape(world * El * gm, N)
    back = torch.empty_like(send)
    dist.all_to_all_single(back, send)
    E = El * world
    valid = (ids >= 0) & (ids < E) & (slots >= 0)
    rows = torch.where(valid, ids * gm + slots, torch.zeros_like(ids))
    w = torch.where(valid, vals.float(), torch.zeros_like(vals, dtype=torch.float32))
    return (back[rows].float() * w[..., None]).sum(dim=1).to(torch.bfloat16)


def time_device(fn, steps: int, warmup: int, sampler_device=None):
    sampler = ClockSampler(sampler_device) if sampler_device is not None else None
    for _ in range(warmup):
        fn()
    dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler:
        sampler.mark_start()
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    if sampler:
        sampler.mark_end()
    clocks = sampler.stop() if sampler else None
    dist.barrier()
    return s.elapsed_time(e) / steps, clocks


class CpuLayer:
    """The oracle (CPU restatement of the reference path) for rank 0's share
    of the layer: routing of every rank's ids (utils.py:28-41), padding of
    rank 0's buckets from every source (the equal-split exchange,
    baseline.py:23) and fp32 expert GEMMs (baseline.py:50).  ``step`` runs
    the routing in full and as many experts as fit the time budget, and
    returns (valid FLOPs, seconds, experts done)."""

    def __init__(self, wl, world: int):
        import oracle
        self.oracle = oracle
        try:
            from threadpoolctl import threadpool_info
            self.cores = max([i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
                             or [os.cpu_count() or 1])
        except Exception:
            self.cores = os.cpu_count() or 1
        self.wl, self.world = wl, world
        self.El = wl.local_experts(world)
        self.ids = [workloads.top_idxs(wl, r).numpy() for r in range(world)]
        self.tok = [workloads.tokens(wl, r).float().numpy() for r in range(world)]
        g = torch.Generator().manual_seed(wl.seed + 10086)
        # One rank-0 expert's weights are reused for every sampled expert: the
        # arithmetic is identical and the sample stays within host memory.
        self.w = (0.02 * torch.randn(wl.H, wl.N, generator=g)).numpy()
        self.next_expert = 0

    def step(self, budget_s: float):
        o = self.oracle
        t0 = time.perf_counter()
        routed = [o.bucketize(ids, self.wl.E) for ids in self.ids]
        gm = max(o.local_max(c) for c, _, _ in routed)
        flops, done = 0.0, 0
        while done < self.El and (done == 0 or time.perf_counter() - t0 < budget_s):
            le = (self.next_expert + done) % self.El
            blocks = []
            for r, (c, off, p) in enumerate(routed):
                blk = np.zeros((gm, self.wl.H), np.float32)
                blk[:c[le]] = self.tok[r][p[off[le]:off[le] + c[le]]]
                blocks.append(blk)
                flops += 2.0 * float(c[le]) * self.wl.H * self.wl.N
            np.matmul(np.concatenate(blocks), self.w)
            done += 1
        self.next_expert = (self.next_expert + done) % self.El
        return flops, time.perf_counter() - t0, done


def cpu_oracle_sample(wl, world: int, budget_s: float = 10.0) -> dict:
    layer = CpuLayer(wl, world)
    flops, dt, done = layer.step(budget_s)
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": int(layer.cores), "kind": "port",
            "sample": f"rank 0 of {world}: routing of all ranks, padding and fp32 GEMMs of {done}/{layer.El} "
                      f"local experts ({dt:.1f} s)"}


def overrides(args) -> dict:
    o = {}
    if args.tokens:
        o["T"] = args.tokens
    if args.experts:
        o["E"] = args.experts
    return o


def run_reference_arm(args) -> int:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    wl = workloads.get(args.workload, **overrides(args))
    # Each step is a bounded sample of the layer, sized so that warm-up and
    # timed steps together take a couple of minutes of host time.
    budget = min(max(150.0 / (args.steps + args.warmup), 0.05), 10.0)
    prep = CpuLayer(wl, args.gpus)
    for _ in range(args.warmup):
        prep.step(budget)
    vals, secs = [], []
    for _ in range(args.steps):
        flops, dt, done = prep.step(budget)
        vals.append(flops / dt / 1e12)
        secs.append(dt)
    value = statistics.median(vals)
    cb = {"value": value, "unit": "TFLOP/s", "cores": prep.cores, "kind": "port",
          "sample": f"per step: routing of all {args.gpus} ranks, padding and fp32 GEMMs of about {done} of "
                    f"{prep.El} local experts of rank 0 (~{statistics.median(secs):.2f} s)"}
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.median(secs) * 1e3,
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": {"workload": wl.name, "tokens_per_rank": wl.T, "hidden": wl.H, "experts": wl.E, "top_k": wl.K,
                       "out_dim": wl.N, "world_size": args.gpus, "routing": wl.routing},
            "cpu_baseline": cb,
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_mlp_path(args) -> int:
    """The full expert MLP (``mlp.run``: compact exchange + [gate|up] GEMM,
    SwiGLU, down GEMM) against NCCL a2a + bmm(w13) + silu*up + bmm(w2) over
    padded rows, on the same inputs.  FFN width F = the workload's out_dim."""
    from nvshmem_testing_b200 import mlp

    rank, world, local = init_dist(args.gpus)
    dev = torch.device("cuda", local)
    wl = workloads.get(args.workload, dtype=torch.bfloat16, **overrides(args))
    El, H, F = wl.local_experts(world), wl.H, wl.N
    tokens = workloads.tokens(wl, rank, device=dev)
    ids = workloads.top_idxs(wl, rank).to(dev)
    g = torch.Generator(device=dev).manual_seed(wl.seed + 10086 + rank)
    w13 = (0.02 * torch.randn(El, H, 2 * F, generator=g, device=dev)).to(torch.bfloat16)
    w2 = (0.02 * torch.randn(El, F, H, generator=g, device=dev)).to(torch.bfloat16)
    coalesced, chunk, lengths = utils.dispatch(tokens, ids, wl.E, world)
    compact, total, _ = utils.dispatch(tokens, ids, wl.E, world, general_a2a=True)
    counts = torch.tensor(lengths, dtype=torch.int32, device=dev)
    recv_counts = utils.recv_counts_from(counts, world)
    gm = chunk // El
    rc_cpu = recv_counts.cpu()
    rows_in = int(rc_cpu.sum())
    remote_in = rows_in - int(rc_cpu[rank].sum())
    remote_out = int(counts.view(world, El).sum()) - int(counts.view(world, El)[rank].sum())

    w13f = mlp.fuse_gate_up(w13) if F % 128 == 0 else None

    def ours():
        if w13f is not None:  # activation in the first GEMM's epilogue
            return mlp.run(rank, compact, total, world, w13f, w2, recv_counts, max_count=gm, recv_rows=rows_in,
                           w13_fused=True)
        return mlp.run(rank, compact, total, world, w13, w2, recv_counts, max_count=gm, recv_rows=rows_in)

    def ours_separate():
        return mlp.run(rank, compact, total, world, w13, w2, recv_counts, max_count=gm, recv_rows=rows_in)

    def nccl():
        a = nccl_a2a_bmm(coalesced, chunk, world, w13)
        h = torch.nn.functional.silu(a[..., :F]) * a[..., F:]
        return torch.bmm(h, w2)

    y = ours()
    ref = nccl()
    ref = torch.cat([ref[le, src * gm:src * gm + int(rc_cpu[src, le])] for le in range(El) for src in range(world)])
    scale = float(ref.float().abs().max()) if ref.numel() else 1.0
    ok = bool(torch.allclose(y.float(), ref.float(), rtol=1e-2, atol=1e-2 * scale))
    del ref, y
    ms, clocks = time_device(ours, args.steps, args.warmup, sampler_device=local)
    ms_s, _ = time_device(ours_separate, max(args.steps // 3, 5), args.warmup)
    ms_n, _ = time_device(nccl, max(args.steps // 3, 5), args.warmup)
    ms, ms_s, ms_n = max_over_ranks(ms), max_over_ranks(ms_s), max_over_ranks(ms_n)
    flops_rank = 6.0 * rows_in * H * F
    flops_total = sum_over_ranks(flops_rank)
    peaks, src = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    # weights once; rows in, the [gate|up] rows out and back in, h out and in, y out
    hbm = 3 * El * H * F * 2 + rows_in * (H * 2 + 2 * F * 2 * 2 + F * 2 * 2 + H * 2) + \
        (remote_in + remote_out) * H * 2
    t_gemm = flops_rank / (peak * 1e12) * 1e6
    t_hbm = hbm / (hbm_peak * 1e9) * 1e6
    t_link = max(remote_in, remote_out) * H * 2 / (NVLINK_GBS * 1e9) * 1e6
    roof = max_over_ranks(max(t_gemm, t_hbm, t_link))
    bound = "hbm" if t_hbm > t_gemm else "tensor"
    line = {"metric": "fused dispatch + full expert MLP (gate/up, SwiGLU, down) µs/layer & TFLOP/s vs NCCL",
            "path": "mlp", "value": flops_total / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "us_per_layer": ms * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded)",
            "config": {"workload": wl.name + "+mlp", "tokens_per_rank": wl.T, "hidden": H, "experts": wl.E,
                       "local_experts": El, "top_k": wl.K, "ffn": F, "routing": wl.routing, "gm": gm,
                       "parallelism": f"ep{world}"},
            "parity_vs_nccl_allclose": ok,
            "roofline": {"bound": bound, "layer_roofline_us": roof, "layer_frac": roof / (ms * 1e3),
                         "bounds_us": {"tensor": t_gemm, "hbm": t_hbm, "nvlink": t_link},
                         "algorithmic_hbm_bytes": hbm, "peak_source": src},
            "fused_swiglu": w13f is not None, "separate_swiglu_us": ms_s * 1e3,
            "nccl_mlp": {"us_per_layer": ms_n * 1e3, "value": flops_total / (ms_n * 1e-3) / 1e12,
                         "what": "NCCL a2a + bmm(w13) + silu*up + bmm(w2) over padded rows"},
            "gpu_launches": (2 if w13f is not None else 3) * args.steps, "clocks": clocks}
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier()
    from nvshmem_testing_b200 import symm
    symm.release_all()
    dist.destroy_process_group()
    return 0


def run_router_path(args) -> int:
    """The router (``utils.router``: tcgen05 logits GEMM + softmax/top-k
    kernel) on one rank's tokens, against torch's einsum + softmax + topk
    (the reference's utils.py:23-25) on the same resident inputs."""
    rank, world, local = init_dist(args.gpus)
    dev = torch.device("cuda", local)
    wl = workloads.get(args.workload, dtype=torch.bfloat16, **overrides(args))
    x = workloads.tokens(wl, rank, device=dev)
    g = torch.Generator(device=dev).manual_seed(wl.seed + 77)
    rw = (0.001 * torch.randn(wl.H, wl.E, generator=g, device=dev)).to(torch.bfloat16)  # the reference's scale
    logits = torch.empty((wl.T, wl.E), dtype=torch.bfloat16, device=dev)
    K = wl.K

    def ours():
        return utils.router(x, rw, K, logits=logits)

    def torch_router():
        probs = torch.softmax(torch.einsum("bh,he->be", x, rw), dim=-1)
        return torch.topk(probs, K)

    v, i = ours()
    tv, _ = torch_router()
    torch.cuda.synchronize()
    vals_equal = bool(torch.allclose(v, tv.float(), rtol=2 ** -7, atol=0))  # top values, tie-invariant
    ms, clocks = time_device(ours, args.steps, args.warmup, sampler_device=local)
    ms_t, _ = time_device(torch_router, args.steps, args.warmup)
    ms, ms_t = max_over_ranks(ms), max_over_ranks(ms_t)
    # The same calls replayed from CUDA graphs: device time without the host's
    # per-launch cost (both are launch-bound when called eagerly).
    graphs = {}
    for name, fn in (("ours", ours), ("torch", torch_router)):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        graphs[name] = gr
    ms_g, _ = time_device(graphs["ours"].replay, args.steps, args.warmup)
    ms_tg, _ = time_device(graphs["torch"].replay, args.steps, args.warmup)
    ms_g, ms_tg = max_over_ranks(ms_g), max_over_ranks(ms_tg)
    graphs.clear()
    peaks, src = load_peaks()
    flops = 2.0 * wl.T * wl.H * wl.E
    hbm = wl.T * wl.H * 2 + wl.H * wl.E * 2 + 2 * wl.T * wl.E * 2 + wl.T * K * 12
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    t_roof = max(flops / (peak * 1e12), hbm / (hbm_peak * 1e9))
    line = {"metric": "router µs (einsum + softmax + top-k) per rank", "path": "router",
            "value": ms * 1e3, "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; router 0.001*N(0,1) like the reference)",
            "config": {"workload": wl.name + "+router", "tokens_per_rank": wl.T, "hidden": wl.H, "experts": wl.E,
                       "top_k": K},
            "top_vals_match_torch": vals_equal, "torch_us": ms_t * 1e3,
            "graph_us": ms_g * 1e3, "torch_graph_us": ms_tg * 1e3,
            "roofline": {"bound": "hbm" if hbm / (hbm_peak * 1e9) > flops / (peak * 1e12) else "tensor",
                         "roofline_us": t_roof * 1e6, "frac": t_roof / (ms * 1e-3),
                         "frac_graph": t_roof / (ms_g * 1e-3), "peak_source": src,
                         "flops": flops, "algorithmic_hbm_bytes": hbm},
            "gpu_launches": 3 * args.steps,  # count word, logits GEMM, softmax/top-k
            "clocks": clocks}
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


def run_combine_path(args) -> int:
    """The layer with its return path (``combine.run``): one JSON line like
    the default path's, with the NCCL a2a + bmm + reverse a2a + combine arm."""
    from nvshmem_testing_b200 import combine

    rank, world, local = init_dist(args.gpus)
    dev = torch.device("cuda", local)
    wl = workloads.get(args.workload, dtype=torch.bfloat16, **overrides(args))
    El = wl.local_experts(world)
    tokens = workloads.tokens(wl, rank, device=dev)
    ids_cpu = workloads.top_idxs(wl, rank)
    vals_cpu = workloads.top_vals(wl, rank)
    ids, vals = ids_cpu.to(dev), vals_cpu.to(dev)
    weights = workloads.weights(wl, rank, world, device=dev)
    r = utils.route(ids, wl.E, with_slots=True)
    gm = utils.global_max_count(r)
    coalesced = utils.pack_padded(tokens, r, gm)
    chunk = El * gm
    counts = r.counts
    recv_counts = utils.recv_counts_from(counts, world)
    rc_cpu, c_cpu = recv_counts.cpu(), counts.cpu().view(world, El)
    rows_in = int(rc_cpu.sum())
    remote_in = rows_in - int(rc_cpu[rank].sum())
    remote_out = int(c_cpu.sum()) - int(c_cpu[rank].sum())
    flops_rank = 2.0 * rows_in * wl.H * wl.N
    # NVLink per direction: rows out and expert outputs back, both ways.
    link_out = remote_out * wl.H * 2 + remote_in * wl.N * 2
    link_in = remote_in * wl.H * 2 + remote_out * wl.N * 2
    nvlink_bytes = max(link_out, link_in)

    def step():
        return combine.run(rank, coalesced, chunk, world, weights, recv_counts, ids, vals, r.slots)

    ours = step()
    torch.cuda.synchronize()
    ok = True
    if not args.no_nccl:
        ref = nccl_layer_combine(coalesced, chunk, world, weights, ids, vals, r.slots)
        ok = bool(torch.allclose(ours.float(), ref.float(), rtol=1e-2, atol=1e-2))
        del ref
    del ours

    ms, clocks = time_device(step, args.steps, args.warmup, sampler_device=local)
    ms_max = max_over_ranks(ms)
    flops_total = sum_over_ranks(flops_rank)
    value = flops_total / (ms_max * 1e-3) / 1e12

    nccl = None
    if not args.no_nccl:
        ms_n, _ = time_device(lambda: nccl_layer_combine(coalesced, chunk, world, weights, ids, vals, r.slots),
                              max(args.steps // 3, 10), args.warmup)
        ms_n = max_over_ranks(ms_n)
        nccl = {"us_per_layer": ms_n * 1e3, "value": flops_total / (ms_n * 1e-3) / 1e12, "unit": "TFLOP/s",
                "what": "NCCL a2a + bmm over padded rows + reverse a2a + torch gather/top-k weighted sum"}

    # end to end through the public API (combine.moe_layer) from pinned host buffers
    x_host = workloads.tokens(wl, rank).pin_memory()
    ids_host, vals_host = ids_cpu.pin_memory(), vals_cpu.pin_memory()
    y_host = torch.empty((wl.T, wl.N), dtype=torch.bfloat16).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (x_host, ids_host, vals_host))
    d2h = y_host.numel() * y_host.element_size()

    def e2e_step():
        x = x_host.to(dev, non_blocking=True)
        i = ids_host.to(dev, non_blocking=True)
        v = vals_host.to(dev, non_blocking=True)
        y_host.copy_(combine.moe_layer(x, i, v, weights), non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(3):
        e2e_step()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.e2e_steps):
        e2e_step()
    e.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s.elapsed_time(e) / args.e2e_steps)
    dist.barrier()

    peaks, peaks_src = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    K = ids.shape[1]
    # weights once, every valid row once, remote rows read for sending and
    # written by peers, every output row written once (return region, local
    # or remote) and read once by the combine, ids/vals/slots and y.
    rows_out_total = int(c_cpu.sum())
    hbm_bytes = (El * wl.H * wl.N * 2 + rows_in * wl.H * 2 + (remote_in + remote_out) * wl.H * 2
                 + rows_in * wl.N * 2 + rows_out_total * wl.N * 2 + wl.T * K * 16 + wl.T * wl.N * 2)
    t_gemm_us = flops_rank / (peak * 1e12) * 1e6
    t_hbm_us = hbm_bytes / (hbm_peak * 1e9) * 1e6
    t_link_us = nvlink_bytes / (NVLINK_GBS * 1e9) * 1e6
    roof_us = max_over_ranks(max(t_gemm_us, t_hbm_us, t_link_us))
    if t_hbm_us > t_gemm_us:
        bound, achieved, peak_v, unit = "hbm", hbm_bytes / (ms_max * 1e-3) / 1e9, hbm_peak, "GB/s"
        peak_note = f"{peaks_src} hbm_gbs"
    else:
        bound, achieved, peak_v, unit = "tensor", flops_rank / (ms_max * 1e-3) / 1e12, peak, "TFLOP/s"
        peak_note = f"{peaks_src} bf16_tflops (burst)"
    line = {
        "metric": METRIC_COMBINE, "path": "combine", "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "us_per_layer": ms_max * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded)",
        "config": {"workload": wl.name + "+combine", "tokens_per_rank": wl.T, "hidden": wl.H, "experts": wl.E,
                   "local_experts": El, "top_k": wl.K, "out_dim": wl.N, "routing": wl.routing, "gm": gm,
                   "parallelism": f"ep{world}", "l2": "inputs larger than L2 (weights and tokens > 126 MB)"},
        "parity_vs_nccl_allclose": ok,
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak_v, "unit": unit,
                     "frac": achieved / peak_v, "peak_source": peak_note, "traffic": None,
                     "algorithmic_hbm_bytes": hbm_bytes, "tensor_tflops": flops_rank / (ms_max * 1e-3) / 1e12,
                     "bounds_us": {"tensor": t_gemm_us, "hbm": t_hbm_us, "nvlink": t_link_us},
                     "layer_roofline_us": roof_us, "layer_frac": roof_us / (ms_max * 1e3),
                     "nvlink_bytes_rank": nvlink_bytes},
        "cpu_baseline": None,
        "e2e": {"value": flops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "us_per_layer": e2e_ms * 1e3,
                "what": "pinned host x+ids+vals -> combine.moe_layer (route, pack, count a2a, fused return, "
                        "combine) -> pinned host y"},
        "nccl_layer_combine": nccl,
        "gpu_launches": 2 * args.steps,  # fused kernel + combine kernel per step
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier()
    from nvshmem_testing_b200 import symm
    symm.release_all()
    dist.destroy_process_group()
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="deepseek_v3", choices=sorted(workloads.CONFIGS))
    ap.add_argument("--tokens", type=int, default=0, help="override tokens per rank")
    ap.add_argument("--experts", type=int, default=0, help="override total experts (small profiling cases)")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-nccl", action="store_true")
    ap.add_argument("--path", choices=["dispatch_gemm", "general", "combine", "router", "mlp"],
                    default="dispatch_gemm",
                    help="dispatch_gemm: the reference's path (default); general: the unpadded exchange "
                         "(general_a2a=True); combine: with return + top-k combine; router: the router "
                         "(einsum, softmax, top-k) before the path; mlp: the full gated expert MLP "
                         "(FFN width = the workload's out_dim)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.path == "combine":
        return run_combine_path(args)
    if args.path == "router":
        return run_router_path(args)
    if args.path == "mlp":
        return run_mlp_path(args)

    rank, world, local = init_dist(args.gpus)
    dev = torch.device("cuda", local)
    wl = workloads.get(args.workload, dtype=torch.bfloat16, **overrides(args))
    El = wl.local_experts(world)

    # ---- inputs (seeded, generated on the device) and routing
    tokens = workloads.tokens(wl, rank, device=dev)
    ids_cpu = workloads.top_idxs(wl, rank)
    ids = ids_cpu.to(dev)
    weights = workloads.weights(wl, rank, world, device=dev)
    general = args.path == "general"
    coalesced, chunk, lengths = utils.dispatch(tokens, ids, wl.E, world)
    counts = torch.tensor(lengths, dtype=torch.int32, device=dev)
    recv_counts = utils.recv_counts_from(counts, world)
    gm = chunk // El
    if general:  # compact send buffer; the padded one stays for the NCCL arm
        compact, total, _ = utils.dispatch(tokens, ids, wl.E, world, general_a2a=True)
    rc_cpu = recv_counts.cpu()
    rows_in = int(rc_cpu.sum())
    remote_in = rows_in - int(rc_cpu[rank].sum())
    remote_out = int(counts.view(world, El).sum()) - int(counts.view(world, El)[rank].sum())
    flops_rank = 2.0 * rows_in * wl.H * wl.N
    nvlink_bytes = max(remote_in, remote_out) * wl.H * 2

    def step():
        if general:
            return apg.run(rank, compact, total, 1, wl.T, wl.H, wl.E, world, None, True, weights, recv_counts,
                           max_count=gm, recv_rows=rows_in)
        return apg.run(rank, coalesced, chunk, 1, wl.T, wl.H, wl.E, world, None, False, weights, recv_counts)

    # correctness guard against the NCCL path on this very input
    ours = step()
    torch.cuda.synchronize()
    apg.raise_if_device_error(apg.get_workspace(world, El, wl.H, gm, local, None, rank, apg.DEFAULT_PUSH_ROWS))
    ok = True
    if not args.no_nccl:
        ref = nccl_a2a_bmm(coalesced, chunk, world, weights)
        if general:  # drop the padded rows of the NCCL result: cells (le, src) back to back
            ref = torch.cat([ref[le, src * gm:src * gm + int(rc_cpu[src, le])]
                             for le in range(El) for src in range(world)])
        ok = bool(torch.allclose(ours.float(), ref.float(), rtol=1e-2, atol=1e-2))
        del ref
    del ours

    ms, clocks = time_device(step, args.steps, args.warmup, sampler_device=local)
    ms_max = max_over_ranks(ms)
    flops_total = sum_over_ranks(flops_rank)
    value = flops_total / (ms_max * 1e-3) / 1e12
    gpu_launches = args.steps  # one fused kernel per step

    nccl = None
    if not args.no_nccl:
        ms_n, _ = time_device(lambda: nccl_a2a_bmm(coalesced, chunk, world, weights), max(args.steps // 3, 10),
                              args.warmup)
        ms_n = max_over_ranks(ms_n)
        nccl = {"us_per_layer": ms_n * 1e3, "value": flops_total / (ms_n * 1e-3) / 1e12, "unit": "TFLOP/s",
                "what": "NCCL all_to_all_single + view/permute/flatten + torch.bmm over padded rows"}

    # ---- end to end through the public API from pinned host buffers
    tok_host = workloads.tokens(wl, rank).pin_memory()  # CPU-generated, same shape/distribution
    ids_host = ids_cpu.pin_memory()
    out_host = torch.empty((rows_in, wl.N) if general else (El, world * gm, wl.N), dtype=torch.bfloat16).pin_memory()
    h2d = tok_host.numel() * tok_host.element_size() + ids_host.numel() * ids_host.element_size()
    d2h = out_host.numel() * out_host.element_size()

    def e2e_step():
        t = tok_host.to(dev, non_blocking=True)
        i = ids_host.to(dev, non_blocking=True)
        co, ch, ln = utils.dispatch(t, i, wl.E, world, general_a2a=general)
        rc = utils.recv_counts_from(torch.tensor(ln, dtype=torch.int32, device=dev), world)
        o = apg.run(rank, co, ch, 1, wl.T, wl.H, wl.E, world, None, general, weights, rc)
        out_host.copy_(o, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(3):
        e2e_step()
    dist.barrier()
    t0 = time.perf_counter()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.e2e_steps):
        e2e_step()
    e.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s.elapsed_time(e) / args.e2e_steps)
    dist.barrier()
    e2e_value = flops_total / (e2e_ms * 1e-3) / 1e12

    peaks, peaks_src = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    # Algorithmic HBM bytes of one launch on this rank: expert weights once,
    # every valid row once, the whole padded output, and the remote rows read
    # for sending plus written by peers.
    out_rows = rows_in if general else El * world * gm  # the compact output has no padded rows
    hbm_bytes = (El * wl.H * wl.N * 2 + rows_in * wl.H * 2 + out_rows * wl.N * 2
                 + (remote_in + remote_out) * wl.H * 2)
    t_gemm_us = flops_rank / (peak * 1e12) * 1e6
    t_hbm_us = hbm_bytes / (hbm_peak * 1e9) * 1e6
    t_link_us = nvlink_bytes / (NVLINK_GBS * 1e9) * 1e6
    roof_us = max_over_ranks(max(t_gemm_us, t_hbm_us, t_link_us))
    if t_hbm_us > t_gemm_us:
        bound, achieved, peak_v, unit = "hbm", hbm_bytes / (ms_max * 1e-3) / 1e9, hbm_peak, "GB/s"
        peak_note = f"{peaks_src} hbm_gbs"
    else:
        bound, achieved, peak_v, unit = "tensor", flops_rank / (ms_max * 1e-3) / 1e12, peak, "TFLOP/s"
        peak_note = f"{peaks_src} bf16_tflops (burst)"
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "us_per_layer": ms_max * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": wl.name + ("+general_a2a" if general else ""), "tokens_per_rank": wl.T,
                   "hidden": wl.H, "experts": wl.E,
                   "local_experts": El, "top_k": wl.K, "out_dim": wl.N, "routing": wl.routing, "gm": gm,
                   "parallelism": f"ep{world}", "l2": "inputs larger than L2 (weights and tokens > 126 MB)"},
        "parity_vs_nccl_allclose": ok,
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak_v, "unit": unit,
                     "frac": achieved / peak_v, "peak_source": peak_note,
                     "traffic": load_traffic(wl.name, world), "algorithmic_hbm_bytes": hbm_bytes,
                     "tensor_tflops": flops_rank / (ms_max * 1e-3) / 1e12,
                     "bounds_us": {"tensor": t_gemm_us, "hbm": t_hbm_us, "nvlink": t_link_us},
                     "layer_roofline_us": roof_us, "layer_frac": roof_us / (ms_max * 1e3),
                     "nvlink_bytes_rank": nvlink_bytes},
        "cpu_baseline": None,
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "us_per_layer": e2e_ms * 1e3,
                "what": "pinned host tokens+ids -> route/pack -> count exchange -> fused run -> pinned host output"},
        "nccl_a2a_bmm": nccl,
        "gpu_launches": gpu_launches,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_oracle_sample(wl, world)
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier()
    from nvshmem_testing_b200 import symm
    symm.release_all()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
