"""Benchmark: fused MoE expert-parallel layer (dispatch + grouped GEMM).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]
                    [--path dispatch_gemm|general|combine|router|mlp]

One process per GPU (torchrun for N > 1).  A step is one call of the fused
layer ``alltoall_persistent_gemm.run`` on this rank's padded, expert-major
token buffer (inputs resident in HBM): count exchange, NVLink dispatch of the
valid rows, and the grouped GEMM over the local experts.  Weak scaling: the
tokens per rank are fixed; experts split E/N per rank.

Printed (rank 0, one JSON line): whole-job TFLOP/s over valid rows (``value``),
µs per layer, the roofline of the fused kernel, the same metric end to end
through the public API from pinned host buffers (``e2e``, with the time of
the host copies alone beside it), the reference's NCCL all_to_all_single +
bmm on the same inputs, the oracle's CPU time on the host cores
(``cpu_baseline``), the oracle's check of this very run (``parity_oracle``:
routing, counts and send buffer bit for bit, sampled expert outputs within
the stated tolerance, padded rows zero), the kernel's device timeline and
achieved NVLink bandwidth (``timeline``, ``nvlink``), and the other
workloads at the same N (``other_configs``).  ``--impl reference`` times the
oracle (the CPU restatement of the reference path) on the host cores
instead, with the reference's CPU/gloo configuration beside it.

``--path`` selects another layer: ``general`` (the unpadded exchange),
``combine`` (with the return path and top-k combine), ``router`` (the step
before the path) or ``mlp`` (the full gated expert MLP).
"""
from __future__ import annotations

import os
import sys

# The reference arm runs on the host cores alone (rank 0): give numpy and
# torch every core before they load (torchrun sets OMP_NUM_THREADS=1).
if "reference" in sys.argv[1:] and "--impl" in sys.argv[1:]:
    _cores = str(os.cpu_count() or 1)
    for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_v] = _cores

import argparse  # noqa: E402
import json  # noqa: E402
import socket  # noqa: E402
import statistics  # noqa: E402
import subprocess  # noqa: E402
import time  # noqa: E402
from datetime import timedelta  # noqa: E402
from pathlib import Path  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from nvshmem_testing_b200 import alltoall_persistent_gemm as apg  # noqa: E402
from nvshmem_testing_b200 import _native, symm, timeline, utils, workloads  # noqa: E402

METRIC = "fused dispatch+grouped-GEMM µs/layer & TFLOP/s, 1/2/4/8 B200 vs NCCL a2a+GEMM"
METRIC_COMBINE = "fused dispatch+grouped-GEMM+return+top-k combine µs/layer & TFLOP/s vs NCCL a2a+GEMM+a2a+combine"
# NVLink 5 per direction per GPU: the nominal 900 GB/s bounds the layer's
# transfer time (the target the layer is held to); this pool's measured peer
# copy, 770 GB/s, is reported beside it, and the run measures its own.
NVLINK_GBS = 900.0
NVLINK_POOL_GBS = 770.0
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# Other workloads measured at every N after the headline (name, overrides, general_a2a).
OTHER_CONFIGS = [("mixtral", {}, False), ("skewed_zipf", {}, False), ("skewed_zipf", {}, True),
                 ("decode", {"T": 16}, False), ("decode", {"T": 256}, False), ("decode", {"T": 1024}, False),
                 ("decode", {"T": 8192}, False)]


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
    (profiles/traffic.txt: lines "workload world bytes [nvlink]"): the bytes,
    and whether the rows crossing NVLink (read by senders, written by peers)
    must be added because the capture ran on one GPU without them."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None, False
    for line in p.read_text().splitlines():
        f = line.split()
        if len(f) >= 3 and not line.startswith("#") and f[0] == workload and f[1] == str(world):
            return int(float(f[2])), len(f) >= 4 and f[3] == "+nvlink"
    return None, False


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


def gather(obj):
    """Every rank's ``obj``, in rank order (on every rank)."""
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


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


# Host time per call of the last ``time_device`` loop (ms): how long the
# host took to issue one step.  A step whose device time is close to this
# is bound by the host's launch path, not by the GPU.
LAST_HOST_MS = [0.0]


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
    h0 = time.perf_counter()
    for _ in range(steps):
        fn()
    LAST_HOST_MS[0] = (time.perf_counter() - h0) * 1e3 / steps
    e.record()
    torch.cuda.synchronize()
    if sampler:
        sampler.mark_end()
    clocks = sampler.stop() if sampler else None
    dist.barrier()
    return s.elapsed_time(e) / steps, clocks


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


class LayerCase:
    """One workload's layer on this rank: seeded inputs resident in HBM (the
    tokens drawn on the host, so that the oracle can redraw every rank's),
    the device routing, the padded or compact send buffer and the counts."""

    def __init__(self, wl, rank: int, world: int, dev, general: bool = False):
        self.wl, self.rank, self.world, self.dev, self.general = wl, rank, world, dev, general
        self.El = El = wl.local_experts(world)
        self.tok_cpu = workloads.tokens(wl, rank)
        self.ids_cpu = workloads.top_idxs(wl, rank)
        self.tokens = self.tok_cpu.to(dev)
        self.ids = self.ids_cpu.to(dev)
        self.weights = workloads.weights(wl, rank, world, device=dev)
        self.routing = utils.route(self.ids, wl.E)
        self.gm = utils.global_max_count(self.routing)
        self.chunk = El * self.gm
        self.padded = utils.pack_padded(self.tokens, self.routing, self.gm)
        self.counts = self.routing.counts
        self.recv_counts = utils.recv_counts_from(self.counts, world)
        self.rc_cpu = self.recv_counts.cpu()
        c_cpu = self.counts.cpu().view(world, El)
        self.rows_in = int(self.rc_cpu.sum())
        self.remote_in = self.rows_in - int(self.rc_cpu[rank].sum())
        self.remote_out = int(c_cpu.sum()) - int(c_cpu[rank].sum())
        self.flops_rank = 2.0 * self.rows_in * wl.H * wl.N
        self.nvlink_bytes = max(self.remote_in, self.remote_out) * wl.H * 2
        if general:
            self.total = int(c_cpu.sum())
            self.compact = utils.pack_compact(self.tokens, self.routing, self.total)
        self.name = wl.name + ("+general_a2a" if general else "") + \
            (f"_T{wl.T}" if wl.name == "decode" else "")

    def step(self, trace=None):
        wl = self.wl
        if self.general:
            return apg.run(self.rank, self.compact, self.total, 1, wl.T, wl.H, wl.E, self.world, None, True,
                           self.weights, self.recv_counts, max_count=self.gm, recv_rows=self.rows_in, trace=trace)
        return apg.run(self.rank, self.padded, self.chunk, 1, wl.T, wl.H, wl.E, self.world, None, False,
                       self.weights, self.recv_counts, trace=trace)

    def nccl(self):
        return nccl_a2a_bmm(self.padded, self.chunk, self.world, self.weights)

    def workspace(self):
        return apg.get_workspace(self.world, self.El, self.wl.H, self.gm, self.dev.index, None, self.rank,
                                 apg.DEFAULT_PUSH_ROWS)

    def allclose_vs_nccl(self) -> bool:
        ours = self.step()
        torch.cuda.synchronize()
        apg.raise_if_device_error(self.workspace())
        ref = self.nccl()
        if self.general:  # drop the padded rows of the NCCL result: cells (le, src) back to back
            gm = self.gm
            ref = torch.cat([ref[le, src * gm:src * gm + int(self.rc_cpu[src, le])]
                             for le in range(self.El) for src in range(self.world)])
        ok = bool(torch.allclose(ours.float(), ref.float(), rtol=1e-2, atol=1e-2))
        del ours, ref
        return ok

    def hbm_bytes(self) -> int:
        """Algorithmic HBM bytes of one launch on this rank: expert weights
        once, every valid row once, the output (padded or compact), and the
        remote rows read for sending plus written by peers."""
        wl = self.wl
        out_rows = self.rows_in if self.general else self.El * self.world * self.gm
        return (self.El * wl.H * wl.N * 2 + self.rows_in * wl.H * 2 + out_rows * wl.N * 2
                + (self.remote_in + self.remote_out) * wl.H * 2)

    def roofline(self, ms_max: float, peaks: dict, peaks_src: str) -> dict:
        peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        hbm = self.hbm_bytes()
        t_gemm = self.flops_rank / (peak * 1e12) * 1e6
        t_hbm = hbm / (hbm_peak * 1e9) * 1e6
        t_link = self.nvlink_bytes / (NVLINK_GBS * 1e9) * 1e6
        roof = max_over_ranks(max(t_gemm, t_hbm, t_link))
        if t_hbm > t_gemm:
            bound, achieved, peak_v, unit = "hbm", hbm / (ms_max * 1e-3) / 1e9, hbm_peak, "GB/s"
            note = f"{peaks_src} hbm_gbs"
        else:
            bound, achieved, peak_v, unit = "tensor", self.flops_rank / (ms_max * 1e-3) / 1e12, peak, "TFLOP/s"
            note = f"{peaks_src} bf16_tflops (burst)"
        traffic, add_link = load_traffic(self.wl.name if not self.general else self.name, self.world)
        if traffic is not None and add_link:
            traffic += (self.remote_in + self.remote_out) * self.wl.H * 2
        return {"bound": bound, "achieved": achieved, "peak": peak_v, "unit": unit, "frac": achieved / peak_v,
                "peak_source": note, "traffic": traffic,
                "traffic_source": ("ncu capture of the same launch" if traffic is not None and not add_link else
                                   "ncu capture of the receiver's GEMM on one GPU + rows crossing NVLink (read "
                                   "for sending, written by peers), counted" if traffic is not None else None),
                "algorithmic_hbm_bytes": hbm, "tensor_tflops": self.flops_rank / (ms_max * 1e-3) / 1e12,
                "bounds_us": {"tensor": t_gemm, "hbm": t_hbm, "nvlink": t_link},
                "layer_roofline_us": roof, "layer_frac": roof / (ms_max * 1e3),
                "nvlink_bytes_rank": self.nvlink_bytes, "nvlink_gbs_bound": NVLINK_GBS}

    def timeline(self) -> dict:
        """One traced launch after the timed region: per-rank device timeline
        and the NVLink bandwidth the dispatch reached."""
        sms = torch.cuda.get_device_properties(self.dev).multi_processor_count
        tr = torch.zeros(sms * _native.TRACE_WORDS, dtype=torch.int64, device=self.dev)
        # Start every rank together, so no rank's timeline holds another
        # rank's late start as waiting.
        torch.cuda.synchronize()
        if dist.is_initialized():
            dist.barrier()
        self.step(trace=tr)
        torch.cuda.synchronize()
        t = tr.view(-1, _native.TRACE_WORDS).cpu()
        n = int((t[:, 0] != 0).sum())
        mine = timeline.summarize(t.flatten(), n)
        mine["rank"] = self.rank
        return gather(mine)

    def oracle_check(self, experts: list[int], rows_per_cell: int, send_buffer: bool = True) -> dict:
        """The oracle as the checker of this run (outside every timed
        region): this rank's routing (counts, offsets, permutation) and, with
        every rank's ids redrawn on the host, the receive counts and gm, bit
        for bit; the send buffer bit for bit; for the sampled local experts,
        up to ``rows_per_cell`` rows of every source's cell against fp32
        GEMMs of the redrawn source tokens (max error relative to the
        largest reference magnitude, and allclose(rtol=1e-2, atol=1e-2));
        and every padded output row exactly zero.  Gathered over ranks."""
        import oracle
        wl, W, me, El, gm = self.wl, self.world, self.rank, self.El, self.gm
        t0 = time.perf_counter()
        ids = [self.ids_cpu.numpy() if r == me else workloads.top_idxs(wl, r).numpy() for r in range(W)]
        routed = [oracle.bucketize(i, wl.E) for i in ids]
        c, o, p = routed[me]
        n = int(o[-1])
        res = {"rank": me}
        res["routing_bit_exact"] = bool(np.array_equal(self.counts.cpu().numpy(), c) and
                                        np.array_equal(self.routing.offsets.cpu().numpy(), o) and
                                        np.array_equal(self.routing.perm[:n].cpu().numpy(), p))
        rcm = oracle.recv_counts_matrix([r[0] for r in routed], me, W)
        res["recv_counts_bit_exact"] = bool(np.array_equal(self.rc_cpu.numpy(), rcm))
        res["gm_matches"] = gm == max(oracle.local_max(r[0]) for r in routed)
        tok_bits = bf16_bits(self.tok_cpu)
        if send_buffer:
            if self.general:
                ref_send = oracle.compact_coalesce(tok_bits, c, o, p)
                res["send_buffer_bit_exact"] = bool(np.array_equal(bf16_bits(self.compact), ref_send))
            else:
                ref_send = oracle.pad_coalesce(tok_bits, c, o, p, gm)
                res["send_buffer_bit_exact"] = bool(np.array_equal(bf16_bits(self.padded), ref_send))
            del ref_send
        out = self.step()
        torch.cuda.synchronize()
        apg.raise_if_device_error(self.workspace())
        # cell (le, src) of the compact output starts after every earlier (le', src') cell
        ooff = np.concatenate([[0], np.cumsum(self.rc_cpu.numpy().T.reshape(-1))])
        err = scale = 0.0
        close, rows_checked = True, 0
        src_tok = {}
        for le in experts:
            e = me * El + le
            w = oracle.bf16_bits_to_f32(bf16_bits(self.weights[le]))
            for src in range(W):
                cnt = int(rcm[src, le])
                if cnt == 0:
                    continue
                rows = np.unique(np.linspace(0, cnt - 1, min(rows_per_cell, cnt)).round().astype(np.int64))
                if src not in src_tok:
                    src_tok[src] = tok_bits if src == me else bf16_bits(workloads.tokens(wl, src))
                ref = oracle.expert_cell(oracle.bf16_bits_to_f32(src_tok[src]), routed[src], e, w, rows)
                idx = torch.as_tensor(rows, device=self.dev)
                if self.general:
                    got = out[int(ooff[le * W + src]) + idx]
                else:
                    got = out[le, src * gm + idx]
                g = got.float().cpu().numpy()
                err = max(err, float(np.abs(g - ref).max()))
                scale = max(scale, float(np.abs(ref).max()))
                close &= bool(np.allclose(g, ref, rtol=1e-2, atol=1e-2))
                rows_checked += rows.size
        res["max_rel_err"] = err / max(scale, 1e-30)
        res["allclose"] = close
        res["rows_checked"] = rows_checked
        if not self.general:
            i = torch.arange(gm, device=self.dev)
            valid = (i[None, None, :] < self.recv_counts.t()[:, :, None]).reshape(El, W * gm)
            res["padded_rows_zero"] = bool(out.masked_fill(valid[..., None], 0).abs().amax().item() == 0)
        del out
        res["seconds"] = time.perf_counter() - t0
        allr = gather(res)
        keys_all = ["routing_bit_exact", "recv_counts_bit_exact", "gm_matches", "send_buffer_bit_exact", "allclose",
                    "padded_rows_zero"]
        summary = {k: all(r[k] for r in allr) for k in keys_all if k in res}
        summary["max_rel_err"] = max(r["max_rel_err"] for r in allr)
        summary["tolerance"] = "max |err| <= 1e-2 x max |ref| and allclose(rtol=1e-2, atol=1e-2)"
        summary["ok"] = all(v for k, v in summary.items() if isinstance(v, bool)) and summary["max_rel_err"] <= 1e-2
        summary["rows_checked"] = sum(r["rows_checked"] for r in allr)
        summary["experts_sampled_per_rank"] = len(experts)
        summary["oracle_seconds_max"] = max(r["seconds"] for r in allr)
        return summary


def measure_case(case: LayerCase, steps: int, warmup: int, peaks, peaks_src, nccl_steps: int,
                 sampler_device=None, no_nccl: bool = False) -> dict:
    """Device-timed µs/layer of ``case.step`` (max over ranks), the NCCL arm
    on the same inputs and the roofline."""
    ok = case.allclose_vs_nccl() if not no_nccl else None
    ms, clocks = time_device(case.step, steps, warmup, sampler_device=sampler_device)
    host_max = max_over_ranks(LAST_HOST_MS[0])
    ms_max = max_over_ranks(ms)
    flops_total = sum_over_ranks(case.flops_rank)
    r = {"workload": case.name, "us_per_layer": ms_max * 1e3, "value": flops_total / (ms_max * 1e-3) / 1e12,
         "unit": "TFLOP/s", "gm": case.gm, "local_experts": case.El, "parity_vs_nccl_allclose": ok,
         "host_us_per_call": host_max * 1e3,
         "roofline": case.roofline(ms_max, peaks, peaks_src), "_flops_total": flops_total, "_ms": ms_max,
         "_clocks": clocks}
    if not no_nccl:
        ms_n, _ = time_device(case.nccl, nccl_steps, min(warmup, 3))
        ms_n = max_over_ranks(ms_n)
        r["nccl_a2a_bmm"] = {"us_per_layer": ms_n * 1e3, "value": flops_total / (ms_n * 1e-3) / 1e12,
                             "unit": "TFLOP/s",
                             "what": "NCCL all_to_all_single + view/permute/flatten + torch.bmm over padded rows"}
        r["speedup_vs_nccl"] = ms_n / ms_max
    return r


def e2e_measure(case: LayerCase, steps: int) -> dict:
    """The same metric end to end through the public API
    (``alltoall_persistent_gemm.layer``: device routing, padded pack, fused
    exchange + GEMM with the counts exchanged in the kernel): every step
    copies its token rows and routing ids from pinned host memory to the
    device and its [El, W*gm, N] output back to pinned host memory.  Steps
    are pipelined over three streams (host-to-device copies, compute,
    device-to-host copies) with double-buffered inputs and outputs, the way
    a serving loop overlaps them; the timed region (CUDA events, max over
    ranks) spans all copies of every step.  Also reported: the same loop one
    step at a time (``serial_us``), and the copies alone (``copy_floor_us``:
    the same bytes over the same streams with no compute)."""
    wl, dev = case.wl, case.dev
    tok_host = case.tok_cpu.pin_memory()
    ids_host = case.ids_cpu.pin_memory()
    shape = (case.El, case.world * case.gm, wl.N)
    out_host = [torch.empty(shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    tok_dev = [torch.empty_like(case.tokens) for _ in range(2)]
    ids_dev = [torch.empty_like(case.ids) for _ in range(2)]
    out_dev = torch.empty(shape, dtype=torch.bfloat16, device=dev)  # the copy-floor loop's source
    h2d_bytes = tok_host.numel() * tok_host.element_size() + ids_host.numel() * ids_host.element_size()
    d2h_bytes = out_host[0].numel() * out_host[0].element_size()
    comp = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    for ev in ev_done:
        ev.record(comp)

    def one(i: int, compute: bool = True):
        b = i & 1
        h2d.wait_event(ev_done[b])  # the step two back has finished reading buffers b
        with torch.cuda.stream(h2d):
            tok_dev[b].copy_(tok_host, non_blocking=True)
            ids_dev[b].copy_(ids_host, non_blocking=True)
            ev_in[b].record(h2d)
        comp.wait_event(ev_in[b])
        out = apg.layer(tok_dev[b], ids_dev[b], wl.E, case.weights) if compute else out_dev
        ev_done[b].record(comp)
        d2h.wait_event(ev_done[b])
        with torch.cuda.stream(d2h):
            out_host[b].copy_(out, non_blocking=True)
        if compute:
            out.record_stream(d2h)

    def timed(n: int, compute: bool = True, serial: bool = False) -> float:
        for i in range(3):
            one(i, compute)
        comp.wait_stream(d2h)
        torch.cuda.synchronize(dev)
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(comp)
        for i in range(n):
            one(i, compute)
            if serial:
                comp.wait_stream(d2h)
                comp.synchronize()
        comp.wait_stream(d2h)
        e.record(comp)
        torch.cuda.synchronize(dev)
        dist.barrier()
        return max_over_ranks(s.elapsed_time(e) / n)

    ms = timed(steps)
    # the pipelined loop's last output against a direct call on the resident inputs
    ref = apg.layer(case.tokens, case.ids, wl.E, case.weights)
    torch.cuda.synchronize(dev)
    same = bool(torch.equal(out_host[(steps - 1) & 1], ref.cpu()))
    del ref
    ms_serial = timed(max(steps // 2, 3), serial=True)
    ms_floor = timed(steps, compute=False)
    flops_total = sum_over_ranks(case.flops_rank)
    return {"value": flops_total / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d_bytes,
            "d2h_bytes_per_step": d2h_bytes, "us_per_layer": ms * 1e3, "serial_us": ms_serial * 1e3,
            "copy_floor_us": ms_floor * 1e3, "frac_of_copy_floor": ms_floor / ms,
            "output_equals_resident_call": same,
            "what": "pinned host tokens+ids -> alltoall_persistent_gemm.layer (device routing, pack, fused "
                    "exchange+GEMM, counts exchanged in the kernel) -> pinned host output; three streams, "
                    "double-buffered"}


def nvlink_probe(case: LayerCase) -> dict | None:
    """Copy-engine peer copies into the workspace receive region of other
    ranks (every rank at once): a ring (each GPU sends to one peer and
    receives from one) and an all-to-all (W-1 concurrent copies, one per
    peer).  GB/s per direction per GPU, max over ranks of the time."""
    if case.world == 1:
        return None
    try:
        from cuda.bindings import runtime as cr
    except Exception as exc:  # pragma: no cover - the image ships cuda-python
        return {"error": f"cuda-python unavailable: {exc}"}
    ws = case.workspace()
    W, me = case.world, case.rank
    bases = ws.peer_bases.cpu().tolist()
    region = (ws.layout.total_bytes - ws.layout.off_data) // 2
    nbytes = int(min(256 << 20, region, case.padded.numel() * 2)) // 4096 * 4096
    src = case.padded.data_ptr()
    kind = cr.cudaMemcpyKind.cudaMemcpyDeviceToDevice
    streams = [torch.cuda.Stream(case.dev) for _ in range(W - 1)]
    res = {}
    part = nbytes // (W - 1) // 4096 * 4096
    for pattern in ("ring", "all_to_all", "shifts"):
        def go():
            if pattern == "ring":  # every rank to its neighbour: a permutation
                peers = [((me + 1) % W, nbytes, streams[0])]
            elif pattern == "all_to_all":  # every rank to every peer at once
                peers = [((me + q) % W, part, streams[q - 1]) for q in range(1, W)]
            else:  # W-1 permutations one after another (shift by q), one stream
                peers = [((me + q) % W, part, streams[0]) for q in range(1, W)]
            for d, n, st in peers:
                # senders to one peer write disjoint parts of its receive region
                dst = int(bases[d]) + int(ws.layout.off_data) + (me * n if pattern != "ring" else 0)
                err, = cr.cudaMemcpyAsync(dst, src, n, kind, st.cuda_stream)
                if err != cr.cudaError_t.cudaSuccess:
                    raise RuntimeError(f"cudaMemcpyAsync: {err}")
            cur = torch.cuda.current_stream(case.dev)
            for st in {id(x[2]): x[2] for x in peers}.values():
                cur.wait_stream(st)
        try:
            for _ in range(2):
                go()
            ms, _ = time_device(go, 5, 1)
            ms = max_over_ranks(ms)
            moved = nbytes if pattern == "ring" else part * (W - 1)
            res[f"{pattern}_gbs"] = moved / (ms * 1e-3) / 1e9
        except Exception as exc:
            res[f"{pattern}_error"] = str(exc)[:200]
    res["bytes"] = nbytes
    res["what"] = ("copy-engine cudaMemcpyAsync into peers' cuMem-mapped workspaces, all ranks at once: ring (one "
                   "peer), all_to_all (W-1 peers at once), shifts (W-1 permutations in turn)")
    return res
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
            "gpu_launches": args.steps * (1 if wl.E <= 256 else 3),  # one router kernel (E <= 256)
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
        self.cores = host_threads()
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


def host_threads() -> int:
    """Threads the BLAS behind numpy actually uses (the core count stated
    beside every CPU figure)."""
    try:
        from threadpoolctl import threadpool_info
        return int(max([i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
                       or [os.cpu_count() or 1]))
    except Exception:
        return os.cpu_count() or 1


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


def _gloo_worker(rank: int, world: int, port: int, steps: int, warmup: int, threads: int, q) -> None:
    """One rank of the reference's CPU/gloo configuration (fp32, T=128,
    H=256, E=4 over 2 ranks, top-1, N=512), stepped with the oracle's
    restatement of that path (routing, count all-to-all, equal-split
    all-to-all, bmm); each step's wall time."""
    try:
        import oracle.gloo_baseline as gb
        torch.set_num_threads(threads)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60))
        wl = workloads.get("cpu_gloo")
        tok = workloads.tokens(wl, rank)
        ids = workloads.top_idxs(wl, rank).numpy()
        w = workloads.weights(wl, rank, world)
        times = []
        for i in range(warmup + steps):
            dist.barrier()
            t0 = time.perf_counter()
            out, rc = gb.gloo_layer(tok, ids, wl.E, w)
            dt = time.perf_counter() - t0
            if i >= warmup:
                times.append(dt)
        flops = 2.0 * float(rc.sum()) * wl.H * wl.N  # valid rows this rank multiplied
        q.put((rank, times, flops, out.shape))
        dist.destroy_process_group()
    except Exception as exc:  # reported by the parent
        q.put((rank, None, str(exc), None))


def time_cpu_gloo(steps: int = 20, warmup: int = 3) -> dict:
    """The reference's CPU/gloo configuration on the host cores: two
    processes (spawned), the cores split between them."""
    import multiprocessing as mp
    world = 2
    threads = max((os.cpu_count() or 2) // world, 1)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, steps, warmup, threads, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            r, times, flops, shape = q.get(timeout=300)
            got[r] = (times, flops, shape)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    if any(v[0] is None for v in got.values()):
        return {"error": "; ".join(str(v[1]) for v in got.values() if v[0] is None)}
    per_step = [max(got[r][0][i] for r in range(world)) for i in range(steps)]
    med = statistics.median(per_step)
    flops = sum(got[r][1] for r in range(world))
    return {"us_per_layer": med * 1e6, "value": flops / med / 1e12, "unit": "TFLOP/s", "world_size": world,
            "cores": threads * world, "threads_per_rank": threads, "dtype": "f32", "steps": steps,
            "what": "CPU/gloo configuration (T=128/rank, H=256, E=4, top-1, N=512, fp32): the oracle's routing + "
                    "count all_to_all + equal-split all_to_all_single + bmm on 2 gloo processes; median step, "
                    "max over ranks"}


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
    if not args.no_cpu_gloo:
        line["cpu_gloo_config"] = time_cpu_gloo()
    print(json.dumps(line), flush=True)
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
    ap.add_argument("--no-cpu-gloo", action="store_true", help="reference arm: skip the CPU/gloo configuration")
    ap.add_argument("--no-nccl", action="store_true")
    ap.add_argument("--no-oracle", action="store_true", help="skip the oracle's check of the run")
    ap.add_argument("--no-other", action="store_true", help="skip the other workloads")
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
    peaks, peaks_src = load_peaks()
    wl = workloads.get(args.workload, dtype=torch.bfloat16, **overrides(args))
    case = LayerCase(wl, rank, world, dev, general=args.path == "general")

    head = measure_case(case, args.steps, args.warmup, peaks, peaks_src, max(args.steps // 3, 10),
                        sampler_device=local, no_nccl=args.no_nccl)
    ms_max, flops_total, clocks = head.pop("_ms"), head.pop("_flops_total"), head.pop("_clocks")
    tl = case.timeline()
    nv = nvlink_probe(case) if world > 1 else None
    nvlink = None
    if world > 1:
        ach = [t.get("nvlink_out_gbs") for t in tl]
        ach = [a for a in ach if a is not None]
        nvlink = {"achieved_out_gbs_per_rank": ach, "achieved_out_gbs_min": min(ach) if ach else None,
                  "nominal_gbs": NVLINK_GBS, "pool_measured_peer_copy_gbs": NVLINK_POOL_GBS,
                  "frac_of_nominal": (min(ach) / NVLINK_GBS) if ach else None,
                  "probe": nv,
                  "what": "bytes each rank stored into peers during one traced launch / (schedule ready -> "
                          "last push item done), from the kernel's device timeline"}
    e2e = e2e_measure(case, args.e2e_steps) if args.path == "dispatch_gemm" else None
    parity = None if args.no_oracle else case.oracle_check(sorted({0, case.El - 1}), 64)
    line = {
        "metric": METRIC, "value": flops_total / (ms_max * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "us_per_layer": ms_max * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded)",
        "config": {"workload": case.name, "tokens_per_rank": wl.T, "hidden": wl.H, "experts": wl.E,
                   "local_experts": case.El, "top_k": wl.K, "out_dim": wl.N, "routing": wl.routing, "gm": case.gm,
                   "parallelism": f"ep{world}", "l2": "inputs larger than L2 (weights and tokens > 126 MB)",
                   "push_ctas": apg.placement(world, case.El)[0], "local_first": apg.placement(world, case.El)[1],
                   "push_warps": apg.push_setup()[0], "push_mode": apg.push_setup()[1],
                   "ready_first": apg.DEFAULT_READY_FIRST and world > 1, "merged": apg.DEFAULT_MERGED and world > 1,
                   "row_groups": apg.DEFAULT_ROW_GROUPS,
                   "push_rows": apg.DEFAULT_PUSH_ROWS},
        "parity_vs_nccl_allclose": head["parity_vs_nccl_allclose"],
        "host_us_per_call": head["host_us_per_call"],
        "parity_oracle": parity,
        "roofline": head["roofline"],
        "cpu_baseline": None,
        "e2e": e2e,
        "nccl_a2a_bmm": head.get("nccl_a2a_bmm"),
        "speedup_vs_nccl": head.get("speedup_vs_nccl"),
        "timeline": {"rank0": tl[0], "slowest_rank": max(tl, key=lambda t: t["layer_us"])},
        "nvlink": nvlink,
        "gpu_launches": args.steps,  # one fused kernel per step
        "clocks": clocks,
    }
    del case
    torch.cuda.synchronize()
    symm.release_all()
    torch.cuda.empty_cache()
    if not args.no_other and args.path == "dispatch_gemm" and not args.tokens and not args.experts:
        others = []
        for name, over, general in OTHER_CONFIGS:
            w2 = workloads.get(name, dtype=torch.bfloat16, **over)
            if w2.E % world:
                continue
            c2 = LayerCase(w2, rank, world, dev, general=general)
            steps2 = 10 if w2.T >= 1024 else 20
            r = measure_case(c2, steps2, 3, peaks, peaks_src, 10, no_nccl=args.no_nccl)
            for k in ("_ms", "_flops_total", "_clocks"):
                r.pop(k)
            rf = r["roofline"]
            r["roofline"] = {k: rf[k] for k in ("bound", "frac", "layer_roofline_us", "layer_frac", "bounds_us")}
            r["parity_oracle"] = None if args.no_oracle else c2.oracle_check([c2.El // 2], 16, send_buffer=False)
            tl2 = c2.timeline()
            slow = max(tl2, key=lambda t: t["layer_us"])
            r["timeline_slowest_rank"] = {k: slow.get(k) for k in ("layer_us", "counts_us", "sched_us", "push_end_us",
                                                                   "nvlink_out_gbs", "gemm_end_us", "flag_wait_us")}
            others.append(r)
            del c2
            torch.cuda.synchronize()
            symm.release_all()
            torch.cuda.empty_cache()
        line["other_configs"] = others
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_oracle_sample(wl, world)
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier()
    symm.release_all()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
