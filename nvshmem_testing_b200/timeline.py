"""Summary of the fused kernel's per-CTA device timeline (the ``trace``
argument of ``alltoall_persistent_gemm.run``).

Each CTA records globaltimer stamps and counters (``_native.TRACE_FIELDS``):
kernel entry, counts ready, schedule built, the ends of the producer, MMA,
epilogue and push roles, and the time its roles spent waiting.  From one
launch's records this module derives where the launch spent its time and
the bandwidth the dispatch reached over NVLink:

* ``layer_us``: first CTA entry to last CTA exit;
* ``push_window_us``: schedule ready (first CTA) to the last push item's end
  (the exchange's duration as the senders see it) and
  ``nvlink_out_gbs`` = bytes this rank stored into peers / that window;
* ``first_push_end_us`` / ``gemm_end_us`` (last epilogue) / ``tail_us`` (last
  epilogue end minus the median one);
* per computing pair (leader CTAs): mean and max of the producer's flag wait
  (rows not yet arrived), the MMA issuer's wait for loaded stages, the
  producer's wait for free stages, and the issuer's busy fraction.
"""
from __future__ import annotations

import numpy as np

from ._native import TRACE_FIELDS, TRACE_WORDS

_F = {n: i for i, n in enumerate(TRACE_FIELDS)}


def summarize(trace, num_ctas: int) -> dict:
    """``trace``: the int64 device (or host) tensor / array passed to ``run``,
    at least ``num_ctas * TRACE_WORDS`` words.  Returns a dict of floats
    (microseconds, GB/s, counts)."""
    t = np.asarray(trace.cpu().numpy() if hasattr(trace, "cpu") else trace, dtype=np.int64)
    t = t[:num_ctas * TRACE_WORDS].reshape(num_ctas, TRACE_WORDS)
    col = lambda n: t[:, _F[n]]
    start = col("start")
    t0 = int(start.min())
    us = lambda x: (np.asarray(x, dtype=np.float64) - t0) / 1e3
    leaders = t[0::2]
    tiles = leaders[:, _F["tiles"]]
    computing = tiles > 0
    items = col("push_items")
    pushed = col("push_bytes")
    pushers = items > 0
    out = {
        "layer_us": float(us(col("end").max())),
        "counts_us": float(np.median(us(col("counts")))),
        "sched_us": float(np.median(us(col("sched")))),
        "push_items": int(items.sum()),
        "push_bytes": int(pushed.sum()),
        "push_ctas_active": int(pushers.sum()),
    }
    sched0 = float(us(col("sched")).min())
    if pushers.any():
        pend = us(col("push_end")[pushers])
        window = float(pend.max()) - sched0
        out["first_push_end_us"] = float(pend.min())
        out["push_end_us"] = float(pend.max())
        out["push_window_us"] = window
        out["nvlink_out_gbs"] = float(pushed.sum()) / (window * 1e-6) / 1e9 if window > 0 else None
    epi = us(t[:, _F["epi_end"]][np.repeat(computing, 2)[:num_ctas]]) if computing.any() else np.zeros(0)
    if epi.size:
        out["gemm_end_us"] = float(epi.max())
        out["tail_us"] = float(epi.max() - np.median(epi))
    if computing.any():
        lw = leaders[computing]
        span = (lw[:, _F["mma_end"]] - np.maximum(lw[:, _F["sched"]], 0)).astype(np.float64)
        issue = lw[:, _F["mma_issue_ns"]].astype(np.float64)
        for name, key in (("flag_wait_us", "flag_wait_ns"), ("stage_wait_us", "full_wait_ns"),
                          ("free_stage_wait_us", "empty_wait_ns"), ("acc_wait_us", "acc_wait_ns")):
            v = lw[:, _F[key]].astype(np.float64) / 1e3
            out[name] = {"mean": float(v.mean()), "max": float(v.max())}
        out["pairs_computing"] = int(computing.sum())
        out["tiles_per_pair"] = {"min": int(tiles[computing].min()), "max": int(tiles[computing].max())}
        with np.errstate(divide="ignore", invalid="ignore"):
            busy = np.where(span > 0, issue / span, 0.0)
        out["mma_issue_busy"] = float(busy.mean())
    return out
