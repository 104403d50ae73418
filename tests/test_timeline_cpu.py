"""The device-timeline summary (timeline.summarize) on a synthetic trace:
window, NVLink bandwidth, per-pair waits."""
import numpy as np

from nvshmem_testing_b200 import _native as N
from nvshmem_testing_b200 import timeline


def _trace(ctas=4):
    F = {n: i for i, n in enumerate(N.TRACE_FIELDS)}
    t = np.zeros((ctas, N.TRACE_WORDS), np.int64)
    t0 = 10_000_000
    for c in range(ctas):
        t[c, F["start"]] = t0 + 100 * c
        t[c, F["counts"]] = t0 + 2_000
        t[c, F["sched"]] = t0 + 6_000
        t[c, F["end"]] = t0 + 1_000_000 + 1_000 * c
        t[c, F["epi_end"]] = t0 + 990_000 + 1_000 * c
        t[c, F["push_items"]] = 10
        t[c, F["push_bytes"]] = 100_000_000
        t[c, F["push_end"]] = t0 + 506_000 - 1_000 * c
    for c in range(0, ctas, 2):  # leaders
        t[c, F["tiles"]] = 5
        t[c, F["flag_wait_ns"]] = 20_000 * (c + 1)
        t[c, F["full_wait_ns"]] = 100_000
        t[c, F["empty_wait_ns"]] = 50_000
        t[c, F["mma_end"]] = t0 + 980_000
        t[c, F["mma_issue_ns"]] = 487_000
    return t


def test_summary_of_a_synthetic_trace():
    s = timeline.summarize(_trace().reshape(-1), 4)
    assert s["layer_us"] == 1003.0  # last end - first start
    assert s["sched_us"] == 6.0 and s["counts_us"] == 2.0
    assert s["push_bytes"] == 400_000_000 and s["push_items"] == 40 and s["push_ctas_active"] == 4
    assert s["push_end_us"] == 506.0 and s["first_push_end_us"] == 503.0
    assert abs(s["push_window_us"] - 500.0) < 1e-9
    assert abs(s["nvlink_out_gbs"] - 800.0) < 1e-6  # 400 MB in 500 us
    assert s["pairs_computing"] == 2 and s["tiles_per_pair"] == {"min": 5, "max": 5}
    assert s["flag_wait_us"] == {"mean": 40.0, "max": 60.0}
    assert s["stage_wait_us"]["mean"] == 100.0
    assert abs(s["mma_issue_busy"] - 0.5) < 1e-9  # 487 us of 974 us
    assert s["gemm_end_us"] == 993.0
