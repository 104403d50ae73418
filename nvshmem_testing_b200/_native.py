"""ctypes binding of libmoe_ep.so (the C ABI declared in include/moe_ep.h).

The library is built in-tree by ``nvshmem_testing_b200.build``.  There is no
fallback: if the library is missing or a symbol is absent, importing the
binding raises, and every device operation of this package raises with it.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libmoe_ep.so"

OK, BAD_ARG, CUDA_ERR, TIMEOUT, CAPACITY, BAD_ROUTE, SCRATCH_LIMIT = 0, 1, 2, 3, 4, 5, 6
STATUS_NAMES = {OK: "ok", BAD_ARG: "bad argument", CUDA_ERR: "CUDA error", TIMEOUT: "timed out waiting for a peer",
                CAPACITY: "receive capacity exceeded", BAD_ROUTE: "bad routing input",
                SCRATCH_LIMIT: "size exceeds the fixed scratch of moe_ep_run_noalloc"}
NOALLOC_MAX_EXPERTS = 64
PUSH_BULK, PUSH_BY_DESTINATION, PUSH_HYBRID, PUSH_L2_STREAM = 1, 2, 4, 8
SCHED_READY_FIRST, SCHED_MERGED, SCHED_ROW_GROUPS_SHIFT = 1, 2, 4
ABI_VERSION = 3

# Every symbol include/moe_ep.h declares.
EXPORTED = ["moe_ep_abi_version", "moe_ep_status_string", "moe_ep_num_sms", "moe_route", "moe_pack_padded",
            "moe_symm_alloc", "moe_symm_import", "moe_symm_free", "moe_ep_workspace_layout", "moe_ep_workspace_reset", "moe_ep_run",
            "moe_ep_read_status", "moe_ep_run_noalloc", "moe_route_slots", "moe_ep_workspace_layout_ret",
            "moe_ep_run_combine", "moe_pack_compact", "moe_ep_run_compact", "moe_router", "moe_swiglu",
            "moe_ep_run_compact_swiglu", "moe_publish_i32"]


class MoeEpError(RuntimeError):
    """A libmoe_ep call or a device-side check failed."""

    def __init__(self, code: int, what: str, detail: str = ""):
        self.code = code
        msg = f"{what}: status {code} ({STATUS_NAMES.get(code, 'unknown')})"
        super().__init__(msg + (f" {detail}" if detail else ""))


class Layout(ctypes.Structure):
    _fields_ = [("off_cmat", ctypes.c_uint64), ("off_cflag", ctypes.c_uint64), ("off_dflag", ctypes.c_uint64),
                ("off_free", ctypes.c_uint64), ("off_local", ctypes.c_uint64), ("ctrl_bytes", ctypes.c_uint64),
                ("off_data", ctypes.c_uint64), ("total_bytes", ctypes.c_uint64), ("off_rflag", ctypes.c_uint64),
                ("off_ret", ctypes.c_uint64), ("ret_bytes", ctypes.c_uint64)]


class RunParams(ctypes.Structure):
    _fields_ = [("world_size", ctypes.c_int32), ("rank", ctypes.c_int32), ("local_experts", ctypes.c_int32),
                ("hidden", ctypes.c_int32), ("out_dim", ctypes.c_int32), ("elem_bytes", ctypes.c_int32),
                ("gm", ctypes.c_int64), ("tokens", ctypes.c_void_p), ("weights", ctypes.c_void_p),
                ("recv_counts", ctypes.c_void_p), ("out", ctypes.c_void_p), ("peer_bases", ctypes.c_void_p),
                ("local_base", ctypes.c_uint64), ("cap_rows", ctypes.c_int64), ("push_rows", ctypes.c_int32),
                ("max_chunks", ctypes.c_int32), ("epoch", ctypes.c_uint32), ("num_ctas", ctypes.c_uint32),
                ("timeout_ns", ctypes.c_uint64), ("status_host", ctypes.c_void_p), ("trace", ctypes.c_void_p),
                ("push_ctas", ctypes.c_int32), ("local_first", ctypes.c_int32),
                ("counts_are_send", ctypes.c_int32), ("push_warps", ctypes.c_int32), ("push_mode", ctypes.c_int32),
                ("sched_mode", ctypes.c_int32)]


class CombineParams(ctypes.Structure):
    _fields_ = [("top_idxs", ctypes.c_void_p), ("top_vals", ctypes.c_void_p), ("slots", ctypes.c_void_p),
                ("y", ctypes.c_void_p), ("T", ctypes.c_int64), ("ret_rows", ctypes.c_int64), ("K", ctypes.c_int32),
                ("ids_are_int64", ctypes.c_int32), ("vals_are_bf16", ctypes.c_int32), ("reserved", ctypes.c_int32)]


TRACE_WORDS = 24
TRACE_FIELDS = ["start", "counts", "sched", "producer_end", "mma_end", "epi_end", "push_end", "zero_end", "end",
                "tiles", "flag_wait_ns", "full_wait_ns", "push_items", "push_bytes", "empty_wait_ns",
                "epi_wait_ns", "acc_wait_ns", "mma_issue_ns", "kblocks"]


_lib = None


def lib() -> ctypes.CDLL:
    """Load libmoe_ep.so once; raise if it is missing or incomplete."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise MoeEpError(CUDA_ERR, "libmoe_ep.so not built",
                         f"(expected {LIB_PATH}; run `python -m nvshmem_testing_b200.build`)")
    L = ctypes.CDLL(os.fspath(LIB_PATH))
    for name in EXPORTED:
        if not hasattr(L, name):
            raise MoeEpError(CUDA_ERR, f"libmoe_ep.so lacks {name}")
    c_int, c_i64, c_vp, c_u64, c_sz = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_size_t
    P = ctypes.POINTER
    L.moe_ep_abi_version.restype = c_int
    L.moe_ep_status_string.restype = ctypes.c_char_p
    L.moe_ep_status_string.argtypes = [c_int]
    L.moe_ep_num_sms.argtypes = [c_int, P(c_int)]
    L.moe_route.argtypes = [c_vp, c_int, c_i64, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp]
    L.moe_route_slots.argtypes = [c_vp, c_int, c_i64, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]
    L.moe_pack_padded.argtypes = [c_vp, c_i64, c_int, c_vp, c_vp, c_vp, c_int, c_i64, c_vp, c_vp]
    L.moe_symm_alloc.argtypes = [c_int, c_sz, P(c_sz), P(c_u64), P(c_int), P(c_u64)]
    L.moe_symm_import.argtypes = [c_int, c_int, c_sz, P(c_u64), P(c_u64)]
    L.moe_symm_free.argtypes = [c_u64, c_sz, c_u64]
    L.moe_ep_workspace_layout.argtypes = [c_int, c_int, c_i64, c_int, c_i64, c_int, P(Layout)]
    L.moe_ep_workspace_layout_ret.argtypes = [c_int, c_int, c_i64, c_int, c_i64, c_int, c_i64, c_i64, P(Layout)]
    L.moe_ep_workspace_reset.argtypes = [c_u64, P(Layout), c_vp]
    L.moe_ep_run.argtypes = [P(RunParams), c_vp]
    L.moe_ep_run_noalloc.argtypes = [P(RunParams), c_vp]
    L.moe_ep_run_combine.argtypes = [P(RunParams), P(CombineParams), c_vp]
    L.moe_ep_run_compact.argtypes = [P(RunParams), c_i64, c_i64, c_vp]
    L.moe_pack_compact.argtypes = [c_vp, c_i64, c_int, c_vp, c_i64, c_vp, c_vp]
    L.moe_swiglu.argtypes = [c_vp, c_i64, ctypes.c_int32, c_vp, c_vp]
    L.moe_ep_run_compact_swiglu.argtypes = [P(RunParams), c_i64, c_i64, c_vp]
    L.moe_router.argtypes = [c_vp, c_i64, ctypes.c_int32, c_vp, ctypes.c_int32, ctypes.c_int32, c_vp, c_vp,
                             ctypes.c_int32, c_vp, c_vp, c_vp]
    L.moe_ep_read_status.argtypes = [c_u64, P(Layout), P(ctypes.c_uint32)]
    L.moe_publish_i32.argtypes = [c_vp, c_i64, c_vp, c_vp]
    for name in EXPORTED:
        if name not in ("moe_ep_status_string",):
            getattr(L, name).restype = c_int
    if L.moe_ep_abi_version() != ABI_VERSION:
        raise MoeEpError(CUDA_ERR, "libmoe_ep.so ABI version mismatch")
    _lib = L
    return L


def check(code: int, what: str) -> None:
    if code != OK:
        raise MoeEpError(code, what)


def decode_status_word(w: int) -> tuple[int, int, int]:
    """Split a device status word into (code, site, detail)."""
    return (w >> 24) & 0xFF, (w >> 16) & 0xFF, w & 0xFFFF


def workspace_layout(W: int, El: int, H: int, elem_bytes: int, cap_rows: int, max_chunks: int,
                     ret_rows: int = 0, ret_cols: int = 0) -> Layout:
    L = Layout()
    check(lib().moe_ep_workspace_layout_ret(W, El, H, elem_bytes, cap_rows, max_chunks, ret_rows, ret_cols,
                                            ctypes.byref(L)), "moe_ep_workspace_layout_ret")
    return L
