"""The C-ABI library loads on a host without a GPU, exports every symbol its
header declares, and validates arguments before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest

from nvshmem_testing_b200 import _native as N

HEADER = Path(__file__).resolve().parent.parent / "include" / "moe_ep.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|const char\*)\s+(moe_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 10
    lib = N.lib()
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(N.EXPORTED)


def test_abi_version_and_status_strings():
    lib = N.lib()
    assert lib.moe_ep_abi_version() == N.ABI_VERSION
    assert lib.moe_ep_status_string(N.TIMEOUT) == b"timed out waiting for a peer"
    assert lib.moe_ep_status_string(99) == b"unknown status"


def test_workspace_layout_is_host_only_and_aligned():
    L = N.workspace_layout(8, 32, 7168, 2, 7 * 32 * 256, 8)
    assert L.ctrl_bytes <= L.off_data and L.off_data % 4096 == 0
    assert L.total_bytes >= L.off_data + 2 * 7 * 32 * 256 * 7168 * 2
    offs = [L.off_cmat, L.off_cflag, L.off_dflag, L.off_free, L.off_local]
    assert offs == sorted(offs) and all(o % 256 == 0 for o in offs)
    # count matrix: two parities of [W][W][El] int32
    assert L.off_cflag - L.off_cmat >= 2 * 8 * 8 * 32 * 4
    assert L.off_free - L.off_dflag >= 2 * 8 * 32 * 8 * 4
    # "returned" flags share the free-epoch block; no return region by default
    assert L.off_free + 8 * 4 <= L.off_rflag and L.off_rflag + 8 * 4 <= L.off_local
    assert L.ret_bytes == 0 and L.off_ret + L.ret_bytes <= L.total_bytes


def test_workspace_layout_with_return_region():
    base = N.workspace_layout(8, 32, 7168, 2, 7 * 32 * 256, 8)
    L = N.workspace_layout(8, 32, 7168, 2, 7 * 32 * 256, 8, 8 * 32 * 256, 2048)
    # control and receive regions are unchanged; the return region follows
    assert (L.off_cmat, L.off_rflag, L.off_local, L.ctrl_bytes, L.off_data) == \
        (base.off_cmat, base.off_rflag, base.off_local, base.ctrl_bytes, base.off_data)
    assert L.off_ret % 4096 == 0 and L.off_ret >= L.off_data + 2 * 7 * 32 * 256 * 7168 * 2
    assert L.ret_bytes == 8 * 32 * 256 * 2048 * 2 and L.total_bytes >= L.off_ret + L.ret_bytes
    # the no-allocation entry point's one-rank control region still fits its scratch
    one = N.workspace_layout(1, N.NOALLOC_MAX_EXPERTS, 4096, 2, 0, 1)
    assert one.ctrl_bytes + 256 <= 2048


def test_bad_arguments_are_rejected_before_any_device_call():
    lib = N.lib()
    assert lib.moe_route(None, 0, 10, 1, 4, None, None, None, None, None) == N.BAD_ARG
    assert lib.moe_route(None, 0, 0, 1, 5000, None, None, None, None, None) == N.BAD_ARG
    assert lib.moe_pack_padded(None, 7, 2, None, None, None, 4, 1, None, None) == N.BAD_ARG
    assert lib.moe_ep_run(None, None) == N.BAD_ARG
    p = N.RunParams()
    p.world_size, p.rank, p.local_experts, p.hidden, p.out_dim, p.elem_bytes = 2, 2, 1, 64, 64, 2
    assert lib.moe_ep_run(ctypes.byref(p), None) == N.BAD_ARG  # rank out of range
    p.rank, p.hidden = 0, 60  # H not a multiple of 8
    assert lib.moe_ep_run(ctypes.byref(p), None) == N.BAD_ARG
    bad = N.Layout()
    assert lib.moe_ep_workspace_layout(0, 1, 1, 2, 0, 1, ctypes.byref(bad)) == N.BAD_ARG
    assert lib.moe_ep_workspace_layout_ret(1, 1, 1, 2, 0, 1, -1, 8, ctypes.byref(bad)) == N.BAD_ARG
    assert lib.moe_route_slots(None, 0, 10, 1, 4, None, None, None, None, None, None) == N.BAD_ARG
    c = N.CombineParams()
    assert lib.moe_ep_run_combine(None, ctypes.byref(c), None) == N.BAD_ARG
    c.T, c.K, c.ret_rows = 4, 2, 0  # no return region
    assert lib.moe_ep_run_combine(ctypes.byref(p), ctypes.byref(c), None) == N.BAD_ARG
    c.ret_rows, c.K = 64, 33  # K above the routing limit
    assert lib.moe_ep_run_combine(ctypes.byref(p), ctypes.byref(c), None) == N.BAD_ARG
    # router: E not a multiple of 8, K > E, H not a multiple of 8
    assert lib.moe_router(None, 4, 64, None, 12, 2, None, None, 1, None, None, None) == N.BAD_ARG
    assert lib.moe_router(None, 4, 64, None, 16, 17, None, None, 1, None, None, None) == N.BAD_ARG
    assert lib.moe_router(None, 4, 60, None, 16, 2, None, None, 1, None, None, None) == N.BAD_ARG
    assert lib.moe_router(None, 0, 64, None, 16, 2, None, None, 1, None, None, None) == N.OK  # no tokens: nothing to do


def test_launch_option_words():
    """The host side of the placement and tile-order options: values the
    kernel would reject never reach it."""
    from nvshmem_testing_b200 import alltoall_persistent_gemm as apg
    assert apg.placement(1, 4, 8, 4) == (0, 0)  # one rank: nothing to push, no remote tiles
    assert apg.placement(8, 4, None, 99)[1] == 4  # local_first clamps to El
    assert apg.push_setup(3, 8 | 2) == (3, 10)
    for pw, pm in ((0, 0), (7, 0), (2, 16)):
        with pytest.raises(ValueError):
            apg.push_setup(pw, pm)
    assert apg.sched_setup(1, True, True, 3) == 3 << 4  # one rank: no ready-first or merged tiles
    assert apg.sched_setup(8, True, True, 7) == 1 | 2 | (7 << 4)
    assert apg.sched_setup(2, False, False, 0) == 0
    with pytest.raises(ValueError):
        apg.sched_setup(2, False, False, 16)


def test_status_word_decoding():
    assert N.decode_status_word((3 << 24) | (4 << 16) | 7) == (3, 4, 7)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(N, "_lib", None)
    monkeypatch.setattr(N, "LIB_PATH", tmp_path / "absent.so")
    with pytest.raises(N.MoeEpError):
        N.lib()


def test_fused_gate_up_layout():
    """mlp.fuse_gate_up puts, per 256 columns, gate j..j+63, up j..j+63,
    gate j+64..j+127, up j+64..j+127 (the SwiGLU epilogue's layout)."""
    import torch
    from nvshmem_testing_b200 import mlp
    F = 256
    w = torch.arange(2 * F, dtype=torch.float32).view(1, 1, 2 * F).expand(2, 3, 2 * F).contiguous()
    got = mlp.fuse_gate_up(w)[1, 2].long().tolist()
    want = []
    for s in range(F // 128):
        for c in range(2):
            want += [s * 128 + c * 64 + j for j in range(64)] + [F + s * 128 + c * 64 + j for j in range(64)]
    assert got == want
    with pytest.raises(ValueError):
        mlp.fuse_gate_up(torch.zeros(1, 4, 2 * 96))
