"""Symmetric workspaces over cuMem VMM (one per process group and shape).

Replaces ``_get_symm_buffers`` / ``_SYMM_CACHE`` of the reference
(alltoall_persistent_gemm.py:161-204), which allocate a receive buffer and a
signal buffer through torch symmetric memory and rendezvous them through the
c10d store.  Here each rank

1. allocates one device region through ``moe_symm_alloc`` (cuMemCreate with a
   POSIX file-descriptor handle, mapped read-write on its own GPU),
2. zeroes its control region,
3. passes the file descriptor to every peer over an abstract-namespace Unix
   socket (SCM_RIGHTS), and imports and maps the peers' descriptors with
   ``moe_symm_import``,
4. publishes the table of W base addresses to the device.

The region holds the per-parity count matrix, arrival flags, "free" epochs
and the compact receive rows (``moe_ep_layout``), and for the combine path a
return region that peers store expert outputs into.  Workspaces are cached by
(W, El, H, capacity, device, group) like the reference's cache key
(alltoall_persistent_gemm.py:161-163).
"""
from __future__ import annotations

import ctypes
import os
import secrets
import socket
import struct
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native as N


def _barrier(group) -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.barrier(group=group)


def _broadcast_token(group) -> str:
    """A random name shared by all ranks of the group (rank 0's choice)."""
    tok = [secrets.token_hex(8)]
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(tok, src=src, group=group)
    return tok[0]


def exchange_fds(fd: int, rank: int, world: int, tag: str, barrier) -> dict[int, int]:
    """Send `fd` to every peer and receive each peer's descriptor.

    Uses abstract-namespace Unix sockets named after `tag`; a connection
    queued on a listening socket accepts the message before the peer calls
    accept(), so the send loop cannot deadlock.  Returns {peer_rank: fd} with
    descriptors owned by the caller.
    """
    def name(r: int) -> bytes:
        return f"\0moe_ep_{tag}_{r}".encode()

    got: dict[int, int] = {}
    if world == 1:
        return got
    srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
    try:
        srv.bind(name(rank))
        srv.listen(max(world, 8))
        barrier()
        for peer in range(world):
            if peer == rank:
                continue
            c = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
            try:
                c.connect(name(peer))
                socket.send_fds(c, [struct.pack("<i", rank)], [fd])
            finally:
                c.close()
        srv.settimeout(120.0)
        for _ in range(world - 1):
            conn, _ = srv.accept()
            try:
                msg, fds, _, _ = socket.recv_fds(conn, 16, 1)
            finally:
                conn.close()
            if len(msg) < 4 or len(fds) != 1:
                raise RuntimeError("malformed descriptor message during workspace rendezvous")
            got[struct.unpack("<i", msg[:4])[0]] = fds[0]
    finally:
        srv.close()
    barrier()
    return got


@dataclass(frozen=True)
class WorkspaceKey:
    W: int
    El: int
    H: int
    cap_rows: int
    max_chunks: int
    push_rows: int
    device: int
    group: str
    ret_rows: int = 0  # return region (combine): rows of ret_cols bf16 outputs
    ret_cols: int = 0


# Largest epoch a launch may carry (the device word is 32 bits).
EPOCH_LIMIT = 2**32 - 1


class SymmetricWorkspace:
    """One rank's mapped view of all ranks' workspaces."""

    def __init__(self, key: WorkspaceKey, group, rank: int):
        L = N.lib()
        self.key = key
        self.group = group
        self.rank = rank
        self.world = key.W
        self.push_rows = key.push_rows
        self.layout = N.workspace_layout(key.W, key.El, key.H, 2, key.cap_rows, key.max_chunks, key.ret_rows,
                                         key.ret_cols)
        dev = key.device
        mapped = ctypes.c_size_t()
        base = ctypes.c_uint64()
        fd = ctypes.c_int()
        handle = ctypes.c_uint64()
        N.check(L.moe_symm_alloc(dev, self.layout.total_bytes, ctypes.byref(mapped), ctypes.byref(base),
                                 ctypes.byref(fd), ctypes.byref(handle)), "moe_symm_alloc")
        self.bytes = mapped.value
        self.base = base.value
        self._own = (base.value, mapped.value, handle.value)
        self._imports: list[tuple[int, int, int]] = []
        stream = torch.cuda.current_stream(dev)
        N.check(L.moe_ep_workspace_reset(self.base, ctypes.byref(self.layout), ctypes.c_void_p(stream.cuda_stream)),
                "moe_ep_workspace_reset")
        torch.cuda.synchronize(dev)
        # One rank has no peers: no rendezvous (and no collective on `group`,
        # so a rank may hold a private one-rank workspace for local work).
        try:
            if key.W > 1:
                tag = _broadcast_token(group)
                peer_fds = exchange_fds(fd.value, rank, key.W, tag, lambda: _barrier(group))
            else:
                peer_fds = {}
        finally:
            os.close(fd.value)
        bases = [0] * key.W
        bases[rank] = self.base
        try:
            for peer, pfd in sorted(peer_fds.items()):
                pbase = ctypes.c_uint64()
                ph = ctypes.c_uint64()
                try:
                    N.check(L.moe_symm_import(dev, pfd, self.bytes, ctypes.byref(pbase), ctypes.byref(ph)),
                            "moe_symm_import")
                finally:
                    os.close(pfd)
                bases[peer] = pbase.value
                self._imports.append((pbase.value, self.bytes, ph.value))
        except Exception:
            self.close()
            raise
        self.peer_bases = torch.tensor(bases, dtype=torch.int64, device=f"cuda:{dev}")
        # Mapped pinned word the kernels latch device-side errors into.
        self.status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.epoch = 0
        if key.W > 1:
            _barrier(group)  # every rank has zeroed and mapped before the first call

    def next_epoch(self) -> int:
        """The next call's epoch (1, 2, 3, ...).  The device compares epochs
        modulo 2**32 and treats the first two calls as having no earlier call
        to wait for, so the counter never wraps: after 2**32 - 1 calls the
        workspace restarts at 1 (``restart_epochs``, collective: every rank
        reaches it on the same call)."""
        if self.epoch >= EPOCH_LIMIT:
            self.restart_epochs()
        self.epoch += 1
        return self.epoch

    def restart_epochs(self) -> None:
        """Drain this device, zero the control words (counts, flags, epochs,
        counters) on every rank, and start the epochs again; the barriers
        keep any rank from launching before every rank has zeroed."""
        torch.cuda.synchronize(self.key.device)
        if self.world > 1:
            _barrier(self.group)
        self._reset_control()
        if self.world > 1:
            _barrier(self.group)
        self.epoch = 0

    def _reset_control(self) -> None:
        stream = torch.cuda.current_stream(self.key.device)
        N.check(N.lib().moe_ep_workspace_reset(self.base, ctypes.byref(self.layout),
                                               ctypes.c_void_p(stream.cuda_stream)), "moe_ep_workspace_reset")
        torch.cuda.synchronize(self.key.device)

    def host_status(self) -> int:
        return int(self.status_host[0]) & 0xFFFFFFFF

    def read_status(self) -> int:
        out = ctypes.c_uint32()
        N.check(N.lib().moe_ep_read_status(self.base, ctypes.byref(self.layout), ctypes.byref(out)),
                "moe_ep_read_status")
        return out.value

    def close(self) -> None:
        L = N.lib()
        for ptr, size, h in self._imports:
            L.moe_symm_free(ptr, size, h)
        self._imports = []
        if self._own is not None:
            L.moe_symm_free(*self._own)
            self._own = None


_CACHE: dict[WorkspaceKey, SymmetricWorkspace] = {}


def group_name(group) -> str:
    return getattr(group, "group_name", "WORLD") if group is not None else "WORLD"


def get_workspace(W: int, El: int, H: int, gm: int, device: int, group, rank: int,
                  push_rows: int, ret_cols: int = 0) -> SymmetricWorkspace:
    """Cached workspace large enough for padded slots of `gm` rows.

    The remote receive capacity is (W-1)*El*gm rows (every remote slot full),
    i.e. the reference's padded receive buffer without this rank's own slot.
    Capacity is rounded up to a power of two in gm so that calls whose gm
    differs slightly reuse one workspace; all ranks see the same gm (it is the
    all-reduced maximum), so all ranks make the same choice.  With
    ``ret_cols`` > 0 the workspace also holds a return region of W*El*gm_cap
    rows of ``ret_cols`` bf16 values (the combine path).
    """
    gm_cap = 1
    while gm_cap < max(gm, 1):
        gm_cap *= 2
    cap_rows = max(W - 1, 0) * El * gm_cap
    max_chunks = (gm_cap + push_rows - 1) // push_rows
    ret_rows = W * El * gm_cap if ret_cols > 0 else 0
    key = WorkspaceKey(W, El, H, cap_rows, max_chunks, push_rows, device, group_name(group), ret_rows,
                       ret_cols if ret_cols > 0 else 0)
    ws = _CACHE.get(key)
    if ws is None:
        ws = SymmetricWorkspace(key, group, rank)
        _CACHE[key] = ws
    return ws


def release_all() -> None:
    """Free every cached workspace (call on all ranks, with the device idle)."""
    for ws in list(_CACHE.values()):
        ws.close()
    _CACHE.clear()
