"""Host-side multi-process logic on CPU (gloo ranks): the descriptor
exchange used to map peer workspaces, and the count all-to-all layout."""
import os
import traceback

import numpy as np
import pytest

from conftest import free_port


def _fd_worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        from nvshmem_testing_b200 import symm

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        fd = os.memfd_create(f"r{rank}")
        os.write(fd, f"payload-from-rank-{rank}".encode())
        tag = symm._broadcast_token(None)
        got = symm.exchange_fds(fd, rank, world, tag, lambda: symm._barrier(None))
        seen = {}
        for peer, pfd in got.items():
            os.lseek(pfd, 0, os.SEEK_SET)
            seen[peer] = os.read(pfd, 64).decode()
            os.close(pfd)
        os.close(fd)
        dist.destroy_process_group()
        q.put((rank, "ok", seen))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def _counts_worker(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        import oracle
        from nvshmem_testing_b200 import workloads

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        wl = workloads.get("skewed_zipf", T=512, E=8)
        allc = [oracle.bucketize(workloads.top_idxs(wl, r).numpy(), wl.E)[0] for r in range(world)]
        sent = torch.from_numpy(allc[rank]).view(world, -1).contiguous()
        recv = torch.empty_like(sent)
        dist.all_to_all_single(recv, sent)  # benchmark.py:114-118
        ok = np.array_equal(recv.numpy(), oracle.recv_counts_matrix(allc, rank, world))
        # gm: all-reduced MAX (the oracle's fix of utils.py:45-49)
        m = torch.tensor([oracle.local_max(allc[rank])])
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ok = ok and int(m) == max(oracle.local_max(c) for c in allc)
        dist.destroy_process_group()
        q.put((rank, "ok", ok))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def _bound_worker(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        from nvshmem_testing_b200 import alltoall_persistent_gemm as apg

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        rc = torch.tensor([[3, 0], [7, 1]]) if rank == 0 else torch.tensor([[2, 9], [0, 4]])
        rows, bound = apg._general_bound(rc, None)
        zeros = apg._general_bound(torch.zeros(2, 2, dtype=torch.int32), None)
        dist.destroy_process_group()
        q.put((rank, "ok", (rows, bound, zeros)))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def _epoch_worker(rank, world, port, q):
    """A workspace whose epoch counter reaches the 32-bit limit restarts at 1
    on every rank on the same call, zeroing its control words in between."""
    try:
        import types
        import torch.distributed as dist
        from nvshmem_testing_b200 import symm

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        symm.torch.cuda.synchronize = lambda *a, **k: None  # no device here
        ws = object.__new__(symm.SymmetricWorkspace)
        ws.key = types.SimpleNamespace(device=0)
        ws.world, ws.group, ws.epoch = world, None, symm.EPOCH_LIMIT - 2
        resets = []
        ws._reset_control = lambda: resets.append(ws.epoch)
        seq = [ws.next_epoch() for _ in range(4)]
        dist.destroy_process_group()
        q.put((rank, "ok", (seq, resets)))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def _run(target, world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, kind, payload = q.get(timeout=180)
        res[r] = (kind, payload)
    for p in procs:
        p.join(timeout=60)
    return res


@pytest.mark.parametrize("world", [2, 3])
def test_fd_exchange_over_unix_sockets(world):
    res = _run(_fd_worker, world)
    for r, (kind, payload) in res.items():
        assert kind == "ok", payload
        assert payload == {p: f"payload-from-rank-{p}" for p in range(world) if p != r}


def test_count_exchange_matches_oracle():
    res = _run(_counts_worker, 2)
    for r, (kind, payload) in res.items():
        assert kind == "ok", payload
        assert payload is True


def test_general_bound_is_all_reduced():
    """The unpadded exchange sizes its buffers by the largest count over the
    group (all-reduced MAX) and its output by this rank's own rows."""
    res = _run(_bound_worker, 2)
    for r, (kind, payload) in res.items():
        assert kind == "ok", payload
        rows, bound, zeros = payload
        assert rows == (11 if r == 0 else 15)
        assert bound == 9
        assert zeros == (0, 1)  # empty counts: bound at least 1


def test_epochs_restart_before_the_32_bit_limit():
    res = _run(_epoch_worker, 2)
    for r, (kind, payload) in res.items():
        assert kind == "ok", payload
        seq, resets = payload
        assert seq == [2**32 - 2, 2**32 - 1, 1, 2]
        assert resets == [2**32 - 1]
