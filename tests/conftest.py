import os
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA GPUs")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="session")
def single_rank_group():
    """A one-rank NCCL process group on cuda:0 (run() is collective and
    asserts an initialised group, like the reference)."""
    import torch
    import torch.distributed as dist

    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    torch.cuda.set_device(0)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1,
                                device_id=torch.device("cuda", 0))
    yield dist.group.WORLD
