"""Process-group bootstrap (``primus_dlrm/distributed/setup.py:13-64``).

One process per GPU (torchrun env: RANK, LOCAL_RANK, WORLD_SIZE, MASTER_*).
NCCL on CUDA, gloo on CPU.  The timeout is short by default (the reference
uses 30 min) so a rank that dies surfaces as an error on the others instead
of a hang.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def init_distributed(backend: str | None = None, timeout_s: float = 300.0) -> None:
    """Initialise the default process group from torchrun's environment.
    A single-process run (WORLD_SIZE unset or 1) creates no group."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1 or dist.is_initialized():
        if torch.cuda.is_available():
            torch.cuda.set_device(get_local_rank())
        return
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if backend == "nccl":
        torch.cuda.set_device(get_local_rank())
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", get_local_rank()))
    else:
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))


def get_rank() -> int:
    return dist.get_rank() if dist.is_initialized() else int(os.environ.get("RANK", "0"))


def get_world_size() -> int:
    return dist.get_world_size() if dist.is_initialized() else int(os.environ.get("WORLD_SIZE", "1"))


def get_local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", "0"))


def is_main_process() -> bool:
    return get_rank() == 0


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()


def cleanup() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()
