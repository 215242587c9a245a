"""Process-group bootstrap for one-process-per-GPU jobs (torchrun env).

``init_distributed()`` reads ``RANK`` / ``WORLD_SIZE`` / ``LOCAL_RANK`` /
``MASTER_ADDR`` / ``MASTER_PORT`` (as set by ``torch.distributed.run``), binds
the process to ``cuda:LOCAL_RANK`` and creates the NCCL group (``gloo`` on
CPU) with a short timeout so a rank that dies makes the others fail fast
instead of waiting forever.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def env_world() -> tuple:
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def init_distributed(backend: str | None = None, timeout_s: float = 120.0) -> tuple:
    """Initialise the default group if the env describes more than one rank.

    Returns ``(rank, world_size, device)``.
    """
    rank, world, local = env_world()
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
    else:
        device = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        be = backend or ("nccl" if device.type == "cuda" else "gloo")
        kw = {"device_id": device} if be == "nccl" else {}
        dist.init_process_group(be, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world, device


def is_dist() -> bool:
    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


def barrier() -> None:
    if is_dist():
        dist.barrier()


def destroy() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
