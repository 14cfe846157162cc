"""Process-group runtime: one process per GPU, NCCL for the plumbing (gloo on CPU).

Parity: train/h3/lightx2v_train/runtime/distributed.py:11-69 (init with timeout, barrier,
reduce_mean) and train/wan/imaginaire/utils/distributed.py:50-88.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def is_distributed() -> bool:
    return dist.is_available() and dist.is_initialized()


def get_rank() -> int:
    return dist.get_rank() if is_distributed() else 0


def get_world_size(group=None) -> int:
    return dist.get_world_size(group) if is_distributed() else 1


def init_distributed(backend: str | None = None, timeout_s: float = 600.0) -> tuple[int, int, torch.device]:
    """Initialise from torchrun's env (RANK / WORLD_SIZE / LOCAL_RANK / MASTER_*).

    Without those variables this is a single-process run.  Returns (rank, world, device)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cuda = torch.cuda.is_available()
    device = torch.device("cuda", local) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(device)
    if world > 1 and not is_distributed():
        backend = backend or ("nccl" if cuda else "gloo")
        kw = {"device_id": device} if (cuda and backend == "nccl") else {}
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return get_rank(), get_world_size(), device


def barrier():
    if is_distributed():
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def reduce_mean(t: torch.Tensor) -> torch.Tensor:
    if not is_distributed():
        return t
    t = t.clone()
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t / get_world_size()


def max_over_ranks(x: float, device=None) -> float:
    if not is_distributed():
        return float(x)
    dev = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu")
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


@torch.no_grad()
def broadcast_module(module: torch.nn.Module, src: int = 0, group=None):
    """Make every rank hold rank ``src``'s parameters and buffers (random init differs per rank)."""
    if not is_distributed():
        return
    for t in list(module.parameters()) + list(module.buffers()):
        dist.broadcast(t.data, src=src, group=group)
