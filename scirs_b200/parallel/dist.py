"""Process-group plumbing: one process per GPU, torch.distributed for
bootstrap (NCCL on GPUs, gloo for CPU ranks), short timeouts so that ranks
waiting on a dead peer fail instead of hanging.

Reference parity: replaces the in-process stand-ins of the reference
(scirs2-core/src/distributed/collective.rs:72-157 threads + Barrier,
scirs2-autograd/src/distributed/mod.rs:13-84 local averaging) with real
multi-process groups.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def env_rank_world() -> tuple[int, int, int]:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def init(backend: str | None = None, timeout_s: float = 120.0) -> tuple[int, int, int]:
    """Initialise the default process group from the torchrun environment.

    Returns (rank, world_size, local_rank). With WORLD_SIZE=1 nothing is
    initialised. The CUDA device is set to LOCAL_RANK when GPUs exist.
    """
    rank, world, local = env_rank_world()
    use_cuda = torch.cuda.is_available() and backend != "gloo"
    if use_cuda:
        torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29511")
        backend = backend or ("nccl" if use_cuda else "gloo")
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(
            backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s), **kw
        )
    return rank, world, local


def is_dist() -> bool:
    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


def rank() -> int:
    return dist.get_rank() if is_dist() else 0


def world_size() -> int:
    return dist.get_world_size() if is_dist() else 1


def barrier():
    if is_dist():
        dist.barrier()


def max_over_ranks(x: float) -> float:
    """Max of a host scalar over ranks (device-timed numbers use this)."""
    if not is_dist():
        return x
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shutdown():
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
