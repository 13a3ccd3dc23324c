"""Multi-GPU plumbing for the MoE path: one process per GPU over
torch.distributed (NCCL on GPUs, gloo for CPU tests).

The decode/prefill MoE layer shards by tokens: each rank owns a replica of
the layer weights (a C2 layer is 0.86 GB; 40 layers fit one B200's HBM) and
processes its own token batch, so the timed path has no collective. Timing is
taken on the device per rank and reduced with MAX over ranks.
"""
from __future__ import annotations

import os


def env_rank():
    """(rank, local_rank, world_size) from torchrun's environment (1-process defaults)."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def init(backend: str | None = None):
    """Initialises the default process group when WORLD_SIZE > 1; returns (rank, local_rank, world)."""
    import torch
    import torch.distributed as dist

    rank, local, world = env_rank()
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29511")
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group(backend, device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend)
    return rank, local, world


def shard_range(n: int, rank: int, world: int):
    """Contiguous [lo, hi) share of n units for `rank` (sizes differ by at most one)."""
    base, rem = divmod(n, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


def max_over_ranks(value: float, device=None) -> float:
    """MAX of a per-rank float over the process group (identity without one)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(device=None):
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        if device is not None and dist.get_backend() == "nccl":
            dist.barrier(device_ids=[device])
        else:
            dist.barrier()
