"""Data-parallel plumbing of the batched hot path (one process per GPU).

Batch items and channels of the scans and the convolution are independent,
so each rank runs its own batch with no collective on the data path.  The
only exchange is the sum over ranks of the parameter-shaped gradients
(dA of the scans; dkernel/dbias of the convolution), as data-parallel
training needs.  Timing is the maximum over ranks.  torch.distributed is
the transport (NCCL on GPUs, gloo for the CPU tests).
"""
from __future__ import annotations

import os
from datetime import timedelta


def env_rank():
    """(rank, world) from the torchrun environment (1 process: (0, 1))."""
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))


def init(backend: str, timeout_s: float = 120.0, device_id=None):
    """Initialises the default process group from the environment with a
    short timeout, so ranks waiting on a failed peer end with an error."""
    import torch.distributed as dist
    kw = {"timeout": timedelta(seconds=timeout_s)}
    if device_id is not None:
        kw["device_id"] = device_id
    dist.init_process_group(backend, **kw)
    return dist


def shard_seed(base: int, rank: int) -> int:
    """Seed of a rank's synthetic shard (distinct per rank)."""
    return base + rank


def sum_grads(tensors, world: int):
    """In-place sum over ranks of parameter-shaped gradients."""
    if world <= 1:
        return tensors
    import torch.distributed as dist
    for t in tensors:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return tensors


def max_over_ranks(value: float, world: int, device=None) -> float:
    """Maximum of a per-rank scalar (elapsed times) over ranks."""
    if world <= 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def weak_scaling_rate(bytes_per_rank_step: float, world: int, steps: int,
                      elapsed_max_s: float) -> float:
    """Whole-job GB/s: every rank processes its own full batch per step."""
    return bytes_per_rank_step * world * steps / elapsed_max_s / 1e9
