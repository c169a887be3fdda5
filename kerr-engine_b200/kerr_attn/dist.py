"""Multi-GPU plumbing for the attention path: one process per GPU.

Every (batch, head) slab of causal attention is independent, so the path
shards by whole sequences with no exchange on the data path: rank r owns the
contiguous batch slice shard_batch(B, world, r).  The only collectives are the
timing barrier and the max-over-ranks reduction of measured times (NCCL over
NVLink on GPUs, gloo on CPU).  The reference has no multi-process code; its
only reduction is the host-side gradient sum of src/train.rs:257-269, which
belongs to the projection layers outside this path.
"""
from __future__ import annotations

import os


def world() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from the torchrun environment (1 process: 0, 0, 1)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def shard_batch(batch: int, world_size: int, rank: int) -> tuple[int, int]:
    """Contiguous [b0, b1) slice of `batch` sequences owned by `rank`; the
    first batch % world_size ranks take one extra sequence."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of {world_size}")
    if batch < 0:
        raise ValueError("batch must be >= 0")
    base, extra = divmod(batch, world_size)
    b0 = rank * base + min(rank, extra)
    return b0, b0 + base + (1 if rank < extra else 0)


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of `value` over all ranks (identity without a process group).
    `device` is the tensor device the backend needs (a CUDA device for NCCL)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sync(device=None) -> None:
    """Device synchronise, barrier, synchronise: bracket for timed regions."""
    import torch
    import torch.distributed as dist

    cuda = device is not None and torch.device(device).type == "cuda"
    if cuda:
        torch.cuda.synchronize(device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
    if cuda:
        torch.cuda.synchronize(device)
