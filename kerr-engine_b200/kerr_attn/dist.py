"""Multi-GPU plumbing for the attention path: one process per GPU.

Every (batch, head) slab of causal attention is independent, so the path
shards by whole sequences with no exchange on the data path: rank r owns the
contiguous batch slice shard_batch(B, world, r).  The collectives are the
timing barrier, the max-over-ranks reduction of measured times, and the
data-parallel sum of the attention sublayer's parameter gradients
(ProjGradBuckets), NCCL over NVLink on GPUs and gloo on CPU.  The reference
has no multi-process code; its reduction is the host-side gradient sum over
the batch of src/train.rs:257-269, which the all-reduce extends over ranks.
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


class ProjGradBuckets:
    """Gradients of the attention projections, one flat bucket per block, all-
    reduced (sum) across the data-parallel ranks.

    Bucket i holds block i's c_attn weight [3C][C] and bias [3C], then c_proj's
    weight [C][C] and bias [C], then ln_1's weight [C] and bias [C]
    (4C^2 + 6C floats, the reference's attn_c_attn_w / _b, attn_c_proj_w / _b,
    ln_1_weight / _bias).  ``launch(i)`` starts block i's
    all-reduce as soon as its backward has been enqueued, so it overlaps the
    backward of the blocks below it; ``finish()`` waits for every bucket and
    divides by world * batch_per_rank: the reference sums per-sequence
    gradients over the batch and divides by batch_size (src/train.rs:257-269),
    and over ranks the batch is world * batch_per_rank sequences.
    """

    def __init__(self, n_blocks: int, n_embd: int, batch_per_rank: int, device=None):
        import torch

        self.C = n_embd
        self.n_blocks = n_blocks
        self.batch_per_rank = batch_per_rank
        self.numel = 4 * n_embd * n_embd + 6 * n_embd
        self.flat = torch.zeros(n_blocks, self.numel, device=device)
        self._work = []

    def views(self, i: int):
        """(c_attn_w [3C, C], c_attn_b [3C], c_proj_w [C, C], c_proj_b [C]) of block i."""
        C = self.C
        f = self.flat[i]
        a = 3 * C * C
        return (f[:a].view(3 * C, C), f[a:a + 3 * C], f[a + 3 * C:a + 3 * C + C * C].view(C, C),
                f[a + 3 * C + C * C:a + 4 * C + C * C])

    def ln_views(self, i: int):
        """(ln_1_w [C], ln_1_b [C]) of block i."""
        C = self.C
        e = 4 * C * C + 4 * C
        f = self.flat[i]
        return f[e:e + C], f[e + C:e + 2 * C]

    def zero_(self):
        self.flat.zero_()

    def launch(self, i: int):
        """Start block i's all-reduce (no-op without a process group of >1 ranks)."""
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            self._work.append(dist.all_reduce(self.flat[i], op=dist.ReduceOp.SUM, async_op=True))

    def finish(self) -> int:
        """Wait for every launched all-reduce, then scale to the batch mean.
        Returns the world size the gradients were reduced over."""
        import torch.distributed as dist

        for w in self._work:
            w.wait()
        self._work.clear()
        world = dist.get_world_size() if (dist.is_available() and dist.is_initialized()) else 1
        self.flat.mul_(1.0 / (world * self.batch_per_rank))
        return world
