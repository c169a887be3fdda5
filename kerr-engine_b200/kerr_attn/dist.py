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
    """Gradients of the attention sublayer's parameters, one flat buffer per
    block in two all-reduce segments, summed across the data-parallel ranks.

    Block i's buffer holds c_proj's weight [C][C] and bias [C] first (the
    "proj" segment), then c_attn's weight [3C][C] and bias [3C] and ln_1's
    weight [C] and bias [C] (the "rest" segment): 4C^2 + 6C floats, the
    reference's attn_c_proj_w / _b, attn_c_attn_w / _b, ln_1_weight / _bias.
    The backward of a block produces c_proj's gradients first, so
    ``launch_proj(i)`` starts that segment's all-reduce as soon as c_proj's
    dW is enqueued and ``launch(i)`` the rest once the block's backward is;
    both overlap the backward still to come.  ``finish()`` waits for every
    segment and divides by world * batch_per_rank: the reference sums
    per-sequence gradients over the batch and divides by batch_size
    (src/train.rs:257-269), and over ranks the batch is world *
    batch_per_rank sequences.
    """

    def __init__(self, n_blocks: int, n_embd: int, batch_per_rank: int, device=None):
        import torch

        self.C = n_embd
        self.n_blocks = n_blocks
        self.batch_per_rank = batch_per_rank
        self.numel = 4 * n_embd * n_embd + 6 * n_embd
        self.proj_numel = n_embd * n_embd + n_embd
        self.flat = torch.zeros(n_blocks, self.numel, device=device)
        self._work = []
        self._proj_sent = set()

    def views(self, i: int):
        """(c_attn_w [3C, C], c_attn_b [3C], c_proj_w [C, C], c_proj_b [C]) of block i."""
        C = self.C
        f = self.flat[i]
        p = C * C
        a = p + C
        return (f[a:a + 3 * C * C].view(3 * C, C), f[a + 3 * C * C:a + 3 * C * C + 3 * C], f[:p].view(C, C),
                f[p:p + C])

    def ln_views(self, i: int):
        """(ln_1_w [C], ln_1_b [C]) of block i."""
        C = self.C
        e = 4 * C * C + 4 * C
        f = self.flat[i]
        return f[e:e + C], f[e + C:e + 2 * C]

    def zero_(self):
        self.flat.zero_()

    @staticmethod
    def _group():
        import torch.distributed as dist

        return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1

    def launch_proj(self, i: int):
        """Start the all-reduce of block i's c_proj segment (no-op without a
        process group of more than one rank)."""
        import torch.distributed as dist

        if self._group():
            self._work.append(dist.all_reduce(self.flat[i, :self.proj_numel], op=dist.ReduceOp.SUM, async_op=True))
        self._proj_sent.add(i)

    def launch(self, i: int):
        """Start the all-reduce of the rest of block i's buffer (all of it if
        launch_proj(i) was not called)."""
        import torch.distributed as dist

        start = self.proj_numel if i in self._proj_sent else 0
        self._proj_sent.discard(i)
        if self._group():
            self._work.append(dist.all_reduce(self.flat[i, start:], op=dist.ReduceOp.SUM, async_op=True))

    def finish(self) -> int:
        """Wait for every launched all-reduce, then scale to the batch mean.
        Returns the world size the gradients were reduced over."""
        import torch.distributed as dist

        for w in self._work:
            w.wait()
        self._work.clear()
        self._proj_sent.clear()
        world = dist.get_world_size() if (dist.is_available() and dist.is_initialized()) else 1
        self.flat.mul_(1.0 / (world * self.batch_per_rank))
        return world
