"""Host-side multi-rank logic on CPU: world-size-2 gloo process groups."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kerr_attn.dist import max_over_ranks, shard_batch, sync


@pytest.mark.parametrize("batch,world", [(16, 1), (16, 2), (8, 8), (10, 4), (3, 4), (0, 2)])
def test_shard_batch_partitions(batch, world):
    shards = [shard_batch(batch, world, r) for r in range(world)]
    assert shards[0][0] == 0 and shards[-1][1] == batch
    for (a0, a1), (b0, b1) in zip(shards, shards[1:]):
        assert a1 == b0
    sizes = [b1 - b0 for b0, b1 in shards]
    assert max(sizes) - min(sizes) <= 1


def test_shard_batch_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_batch(4, 2, 2)
    with pytest.raises(ValueError):
        shard_batch(-1, 2, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sync()  # barrier on CPU
        m = max_over_ranks(1.5 + rank)
        b0, b1 = shard_batch(16, world, rank)
        got = torch.tensor([b0, b1], dtype=torch.int64)
        gathered = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(gathered, got)
        out[rank] = (m, [tuple(g.tolist()) for g in gathered])
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_shards_with_gloo():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    for rank in range(world):
        m, shards = out[rank]
        assert m == 1.5 + world - 1
        assert shards == [(0, 8), (8, 16)]


def test_max_over_ranks_without_group_is_identity():
    assert max_over_ranks(3.25) == 3.25
