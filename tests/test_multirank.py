"""Host-side multi-rank logic on CPU: world-size-2 gloo process groups."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kerr_attn.dist import ProjGradBuckets, max_over_ranks, shard_batch, sync


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


def _bucket_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        C, blocks, batch = 8, 3, 4
        g = ProjGradBuckets(blocks, C, batch)
        for i in reversed(range(blocks)):  # the backward walks the blocks top-down
            aw, ab, pw, pb = g.views(i)
            pw.fill_(-1.0 * (rank + 1))
            pb.fill_(float(i))
            if i % 2 == 0:  # c_proj's segment sent first on even blocks, with the rest on odd ones
                g.launch_proj(i)
            aw.fill_(rank + 1.0 + i)
            ab.fill_(10.0 * (rank + 1))
            lw, lb = g.ln_views(i)
            lw.fill_(2.0 * (rank + 1))
            lb.fill_(-float(i) * (rank + 1))
            g.launch(i)
        out[rank] = (g.finish(), g.flat.clone())
    finally:
        dist.destroy_process_group()


def test_projection_gradient_allreduce_with_gloo():
    # Each block's bucket is summed over the ranks and scaled by
    # 1 / (world * batch): the batch mean over every rank's sequences.
    world, C, blocks, batch = 2, 8, 3, 4
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_bucket_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn",
                       join=True)
    scale = 1.0 / (world * batch)
    ref = ProjGradBuckets(blocks, C, batch)
    for i in range(blocks):
        aw, ab, pw, pb = ref.views(i)
        aw.fill_(sum(r + 1.0 + i for r in range(world)) * scale)
        ab.fill_(sum(10.0 * (r + 1) for r in range(world)) * scale)
        pw.fill_(sum(-1.0 * (r + 1) for r in range(world)) * scale)
        pb.fill_(world * float(i) * scale)
        lw, lb = ref.ln_views(i)
        lw.fill_(sum(2.0 * (r + 1) for r in range(world)) * scale)
        lb.fill_(sum(-float(i) * (r + 1) for r in range(world)) * scale)
    for rank in range(world):
        w, flat = out[rank]
        assert w == world
        assert torch.allclose(flat, ref.flat)
    assert ref.numel == 4 * C * C + 6 * C
    # The views tile each bucket exactly.
    aw, ab, pw, pb = ref.views(0)
    lw, lb = ref.ln_views(0)
    assert sum(t.numel() for t in (aw, ab, pw, pb, lw, lb)) == ref.numel


def test_projection_buckets_single_process():
    g = ProjGradBuckets(2, 4, 8)
    g.views(1)[0].fill_(8.0)
    g.launch(1)
    assert g.finish() == 1
    assert float(g.views(1)[0].max()) == 1.0 and float(g.views(0)[0].abs().max()) == 0.0
