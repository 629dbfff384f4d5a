"""Host-side logic of the multi-GPU (batch-sharded) path, run as
world_size-2 gloo process groups on CPU: the shards tile the batch exactly
once, and the timing reduction takes the slowest rank (max over ranks)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from thunderfft_b200.shard import conv2d_image_shard, shard_range, weak_scaling_value


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, align, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start, count = shard_range(batch, world, rank, align)
        mine = torch.zeros(batch, dtype=torch.int32)
        mine[start:start + count] = 1
        dist.all_reduce(mine)                         # coverage count per item
        ms = torch.tensor([10.0 + 5.0 * rank], dtype=torch.float64)  # per-rank device time
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        if rank == 0:
            q.put((mine.tolist(), float(ms.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch,align", [(65536, 4), (1001, 4), (3, 1), (0, 8)])
def test_shards_cover_batch_once_and_time_is_max_over_ranks(batch, align):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, align, q)) for r in range(world)]
    for p in procs:
        p.start()
    cover, ms = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(c == 1 for c in cover)
    assert ms == 15.0
    assert abs(weak_scaling_value(1e9, ms, world) - 2 * 1e9 / 0.015 / 1e9) < 1e-9


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_range_properties(world):
    for batch in (0, 1, 7, 64, 1000, 65536):
        for align in (1, 4, 32):
            pieces = [shard_range(batch, world, r, align) for r in range(world)]
            pos = 0
            for start, count in pieces:
                assert start == pos and count >= 0
                pos += count
                if start < batch and start + count < batch:
                    assert start % align == 0 and (start + count) % align == 0
            assert pos == batch


def _conv2d_worker(rank, world, port, images, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b0, nb = conv2d_image_shard(images, world, rank, "strong")
        mine = torch.zeros(images, dtype=torch.int32)
        mine[b0:b0 + nb] = 1
        dist.all_reduce(mine)
        starts = torch.zeros(world, dtype=torch.int64)
        starts[rank] = b0
        dist.all_reduce(starts)
        w0, wn = conv2d_image_shard(images, world, rank, "weak")
        if rank == 0:
            q.put((mine.tolist(), starts.tolist(), (w0, wn)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("images", [64, 7, 2])
def test_conv2d_pairs_split_across_ranks(images):
    """The 2-D convolution's multi-GPU split (bench.py --workload conv2d): as
    world-size-2 gloo ranks, strong scaling covers every batch image exactly
    once and starts each rank's slice on an even image (whole image pairs);
    weak scaling gives a rank the whole batch."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_conv2d_worker, args=(r, world, port, images, q)) for r in range(world)]
    for p in procs:
        p.start()
    cover, starts, weak = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(c == 1 for c in cover)
    assert all(b % 2 == 0 for b in starts)
    assert weak == (0, images)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_conv2d_image_shard_properties(world):
    for images in (1, 2, 7, 64, 2048):
        pieces = [conv2d_image_shard(images, world, r) for r in range(world)]
        pos = 0
        for b0, nb in pieces:
            assert b0 == pos and nb >= 0
            assert b0 % 2 == 0 or b0 == images
            assert nb % 2 == 0 or b0 + nb == images
            pos += nb
        assert pos == images
    with pytest.raises(ValueError):
        conv2d_image_shard(64, 2, 0, "diagonal")
