"""Sharding of a cloud batch over ranks, with world-size-2 gloo process groups on the CPU."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gdl_b200.sharding import local_slice, shard_clouds


def test_shards_tile_the_batch():
    rng = np.random.default_rng(0)
    for world in (1, 2, 3, 4, 8):
        cost = rng.integers(1, 1000, 37).astype(float)
        spans = [shard_clouds(cost, world, r) for r in range(world)]
        covered = [b for c0, c1 in spans for b in range(c0, c1)]
        assert covered == list(range(37))
        loads = [cost[c0:c1].sum() for c0, c1 in spans]
        assert max(loads) <= cost.sum() / world + cost.max()
    assert shard_clouds([], 4, 2) == (0, 0)
    with pytest.raises(ValueError):
        shard_clouds([1.0], 2, 2)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import oracle as O

    rng = np.random.default_rng(5)
    sizes = rng.integers(50, 400, 9)
    ptr = np.concatenate([[0], np.cumsum(sizes)])
    pos = rng.random((int(ptr[-1]), 3), dtype=np.float32)
    k = np.minimum(sizes, 40)
    c0, c1 = shard_clouds(sizes * k, world, rank)
    off, lptr = local_slice(ptr, c0, c1)
    mine = O.fps(pos[off:off + int(lptr[-1])], lptr, k[c0:c1]) + off  # global indices restored
    parts = [None] * world
    dist.all_gather_object(parts, (c0, c1, mine.tolist()))
    if rank == 0:
        out.put(parts)
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_fps_equals_whole_batch_gloo():
    from oracle import oracle as O

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    parts = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(5)
    sizes = rng.integers(50, 400, 9)
    ptr = np.concatenate([[0], np.cumsum(sizes)])
    pos = rng.random((int(ptr[-1]), 3), dtype=np.float32)
    whole = O.fps(pos, ptr, np.minimum(sizes, 40))
    assert [b for c0, c1, _ in parts for b in range(c0, c1)] == list(range(9))
    assert np.array_equal(np.concatenate([np.array(m, np.int64) for _, _, m in parts]), whole)
