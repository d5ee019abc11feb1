"""Multi-rank timing logic of bench.py on CPU (gloo, world size 2).

The data path has no collective (images are sharded by rank); the only
cross-rank steps are the barrier around the timed region and the max over
ranks of the elapsed time.  This checks that logic with two gloo ranks.
"""
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import time

    dist.barrier()
    t0 = time.perf_counter()
    time.sleep(0.05 * (rank + 1))  # rank 1 is the slow one
    t = time.perf_counter() - t0
    dist.barrier()
    tt = torch.tensor([t])
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    # weak scaling: every rank processes its own shard of images
    images = torch.tensor([8])
    dist.all_reduce(images)
    q.put((rank, float(tt.item()), int(images.item())))
    dist.destroy_process_group()


def test_two_rank_max_timing_and_weak_scaling():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert res[0][1] == res[1][1] >= 0.1  # both ranks report the slowest rank's time
    assert res[0][2] == 16


def _shard_worker(rank, world, port, global_batch, q):
    """One rank of a gloo job: takes its shard of the global batch exactly as bench.py does and
    gathers the image indices of every rank."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench

    start, count = bench.shard_range(global_batch, world, rank)
    idx = torch.full((global_batch,), -1, dtype=torch.int64)
    idx[:count] = torch.arange(start, start + count)
    gathered = [torch.empty_like(idx) for _ in range(world)]
    dist.all_gather(gathered, idx)
    total = torch.tensor([count])
    dist.all_reduce(total)
    if rank == 0:
        q.put(([int(v) for g in gathered for v in g if v >= 0], int(total.item())))
    dist.destroy_process_group()


def test_two_rank_shards_cover_the_batch_once():
    """BASELINE config 5 splits a global batch of 512 by image over the ranks: with two gloo ranks
    (and an odd batch) the shards bench.py takes cover every image exactly once."""
    ctx = mp.get_context("spawn")
    for gb in (512, 7):
        q = ctx.Queue()
        port = 30500 + (os.getpid() % 1000) + gb % 10
        procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, gb, q)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        images, total = q.get(timeout=10)
        assert sorted(images) == list(range(gb)) and total == gb


def test_shard_ranges_for_every_world_size():
    import bench

    for gb in (512, 513, 1, 8):
        for world in (1, 2, 4, 8):
            seen = []
            for r in range(world):
                start, count = bench.shard_range(gb, world, r)
                seen.extend(range(start, start + count))
            assert seen == list(range(gb)), (gb, world)
