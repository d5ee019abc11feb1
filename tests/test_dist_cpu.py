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
