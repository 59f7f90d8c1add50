"""World-size-2 gloo test of the multi-GPU host logic (CPU only): each rank
owns a disjoint tenant block, there is no data-path collective, and the
benchmark's timing is the max over ranks."""
import os

import pytest


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from realm_b200.sharding import max_over_ranks, tenant_shard
    mine = tenant_shard(8 * world, world, rank)
    t = max_over_ranks([10.0 * (rank + 1), 1.0 - rank])
    dist.barrier()
    q.put((rank, mine, t))
    dist.destroy_process_group()


def test_two_rank_shard_and_max():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0][1] == list(range(0, 8)) and out[1][1] == list(range(8, 16))
    assert out[0][2] == out[1][2] == [20.0, 1.0]
