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


def _ledger_worker(rank, world, port, q, failing):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    from realm_b200.sharding import RankFailure, StepLedger
    led = StepLedger.from_default_group("t")
    out = []
    for step in range(1, 4):
        if rank == failing == 1 and step == 2:
            led.leave("worker raised during step 2")   # leaves between steps
            q.put((rank, "left"))
            return                                    # no destroy: the process just exits
        if rank == failing == 2 and step == 2:
            os._exit(0)                               # dies without a word
        led.done(step)
        try:
            led.wait_peers(step, timeout_s=3.0)
            out.append(step)
        except RankFailure as e:
            q.put((rank, ("failure", e.ranks, e.step, str(e))))
            return
    q.put((rank, ("ok", out)))
    dist.destroy_process_group()


@pytest.mark.parametrize("world,failing", [(2, 1), (3, 2)])
def test_rank_loss_detected_between_steps(world, failing):
    """A rank that leaves (or vanishes) between steps: the survivors learn of it
    on the host, within the ledger's timeout, before their next launch."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() + 37 * world) % 400
    procs = [ctx.Process(target=_ledger_worker, args=(r, world, port, q, failing)) for r in range(world)]
    for p in procs:
        p.start()
    n_msgs = world if failing == 1 else world - 1  # a vanished rank sends nothing
    res = dict(q.get(timeout=120) for _ in range(n_msgs))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        if r == failing:
            continue
        kind, ranks, step, msg = res[r]
        assert kind == "failure" and ranks == [failing] and step == 2, res[r]
        assert ("raised" in msg) if failing == 1 else ("no heartbeat" in msg)


def test_tenant_shard_64_over_ranks():
    """configs[3] at N = 2 / 4 / 8: 64 tenants split 32 / 16 / 8 per rank by LPT on
    context length, every tenant placed once."""
    from realm_b200.sharding import lpt_shard
    import numpy as np
    lens = np.random.default_rng(4).integers(128, 513, 64).tolist()
    for world in (2, 4, 8):
        bins = lpt_shard(lens, world, equal_counts=True)
        assert sorted(sum(bins, [])) == list(range(64))
        assert all(len(b) == 64 // world for b in bins)
        loads = [sum(lens[t] for t in b) for b in bins]
        assert max(loads) - min(loads) <= max(lens)
