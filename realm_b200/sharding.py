"""Tenant placement and timing reduction for one-process-per-GPU runs.

Tenants are independent (each owns its paged KV cache and only shares the
read-only weights), so a multi-GPU deployment replicates the weights per GPU
and partitions tenants across ranks; the decode path has no collective. The
only cross-rank operations are the benchmark barrier and the max-over-ranks
reduction of measured times, done through torch.distributed (NCCL on GPUs,
gloo in the CPU tests).
"""
from __future__ import annotations

from typing import List, Sequence


def tenant_shard(n_total: int, world: int, rank: int) -> List[int]:
    """Global tenant ids owned by `rank`: a balanced contiguous block."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(n_total, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


def lpt_shard(ctx_lens: Sequence[int], world: int, equal_counts: bool = False) -> List[List[int]]:
    """Longest-processing-time placement by context length (KV bytes per step).

    With equal_counts every rank gets the same number of tenants (the last
    ranks one fewer when it does not divide), so every rank runs a decode
    batch of the same row count."""
    bins = [[] for _ in range(world)]
    load = [0] * world
    cap = [len(ctx_lens) // world + (1 if r < len(ctx_lens) % world else 0) for r in range(world)]
    for t in sorted(range(len(ctx_lens)), key=lambda i: -ctx_lens[i]):
        open_ranks = [i for i in range(world) if not equal_counts or len(bins[i]) < cap[i]]
        r = min(open_ranks, key=lambda i: (load[i], i))
        bins[r].append(t)
        load[r] += ctx_lens[t]
    return [sorted(b) for b in bins]


def max_over_ranks(values: Sequence[float], device=None) -> List[float]:
    """Element-wise max of per-rank measurements (identity when not distributed)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(values)
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


class RankFailure(RuntimeError):
    """A peer rank stopped (or reported a failure) between steps."""

    def __init__(self, ranks, step, why):
        super().__init__(f"rank(s) {sorted(ranks)} did not reach step {step}: {why}")
        self.ranks, self.step = sorted(ranks), step


class StepLedger:
    """Host-side liveness between steps over the process group's key-value store.

    Every rank records the step it has finished (`done(step)`) or that it is
    leaving (`leave(why)`) before it starts another launch. `wait_peers(step,
    timeout_s)` returns once every rank has recorded `step`, and raises
    RankFailure naming the ranks that left or did not arrive in time, so the
    survivors learn of a lost peer on the host instead of inside a collective.
    A rank only ever leaves between steps, with none of its kernels in flight.
    """

    def __init__(self, store, rank: int, world: int, prefix: str = "rb_step"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix
        self.last = 0

    @classmethod
    def from_default_group(cls, prefix: str = "rb_step") -> "StepLedger":
        import torch.distributed as dist
        from torch.distributed import distributed_c10d as c10d
        return cls(c10d._get_default_store(), dist.get_rank(), dist.get_world_size(), prefix)

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def done(self, step: int) -> None:
        self.last = step
        self.store.set(self._key(self.rank), str(step))

    def leave(self, why: str = "left") -> None:
        # keeps the last finished step: peers still waiting for it see it done
        self.store.set(self._key(self.rank), f"x:{self.last}:" + why.replace("\n", " ")[:200])

    def wait_peers(self, step: int, timeout_s: float = 10.0, poll_s: float = 0.01) -> None:
        import time
        deadline = time.monotonic() + timeout_s
        pending = set(range(self.world))
        left = {}
        while True:
            for r in sorted(pending):
                if self.store.check([self._key(r)]):
                    v = self.store.get(self._key(r)).decode()
                    if v.startswith("x:"):
                        last, why = v[2:].split(":", 1)
                        if int(last) < step:
                            left[r] = why
                        pending.discard(r)
                    elif int(v) >= step:
                        pending.discard(r)
            if left:
                raise RankFailure(left, step, "; ".join(f"rank {r}: {w}" for r, w in sorted(left.items())))
            if not pending:
                return
            if time.monotonic() > deadline:
                raise RankFailure(pending, step, f"no heartbeat within {timeout_s:.1f} s")
            time.sleep(poll_s)
