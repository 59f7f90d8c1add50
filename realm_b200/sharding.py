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


def lpt_shard(ctx_lens: Sequence[int], world: int) -> List[List[int]]:
    """Longest-processing-time placement by context length (KV bytes per step)."""
    bins = [[] for _ in range(world)]
    load = [0] * world
    for t in sorted(range(len(ctx_lens)), key=lambda i: -ctx_lens[i]):
        r = min(range(world), key=lambda i: (load[i], i))
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
