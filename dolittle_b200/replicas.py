"""Data-parallel replicas: one engine per GPU, no data-path collective.

Batch-1 generation does not shard, and the independent units of the larger
workloads — steered and unsteered branches, independent interpretation
samples — split across GPUs.  Every rank holds a full engine and processes
its share of the units. The only cross-rank traffic is control: the timing
maximum (the job takes as long as its slowest rank) and gathering results on
rank 0.  The process group is whatever torch.distributed was initialised
with: NCCL on GPUs, gloo in the CPU tests.
"""
from __future__ import annotations


def shard(n_units: int, rank: int, world: int) -> list:
    """Round-robin share of units 0..n_units-1 for `rank` (every unit once)."""
    if world < 1 or not 0 <= rank < world or n_units < 0:
        raise ValueError("bad shard arguments")
    return list(range(rank, n_units, world))


def max_over_ranks(dist, values: list) -> list:
    """Element-wise maximum of per-rank floats (device timings) on every rank."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return list(values)
    import torch
    backend = dist.get_backend()
    device = "cuda" if backend == "nccl" else "cpu"
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def gather_to_rank0(dist, local):
    """Per-rank results as a list ordered by rank on rank 0 (None elsewhere)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return [local]
    out = [None] * dist.get_world_size() if dist.get_rank() == 0 else None
    dist.gather_object(local, out, dst=0)
    return out


def merge_shards(per_rank: list, n_units: int) -> list:
    """Undo shard(): results of units 0..n_units-1 in unit order."""
    world = len(per_rank)
    merged = [None] * n_units
    for r, items in enumerate(per_rank):
        for unit, item in zip(shard(n_units, r, world), items):
            merged[unit] = item
    return merged
