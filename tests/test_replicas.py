"""Replica (data-parallel) host logic on CPU: two gloo ranks.

Sharding covers every unit once, the timing reduction is the maximum over
ranks on every rank, and rank 0 gathers the per-rank results back into unit
order, the way bench.py --gpus N and data-parallel sample runs use them.
"""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from dolittle_b200 import replicas


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n_units):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = replicas.shard(n_units, rank, world)
        results = [f"unit{u}" for u in mine]           # stand-in for one generation per unit
        t = replicas.max_over_ranks(dist, [1.0 + rank, 5.0 - rank])
        assert t == [float(world), 5.0], t
        per_rank = replicas.gather_to_rank0(dist, results)
        if rank == 0:
            merged = replicas.merge_shards(per_rank, n_units)
            assert merged == [f"unit{u}" for u in range(n_units)], merged
        else:
            assert per_rank is None
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_units", [16, 5, 1])
def test_two_gloo_ranks_shard_reduce_and_gather(n_units):
    mp.spawn(_rank_main, args=(2, _free_port(), n_units), nprocs=2, join=True)


def test_shard_covers_each_unit_once():
    for world in (1, 2, 3, 8):
        for n in (0, 1, 7, 16):
            got = sorted(u for r in range(world) for u in replicas.shard(n, r, world))
            assert got == list(range(n))
    with pytest.raises(ValueError):
        replicas.shard(4, 2, 2)


def test_single_process_paths_need_no_process_group():
    assert replicas.max_over_ranks(None, [1.0, 2.0]) == [1.0, 2.0]
    assert replicas.gather_to_rank0(None, ["a"]) == [["a"]]
