"""Multi-rank host logic on CPU with the gloo backend (world size 2): rollout sharding by
whole GRPO groups and the max-over-ranks timing used by bench.py."""

import os
import socket

import pytest
import torch.multiprocessing as mp

from kvstreams.distributed import shard_groups


def test_shards_cover_all_rollouts_once_with_whole_groups():
    for n_groups, g, world in [(64, 8, 8), (64, 8, 3), (5, 4, 8), (1, 8, 2)]:
        n = n_groups * g
        owned = [list(shard_groups(n, g, world, r)) for r in range(world)]
        flat = [i for o in owned for i in o]
        assert sorted(flat) == list(range(n))
        for o in owned:
            assert len(o) % g == 0 and (not o or o[0] % g == 0)
        sizes = [len(o) // g for o in owned]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_groups(10, 4, 2, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    from kvstreams.distributed import reduce_max, reduce_sum, shard_groups

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        mine = shard_groups(512, 8, world, rank)
        # per-rank "elapsed ms" differs; every rank must see the same maximum
        slowest = reduce_max(10.0 + rank)
        total = reduce_sum(len(mine))
        results[rank] = (mine.start, mine.stop, slowest, total)
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_reduce_and_shard():
    world = 2
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, port, results), nprocs=world, join=True, start_method="spawn")
    assert results[0][:2] == (0, 256) and results[1][:2] == (256, 512)
    assert results[0][2] == results[1][2] == 11.0
    assert results[0][3] == results[1][3] == 512
