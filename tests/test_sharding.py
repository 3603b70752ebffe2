"""Host logic of request sharding, run as world-size-2 gloo ranks on CPU."""

from __future__ import annotations

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from copy_on_write_sdm_b200.sharding import least_loaded, reduce_over_ranks, shard_requests


def test_shards_cover_every_request_once():
    for total in (0, 1, 7, 64, 1024, 1023):
        for world in (1, 2, 3, 4, 8):
            owned = [r for rank in range(world) for r in shard_requests(total, world, rank)]
            assert owned == list(range(total))
            sizes = [len(shard_requests(total, world, rank)) for rank in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_requests(4, 2, 2)


def test_least_loaded():
    assert least_loaded([3, 1, 1, 5]) == 1
    assert least_loaded([0]) == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = shard_requests(64 * world, world, rank)
        # each rank "times" its own shard; the job time is the slowest rank
        slowest, tokens = reduce_over_ranks([1.0 + rank, float(len(mine))], op="max")
        total_tokens = reduce_over_ranks([float(len(mine))], op="sum")[0]
        results[rank] = (slowest, tokens, total_tokens, mine.start, mine.stop)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_max_and_sum():
    world = 2
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_rank_main, args=(world, _free_port(), results), nprocs=world, join=True)
        res = dict(results)
    assert res[0][0] == res[1][0] == 2.0  # max over ranks
    assert res[0][2] == res[1][2] == 128.0  # sum over ranks
    assert (res[0][3], res[0][4], res[1][3], res[1][4]) == (0, 64, 64, 128)
