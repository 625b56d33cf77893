"""Request sharding and the post-decode result gather, world size 2 on gloo (CPU)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kvengine_b200.distributed import contiguous_shards, gather_tokens, shard_requests


def test_lpt_shards_are_balanced_and_deterministic():
    costs = [128 + 64, 40, 300, 300, 12, 77, 190, 190, 5]
    a = shard_requests(costs, 3)
    assert a == shard_requests(costs, 3)
    assert sorted(i for s in a for i in s) == list(range(len(costs)))
    loads = [sum(costs[i] for i in s) for s in a]
    assert max(loads) - min(loads) <= max(costs)
    assert contiguous_shards(10, 4) == [[0, 1], [2, 3, 4], [5, 6], [7, 8, 9]]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        costs = [10, 3, 7, 8, 1]
        mine = shard_requests(costs, world)[rank]
        # stand-in for decoding: request i yields i+1 copies of 100+i
        local = {i: [100 + i] * (i + 1) for i in mine}
        got = gather_tokens(local)
        results[rank] = got
    finally:
        dist.destroy_process_group()


def test_gather_tokens_gloo_world2():
    world = 2
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, port, results), nprocs=world, join=True, start_method="spawn")
    want = {i: [100 + i] * (i + 1) for i in range(5)}
    assert dict(results[0]) == want and dict(results[1]) == want


def _failing_worker(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            raise RuntimeError("simulated rank failure before the gather")
        gather_tokens({0: [1, 2, 3]})
    finally:
        dist.destroy_process_group()


def test_a_failed_rank_surfaces_as_an_error_not_a_hang():
    """A rank that dies before the collective makes the others fail within the
    process-group timeout (host-side failure injection; no device involved)."""
    port = _free_port()
    with pytest.raises(Exception):
        mp.start_processes(_failing_worker, args=(2, port), nprocs=2, join=True, start_method="spawn")
