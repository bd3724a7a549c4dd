"""bench.py's request partition (CPU).

Requests are dealt round-robin by global id (sharding.shard_round_robin).
With --strong the config-3 batch is served once in total: rank g of N takes
the requests whose id is g modulo N, and each keeps the context length and
query of that request in the single-GPU run, so the N-GPU step does exactly
the single-GPU work.  Weak scaling serves 64*N distinct requests, 64 per rank.
"""
import numpy as np
import pytest

import bench


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_strong_partition_covers_every_request_once(world):
    total = 64
    ids = [np.arange(total)[rank::world] for rank in range(world)]
    assert sorted(np.concatenate(ids).tolist()) == list(range(total))
    full = bench.workload_contexts(total)
    for rank, gids in enumerate(ids):
        assert np.array_equal(bench.workload_contexts(total)[gids], full[gids])


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_weak_partition_serves_distinct_requests(world):
    sharding = __import__("importlib").import_module("15-618_dynamic_sparse_decode_b200.sharding")
    total = 64 * world
    ids = [sharding.shard_round_robin(np.arange(total), world, rank) for rank in range(world)]
    assert all(len(g) == 64 for g in ids)
    assert sorted(np.concatenate(ids).tolist()) == list(range(total))
    assert np.array_equal(ids[0], np.arange(0, total, world))
    if world == 1:   # at one GPU the weak workload is the config-3 workload itself
        assert np.array_equal(bench.workload_contexts(total)[ids[0]], bench.workload_contexts())


def test_strong_partition_keeps_each_requests_query(dsd):
    saved = bench.BATCH
    try:
        bench.BATCH = 64
        full = bench.queries_host(dsd)
        gids = np.arange(64)[1::4]
        bench.BATCH = len(gids)
        part = bench.queries_host(dsd, gids)
    finally:
        bench.BATCH = saved
    assert np.array_equal(part, full[gids])
