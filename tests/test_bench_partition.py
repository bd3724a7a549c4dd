"""bench.py's request partition for strong scaling (CPU).

With --strong the config-3 batch is served once in total: rank g of N takes
the requests whose id is g modulo N, and each keeps the context length and
query of that request in the single-GPU run, so the N-GPU step does exactly
the single-GPU work.
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
