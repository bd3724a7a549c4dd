"""Request sharding and the stats gather on world_size 2 with gloo (CPU)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp



def test_round_robin_partitions_requests():
    import importlib
    sh = importlib.import_module("15-618_dynamic_sparse_decode_b200.sharding")
    ids = np.arange(2048)
    for world in (1, 2, 4, 8):
        parts = [sh.shard_round_robin(ids, world, r) for r in range(world)]
        assert sorted(np.concatenate(parts).tolist()) == ids.tolist()
        assert max(len(p) for p in parts) - min(len(p) for p in parts) <= 1
    with pytest.raises(ValueError):
        sh.shard_round_robin(ids, 2, 2)


def _worker(rank, world, port, q):
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sh = importlib.import_module("15-618_dynamic_sparse_decode_b200.sharding")
    mine = sh.shard_round_robin(np.arange(10), world, rank)
    stats = sh.gather_rank_stats({"tokens": len(mine), "ms": 1.0 + rank})
    mx = sh.max_over_ranks(1.0 + rank)
    q.put((rank, mine.tolist(), stats, mx))
    dist.destroy_process_group()


def test_gloo_two_ranks_gather_and_max():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1] == [0, 2, 4, 6, 8] and res[1][1] == [1, 3, 5, 7, 9]
    for _, _, stats, mx in res:
        assert [s["tokens"] for s in stats] == [5.0, 5.0]
        assert [s["ms"] for s in stats] == [1.0, 2.0]
        assert mx == 2.0
