"""Request sharding across the GPUs of one box (one process per GPU).

Requests are independent (own pages, own selection, own attention), so GPU g
owns the requests with request_id % world == g, each with its own page pool;
no collective touches the decode path.  The only collective is the final
statistics gather: one all_gather of a few numbers per rank (NCCL over
NVLink on the GPU box, gloo in CPU tests), and the step time every rank
reports is the maximum over ranks.
"""
from __future__ import annotations

import numpy as np


def shard_round_robin(request_ids, world: int, rank: int) -> np.ndarray:
    """The request ids rank `rank` of `world` serves (request_id % world == rank)."""
    ids = np.asarray(request_ids)
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    return ids[ids % world == rank]


def gather_rank_stats(stats: dict, device=None) -> list[dict]:
    """All-gathers a flat dict of numbers from every rank (rank order)."""
    import torch
    import torch.distributed as dist
    keys = sorted(stats)
    t = torch.tensor([float(stats[k]) for k in keys], dtype=torch.float64, device=device)
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [dict(zip(keys, t.tolist()))]
    out = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [dict(zip(keys, o.tolist())) for o in out]


def max_over_ranks(value: float, device=None) -> float:
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
