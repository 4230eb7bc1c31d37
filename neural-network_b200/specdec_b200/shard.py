"""Request-parallel sharding over GPUs (one process per GPU).

Speculative-decoding requests are independent, so N GPUs serve disjoint
request sets with no data-path collective (weak scaling: every rank keeps its
own batch).  The only cross-rank steps are host-side: agreeing on the global
request set, and taking the MAX of the per-rank device times, since the job
finishes when its slowest rank does.
"""
from __future__ import annotations

from typing import Sequence, Tuple

import numpy as np


def request_range(per_rank: int, rank: int, world: int) -> Tuple[int, int]:
    """Rank r serves global requests [r * per_rank, (r + 1) * per_rank)."""
    if not (0 <= rank < world) or per_rank < 1:
        raise ValueError("bad rank / world / per_rank")
    return rank * per_rank, (rank + 1) * per_rank


def shard(global_array: np.ndarray, per_rank: int, rank: int, world: int) -> np.ndarray:
    lo, hi = request_range(per_rank, rank, world)
    if global_array.shape[0] < hi:
        raise ValueError("global request set smaller than world * per_rank")
    return np.ascontiguousarray(global_array[lo:hi])


def max_over_ranks(values: Sequence[float], dist=None, device=None) -> list:
    """Element-wise max of `values` over all ranks (identity without dist)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return [float(v) for v in values]
    import torch

    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def sum_over_ranks(values: Sequence[float], dist=None, device=None) -> list:
    """Element-wise sum of `values` over all ranks (identity without dist):
    the units every rank processed."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return [float(v) for v in values]
    import torch

    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.tolist()
