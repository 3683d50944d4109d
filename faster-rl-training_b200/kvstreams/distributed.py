"""One process per GPU: how rollouts are split across ranks and how timings are combined.

Rollouts are independent streams, so the paged-KV path shards by rollout with no
collective on the data path: every rank owns whole GRPO groups (so group-relative
advantages, training/grpo.py:15-24 of the reference, stay rank-local), its own cache,
pool, tables and free list.  The only cross-rank operations are reductions of scalars
outside the hot path (timings, metrics).
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class RankInfo:
    rank: int
    world: int
    local_rank: int

    @classmethod
    def from_env(cls) -> "RankInfo":
        return cls(int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
                   int(os.environ.get("LOCAL_RANK", 0)))


def shard_groups(num_rollouts: int, group_size: int, world: int, rank: int) -> range:
    """Rollout indices owned by ``rank``: a contiguous run of whole groups, the groups
    spread as evenly as possible (the first ``n_groups % world`` ranks get one more)."""
    if group_size <= 0 or num_rollouts % group_size:
        raise ValueError("number of rollouts must be a multiple of group_size")
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    n_groups = num_rollouts // group_size
    base, extra = divmod(n_groups, world)
    first = rank * base + min(rank, extra)
    count = base + (1 if rank < extra else 0)
    return range(first * group_size, (first + count) * group_size)


def reduce_max(value: float, device: torch.device | None = None) -> float:
    """Maximum of ``value`` over all ranks (identity without an initialised process group)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(value: float, device: torch.device | None = None) -> float:
    """Sum of ``value`` over all ranks (identity without an initialised process group)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
