"""One process per GPU: batch shards and the host-side combination of results.

The fused-block path has no exchange step (each row of the batch is an
independent sequence), so ranks run their own batch shard with no collective
on the data path.  Only the metrics cross ranks, after the forward: the
per-layer spike counts are summed (the reference's per-layer spike rate over
the whole global batch, model.py:286-291) and a timing is reduced to its
maximum.  Works with any torch.distributed backend (NCCL on GPUs, gloo on CPU).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Tuple

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class RankInfo:
    rank: int
    world: int
    local_rank: int


def rank_info() -> RankInfo:
    """RANK / WORLD_SIZE / LOCAL_RANK as set by torchrun (1 process when unset)."""
    return RankInfo(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                    int(os.environ.get("LOCAL_RANK", "0")))


def batch_shard(global_batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [start, stop) of the global batch that `rank` runs; the first
    global_batch % world ranks take one extra row."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def sum_counts(counts: torch.Tensor) -> torch.Tensor:
    """Per-layer spike counts summed over all ranks (every rank gets the sum)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return counts
    parts = [torch.zeros_like(counts) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, counts)
    return torch.stack(parts).sum(0)


def global_counts(counts: torch.Tensor, numel: int) -> Tuple[torch.Tensor, int]:
    """Per-layer spike counts and the per-layer element count summed over all
    ranks, so that count / numel is the reference's spike rate over the whole
    global batch (ranks may hold different numbers of rows)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return counts, int(numel)
    v = torch.cat([counts.reshape(-1).to(torch.int64),
                   torch.tensor([int(numel)], dtype=torch.int64, device=counts.device)])
    parts = [torch.zeros_like(v) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, v)
    tot = torch.stack(parts).sum(0)
    return tot[:-1], int(tot[-1].item())


def max_over_ranks(value: float, device: torch.device) -> float:
    """The largest `value` over all ranks (the job's time is its slowest rank's)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
