"""Data-parallel request sharding across GPUs (one process per GPU).

The reference engine has no multi-device path; requests (pages or crops) are
independent, so the B200 build partitions them by index over the ranks of a
torch.distributed process group (NCCL on GPUs, gloo on CPU tests) and uses a
collective only after the timed region, to gather per-rank results and
timings on rank 0.  Every rank takes the same collective steps in the same
order, errors included, and every wait is bounded by the process group's
timeout.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class RankInfo:
    rank: int
    world: int
    local_rank: int


def rank_info() -> RankInfo:
    """Rank / world / local rank from the torchrun environment (defaults: one process)."""
    return RankInfo(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                    int(os.environ.get("LOCAL_RANK", "0")))


def shard(n_items: int, rank: int, world: int) -> list[int]:
    """Request indices owned by `rank`: rank, rank + world, ... (round robin, so ranks
    differ by at most one request)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    return list(range(rank, n_items, world))


def init(backend: str, timeout_s: float = 120.0, device_id=None) -> RankInfo:
    """Join the process group (127.0.0.1 rendezvous from the environment)."""
    info = rank_info()
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device_id is not None:
        kwargs["device_id"] = device_id
    dist.init_process_group(backend, rank=info.rank, world_size=info.world, **kwargs)
    return info


def gather_to_rank0(obj):
    """Every rank contributes `obj`; rank 0 receives the list in rank order, the others None."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [obj]
    out = [None] * dist.get_world_size() if dist.get_rank() == 0 else None
    dist.gather_object(obj, out, dst=0)
    return out


def max_over_ranks(value: float, device=None) -> float:
    """Max of a scalar over all ranks (the timing rule for multi-GPU numbers)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device=None) -> float:
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def run_sharded(n_requests: int, work, rank: int, world: int):
    """Run `work(index)` for this rank's shard and gather {index: result} on rank 0."""
    local = {i: work(i) for i in shard(n_requests, rank, world)}
    parts = gather_to_rank0(local)
    if parts is None:
        return None
    merged = {}
    for part in parts:
        overlap = merged.keys() & part.keys()
        if overlap:
            raise RuntimeError(f"requests {sorted(overlap)} produced by two ranks")
        merged.update(part)
    if sorted(merged) != list(range(n_requests)):
        raise RuntimeError("gathered results do not cover every request exactly once")
    return merged
