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


def gather_token_ids(tokens, n_requests: int, max_new: int, device=None):
    """Every rank's generated ids (this rank's shard, in shard order) on rank 0 as
    {request index: [ids]}; None on the other ranks.  One all-gather of a fixed-size
    [ceil(n / world), 1 + max_new] int32 block per rank (length, ids, -1 padding), so the
    collective has the same shape on every rank."""
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    rows = (n_requests + world - 1) // world
    block = torch.full((rows, 1 + max_new), -1, dtype=torch.int32)
    for j, toks in enumerate(tokens):
        ids = [int(x) for x in toks]
        if len(ids) > max_new or j >= rows:
            raise ValueError("more tokens or requests than the gather block holds")
        block[j, 0] = len(ids)
        block[j, 1:1 + len(ids)] = torch.tensor(ids, dtype=torch.int32)
    block = block.to(device) if device is not None else block
    if world == 1:
        parts = [block]
    else:
        parts = [torch.empty_like(block) for _ in range(world)]
        dist.all_gather(parts, block)
    if rank != 0:
        return None
    out = {}
    for r, part in enumerate(parts):
        part = part.cpu()
        for j, i in enumerate(shard(n_requests, r, world)):
            n = int(part[j, 0])
            out[i] = [int(x) for x in part[j, 1:1 + n]]
    return out


def tokens_digest(by_request) -> str:
    """sha256 (first 16 hex digits) over every request's ids in request order: equal for
    any GPU count as long as a request's tokens do not depend on how requests are
    batched."""
    import hashlib
    h = hashlib.sha256()
    for i in sorted(by_request):
        h.update(int(i).to_bytes(4, "little") + len(by_request[i]).to_bytes(4, "little"))
        for t in by_request[i]:
            h.update(int(t).to_bytes(4, "little", signed=True))
    return h.hexdigest()[:16]
