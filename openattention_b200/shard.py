"""How a batched decode step is split over the GPUs of one box (one process per GPU).

The decode path has no exchange inside a step: all state and compute are per (request, KV head), so
ranks only meet for timing (max over ranks) and, end to end, to gather attention outputs.  With at
least as many requests as ranks the requests are split in contiguous blocks; with fewer requests
than ranks (batch < 8 on 8 GPUs) the 8 KV heads are split instead, each rank keeping its KV heads
and their 4 query heads for every request (the plan of ours_graph.py:270-340 run per shard).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .geometry import G, HKV


@dataclass(frozen=True)
class Shard:
    kind: str            # "request" or "kvhead"
    req_start: int
    req_count: int
    kv_start: int
    kv_count: int

    @property
    def q_heads(self) -> range:
        return range(self.kv_start * G, (self.kv_start + self.kv_count) * G)


def plan(batch: int, world: int, rank: int) -> Shard:
    """This rank's share of `batch` requests x 8 KV heads.  Every (request, KV head) pair is owned by
    exactly one rank; shares differ by at most one request (or KV head)."""
    if batch <= 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad plan arguments: batch={batch} world={world} rank={rank}")
    if batch >= world:
        base, extra = divmod(batch, world)
        start = rank * base + min(rank, extra)
        return Shard("request", start, base + (1 if rank < extra else 0), 0, HKV)
    if HKV % world:
        raise ValueError(f"{world} ranks cannot split {HKV} KV heads evenly for batch {batch}")
    per = HKV // world
    return Shard("kvhead", 0, batch, rank * per, per)


def request_seed(base: int, rank: int) -> int:
    """Seed of a rank's synthetic requests (independent per rank, fixed across runs)."""
    return base + 1000 * rank


def max_over_ranks(x: float, group=None, device=None) -> float:
    """Maximum of a host float over the ranks of `group` (identity without a process group)."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_rows(local: torch.Tensor, group=None) -> torch.Tensor:
    """Concatenate every rank's (rows, ...) output along dim 0 in rank order (the end-to-end gather of
    request-sharded attention outputs).  All ranks must pass tensors of the same shape."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return local
    world = dist.get_world_size(group)
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    if local.is_cuda:
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    else:
        dist.all_gather(list(out.chunk(world)), local.contiguous(), group=group)
    return out
