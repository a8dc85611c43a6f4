"""Data-parallel serving across the GPUs of one box: one process per GPU, each
with its own engine (a full weight replica) and its own requests. Requests are
independent, so nothing crosses GPUs on the data path; the host only splits
the request list, gathers the action chunks back in request order, and reduces
timings (max over ranks) for reporting.

The reference serves one request at a time on one GPU
(src/models/gwp05/model.cpp:61 serialises predict calls on a mutex); this is
the batched, multi-GPU serving shape of the north star ("independent requests
sharded data-parallel with no collective").

Collectives here are host-side plumbing (torch.distributed: NCCL on GPUs, gloo
on CPU), never part of the per-request compute.
"""
from __future__ import annotations

from typing import Sequence


def shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the contiguous block of `n` requests that `rank` serves:
    blocks differ in size by at most one, the first n % world ranks get the
    larger ones, and the blocks tile [0, n) in rank order."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n < 0:
        raise ValueError("negative request count")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def request_seed(base_seed: int, rank: int, index: int) -> int:
    """Seed of the index-th synthetic request on `rank` (bench workloads: every
    rank gets its own, distinct requests)."""
    return base_seed + 7919 * rank + index


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Largest `value` over all ranks (the job's time is its slowest rank's).
    Without a process group, the value itself."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_throughput(units_per_rank: Sequence[int], seconds_max: float) -> float:
    """Whole-job throughput: the units all ranks processed over the slowest
    rank's time."""
    if seconds_max <= 0:
        raise ValueError("non-positive time")
    return float(sum(units_per_rank)) / seconds_max


def gather_in_order(local: Sequence, n: int, dist=None):
    """Rank 0 receives every rank's results concatenated in request order
    (rank r's block is shard(n, world, r)); other ranks receive None. Without
    a process group, the local results."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return list(local)
    world, rank = dist.get_world_size(), dist.get_rank()
    start, stop = shard(n, world, rank)
    if len(local) != stop - start:
        raise ValueError(f"rank {rank} holds {len(local)} results for requests [{start}, {stop})")
    parts = [None] * world if rank == 0 else None
    dist.gather_object(list(local), parts, dst=0)
    if rank != 0:
        return None
    out = []
    for r, part in enumerate(parts):
        s, e = shard(n, world, r)
        if len(part) != e - s:
            raise ValueError(f"rank {r} returned {len(part)} results for requests [{s}, {e})")
        out.extend(part)
    return out
