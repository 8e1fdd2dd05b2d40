"""Replica sharding of independent utterances or streams over the GPUs of one node.

Utterances and streams share no state (the reference is batch 1 with no cross-request
state, Sources/MoonshineMLX/MoonshineStreaming.swift:8-43), so N GPUs run N full model
replicas, one process per GPU, with no collective on the hot path.  This module holds the
host side of that: the length-balanced partition, the per-rank run, and the gather of ids and
timings on rank 0 over a torch.distributed process group (NCCL on GPUs, gloo on CPU).
"""
from __future__ import annotations

import time
from typing import Callable, List, Optional, Sequence, Tuple


def partition_by_length(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Indices of each rank's share: sorted by length (longest first, ties by index) and dealt
    round-robin, so every rank gets about the same total audio; each rank's list is in
    ascending index order."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    shares: List[List[int]] = [[] for _ in range(world)]
    for k, i in enumerate(order):
        shares[k % world].append(i)
    return [sorted(s) for s in shares]


def run_shard(items: Sequence, share: Sequence[int], transcribe: Callable[[List], List]) -> List:
    """Runs `transcribe` on this rank's items (in index order) and returns its results."""
    return list(transcribe([items[i] for i in share])) if share else []


def gather_results(results: List, share: Sequence[int], n_total: int, group=None) -> Optional[List]:
    """Gathers every rank's (share, results) on rank 0 and returns the results in the original
    order there (None on other ranks).  Without a process group the call is local."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        out = [None] * n_total
        for i, r in zip(share, results):
            out[i] = r
        return out
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    gathered = [None] * world if rank == 0 else None
    dist.gather_object((list(share), results), gathered, dst=0, group=group)
    if rank != 0:
        return None
    out = [None] * n_total
    for sh, res in gathered:
        for i, r in zip(sh, res):
            out[i] = r
    if any(o is None for o in out) and n_total:
        raise RuntimeError("a shard is missing from the gather")
    return out


def max_over_ranks(seconds: float, group=None, device=None) -> float:
    """The largest of every rank's time (the job's wall time is the slowest replica's)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return float(seconds)
    t = torch.tensor([float(seconds)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def sharded_transcription(items: Sequence, lengths: Sequence[int],
                          transcribe: Callable[[List], List], group=None,
                          device=None) -> Tuple[Optional[List], float]:
    """One rank's part of a sharded job: partition, run this rank's share, gather on rank 0.
    Returns (results in input order on rank 0 else None, max-over-ranks seconds)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        dist.barrier(group=group)
    else:
        rank, world = 0, 1
    share = partition_by_length(lengths, world)[rank]
    t0 = time.perf_counter()
    res = run_shard(items, share, transcribe)
    seconds = max_over_ranks(time.perf_counter() - t0, group, device)
    return gather_results(res, share, len(items), group), seconds
