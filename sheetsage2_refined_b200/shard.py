"""Song sharding across the GPUs of one box (one process per GPU).

Songs are independent: each has its own K/V cache, grammar state and
encoder memory, and only the weights are shared (replicated per GPU).  The
work therefore splits by song with no collective on the data path: every
rank decodes its share on its own engine and the token lists are gathered on
the host at the end.

* ``partition_songs`` assigns songs longest-first to the rank with the least
  work so far (LPT scheduling), so that ranks finish together even when song
  lengths span 8x (512..4096 tokens).
* ``gather_to_rank0`` collects every rank's ``{song: result}`` dict on rank 0
  through ``torch.distributed.gather_object`` (gloo or NCCL process group);
  without a process group it returns the local dict.
"""

from __future__ import annotations

import heapq


def partition_songs(costs, world: int) -> list[list[int]]:
    """Song indices per rank, longest first onto the least-loaded rank (ties: lowest rank)."""

    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, rank) for rank in range(world)]
    shares: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, rank = heapq.heappop(heap)
        shares[rank].append(i)
        heapq.heappush(heap, (load + costs[i], rank))
    return shares


def gather_to_rank0(results: dict) -> dict | None:
    """Merge every rank's results on rank 0 (other ranks get None)."""

    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return dict(results)
    world, rank = dist.get_world_size(), dist.get_rank()
    bucket = [None] * world if rank == 0 else None
    dist.gather_object(results, bucket, dst=0)
    if rank != 0:
        return None
    merged: dict = {}
    for part in bucket:
        merged.update(part)
    return merged
