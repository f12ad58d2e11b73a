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
* ``decode_songs`` decodes a queue of songs on one engine with continuous
  batching: every free slot is loaded with the next song, the engine runs
  ``poll_every`` steps, finished slots are taken and refilled
  (transcribe.py:279-362 for songs of one window each).
* ``decode_box`` is the whole box job on the calling rank: its LPT share of
  the songs through ``decode_songs``, then the gather on rank 0.
"""

from __future__ import annotations

import heapq
import time
from dataclasses import dataclass, field
from typing import Any


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


@dataclass
class Song:
    """One window to decode: ``BatchDecoder.load`` arguments (engine.py:180-232)."""

    memory: Any                   # [frames, width] encoder memory (host or device tensor / array)
    prefix: list = field(default_factory=list)
    stop_seconds: float | None = None
    frames: int | None = None     # real frames (None: the engine's)
    target: int | None = None     # table grammar: generated tokens before it ends
    frame_logp: dict | None = None


@dataclass
class DecodeStats:
    """What ``decode_songs`` saw: host seconds since the start and live slots at every poll, the
    loads, and when the last song was loaded (after it the batch can only drain)."""

    polls: list = field(default_factory=list)  # (seconds, live slots)
    loads: int = 0
    drained_at: float | None = None

    def occupancy(self, batch: int) -> float:
        """Time-weighted mean of live slots / batch over the job."""

        if len(self.polls) < 2:
            return 1.0
        total = area = 0.0
        for (t0, live), (t1, _) in zip(self.polls, self.polls[1:]):
            total += t1 - t0
            area += (t1 - t0) * live
        return area / (total * batch) if total > 0 else 1.0

    def tail_seconds(self) -> float:
        """Host seconds from the last load to the end of the job (the batch drains)."""

        if self.drained_at is None or not self.polls:
            return 0.0
        return max(0.0, self.polls[-1][0] - self.drained_at)


def decode_songs(engine, songs: dict, poll_every: int = 32, stats: DecodeStats | None = None,
                 overlap: bool = False) -> dict:
    """Decode ``songs`` (``{key: Song}``, in queue order) on ``engine``; returns ``{key: (tokens, ended)}``.

    Continuous batching as the reference scheduler does it: fill every free
    slot, run ``poll_every`` steps, take the finished slots (one device read per
    poll, ``finished``), refill them, until every song has ended.

    ``overlap`` (engines with ``finished_async``): the host never waits for the
    device to drain.  The next ``poll_every`` steps are queued before the
    flags of the previous ones are read, finished slots are taken
    asynchronously and refilled behind the steps in flight.  A window's
    tokens do not depend on which slot it runs in or when it starts, so the
    results equal the synchronous loop's.
    """

    if overlap and hasattr(engine, "finished_async"):
        return _decode_songs_overlapped(engine, songs, poll_every, stats)

    queue = list(songs)
    live: dict[int, Any] = {}
    results: dict = {}
    t0 = time.perf_counter()

    def refill():
        for slot in engine.free_slots():
            if not queue:
                break
            key = queue.pop(0)
            song = songs[key]
            kwargs = {"frame_logp": song.frame_logp} if song.frame_logp is not None else {}
            if song.target is not None:
                kwargs["target"] = song.target
            engine.load(slot, song.memory, list(song.prefix), song.stop_seconds, song.frames, **kwargs)
            live[slot] = key
            if stats is not None:
                stats.loads += 1
        if stats is not None and not queue and stats.drained_at is None:
            stats.drained_at = time.perf_counter() - t0

    refill()
    while live:
        engine.run(poll_every)
        done = engine.finished()
        if stats is not None:
            stats.polls.append((time.perf_counter() - t0, len(live)))
        for slot in done:
            results[live.pop(slot)] = engine.take(slot)
        refill()
    return results


def _decode_songs_overlapped(engine, songs: dict, poll_every: int, stats: DecodeStats | None) -> dict:
    queue = list(songs)
    live: dict[int, Any] = {}
    pending: dict[int, Any] = {}  # slot -> key of an asynchronous take not yet read
    results: dict = {}
    t0 = time.perf_counter()

    def collect(wait=False):
        for slot in list(pending):
            got = engine.take_ready(slot, wait=wait)
            if got is not None:
                results[pending.pop(slot)] = got

    def refill():
        for slot in engine.free_slots():
            if not queue:
                break
            if slot in pending:  # its tokens must be read before the slot's next take
                results[pending.pop(slot)] = engine.take_ready(slot, wait=True)
            key = queue.pop(0)
            song = songs[key]
            kwargs = {"frame_logp": song.frame_logp} if song.frame_logp is not None else {}
            if song.target is not None:
                kwargs["target"] = song.target
            engine.load(slot, song.memory, list(song.prefix), song.stop_seconds, song.frames, **kwargs)
            live[slot] = key
            if stats is not None:
                stats.loads += 1
        if stats is not None and not queue and stats.drained_at is None:
            stats.drained_at = time.perf_counter() - t0

    refill()
    engine.run(poll_every)
    engine.finished_async()
    snapshot = dict(live)  # the window of every slot when the poll was queued
    while live:
        engine.run(poll_every)
        done = engine.finished_ready(wait=True)
        polled, snapshot = snapshot, dict(live)
        engine.finished_async()
        if stats is not None:
            stats.polls.append((time.perf_counter() - t0, len(live)))
        for slot in done:
            # a slot refilled after the poll was queued still shows its old window's flag
            if slot in live and polled.get(slot) == live[slot]:
                engine.take_async(slot)
                pending[slot] = live.pop(slot)
        refill()
        collect()
    engine.finished_ready(wait=True)  # the last queued poll
    collect(wait=True)
    return results


def decode_box(engine, songs: list, costs, poll_every: int = 32, stats: DecodeStats | None = None) -> dict | None:
    """The box job on this rank: its share of ``songs`` (``partition_songs(costs, world)``), decoded
    with ``decode_songs``, gathered on rank 0 (``{song index: (tokens, ended)}``; None elsewhere)."""

    import torch.distributed as dist

    world, rank = (dist.get_world_size(), dist.get_rank()) if dist.is_available() and dist.is_initialized() else (1, 0)
    share = partition_songs(costs, world)[rank]
    local = decode_songs(engine, {i: songs[i] for i in share}, poll_every, stats)
    return gather_to_rank0(local)
