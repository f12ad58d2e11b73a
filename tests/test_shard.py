"""Song sharding (no GPU): the partition, and a 2-rank gloo run of the gather."""

import os
import socket

import pytest
import torch.multiprocessing as mp

from sheetsage2_refined_b200.shard import gather_to_rank0, partition_songs


def test_partition_is_complete_and_balanced():
    import numpy as np

    rng = np.random.default_rng(3)
    costs = rng.integers(512, 4097, 512).tolist()
    for world in (1, 2, 4, 8):
        shares = partition_songs(costs, world)
        flat = sorted(i for share in shares for i in share)
        assert flat == list(range(len(costs)))
        loads = [sum(costs[i] for i in share) for share in shares]
        assert max(loads) - min(loads) <= max(costs)  # LPT bound


def test_partition_rejects_empty_world():
    with pytest.raises(ValueError):
        partition_songs([1, 2], 0)


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, costs, queue):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        share = partition_songs(costs, world)[rank]
        # stand-in for decoding: each rank "decodes" its songs into token lists
        results = {i: [rank, i, costs[i]] for i in share}
        merged = gather_to_rank0(results)
        if rank == 0:
            queue.put(merged)
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_over_gloo():
    costs = [700, 4000, 512, 2500, 1200, 3333, 900]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, costs, queue)) for r in range(2)]
    for p in procs:
        p.start()
    merged = queue.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(merged) == list(range(len(costs)))
    shares = partition_songs(costs, 2)
    for i, (rank, song, cost) in merged.items():
        assert song == i and cost == costs[i] and i in shares[rank]


def _timing_rank(rank, world, port, queue):
    import sys

    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cpu = torch.device("cpu")
        slowest = bench.reduce_max(100.0 + rank, world, cpu)  # each rank's device time, ms
        tokens = bench.reduce_sum(2048.0 * (rank + 1), world, cpu)
        if rank == 0:
            queue.put((slowest, tokens))
    finally:
        dist.destroy_process_group()


def test_bench_takes_the_slowest_rank_and_all_tokens_over_gloo():
    """The bench's whole-job value: tokens of every rank over the slowest rank's time."""

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_timing_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    slowest, tokens = queue.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert slowest == 101.0 and tokens == 2048.0 * 3


class FakeEngine:
    """The BatchDecoder surface decode_songs drives, without a GPU: a slot loaded with target n
    finishes after n steps with tokens prefix + [song marker] * n."""

    def __init__(self, batch):
        self.batch = batch
        self.loaded = [None] * batch  # (prefix, target, steps done)

    def free_slots(self):
        return [s for s in range(self.batch) if self.loaded[s] is None]

    def load(self, slot, memory, prefix, stop, frames=None, target=None):
        assert self.loaded[slot] is None
        self.loaded[slot] = [list(prefix), int(target), 0, int(memory)]

    def run(self, steps):
        for entry in self.loaded:
            if entry is not None:
                entry[2] = min(entry[1], entry[2] + steps)

    def finished(self):
        return [s for s, e in enumerate(self.loaded) if e is not None and e[2] >= e[1]]

    def take(self, slot):
        prefix, target, _, marker = self.loaded[slot]
        self.loaded[slot] = None
        return prefix + [marker] * target + [2], "eos"


def test_decode_songs_refills_every_slot_and_decodes_each_song_once():
    from sheetsage2_refined_b200.shard import DecodeStats, Song, decode_songs

    import numpy as np

    rng = np.random.default_rng(5)
    targets = rng.integers(10, 200, 37).tolist()
    songs = {i: Song(memory=1000 + i, prefix=[1, 3], target=t) for i, t in enumerate(targets)}
    stats = DecodeStats()
    out = decode_songs(FakeEngine(8), songs, poll_every=16, stats=stats)
    assert sorted(out) == list(range(37)) and stats.loads == 37
    for i, (tokens, ended) in out.items():
        assert tokens == [1, 3] + [1000 + i] * targets[i] + [2] and ended == "eos"
    assert 0.0 < stats.occupancy(8) <= 1.0 and stats.tail_seconds() >= 0.0


def _box_rank(rank, world, port, targets, queue):
    import torch.distributed as dist

    from sheetsage2_refined_b200.shard import Song, decode_box

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        songs = [Song(memory=1000 + i, prefix=[1, 3], target=t) for i, t in enumerate(targets)]
        merged = decode_box(FakeEngine(4), songs, targets, poll_every=8)
        if rank == 0:
            queue.put(merged)
        else:
            assert merged is None
    finally:
        dist.destroy_process_group()


def test_two_rank_box_job_over_gloo():
    """The box job: each rank decodes its LPT share with refill; rank 0 gets every song once."""

    targets = [70, 400, 51, 250, 120, 333, 90, 17, 260, 44, 180]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_box_rank, args=(r, 2, port, targets, queue)) for r in range(2)]
    for p in procs:
        p.start()
    merged = queue.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(merged) == list(range(len(targets)))
    for i, (tokens, ended) in merged.items():
        assert tokens == [1, 3] + [1000 + i] * targets[i] + [2]


class FakeAsyncEngine(FakeEngine):
    """FakeEngine with the asynchronous poll and take: a poll reports the flags as they were when
    it was queued, and a take frees the slot at once."""

    def __init__(self, batch):
        super().__init__(batch)
        self.polled = None
        self.taken = {}

    def finished_async(self):
        self.polled = self.finished()

    def finished_ready(self, wait=False):
        done, self.polled = self.polled, None
        return [s for s in done if self.loaded[s] is not None]

    def take_async(self, slot):
        self.taken[slot] = self.take(slot)

    def take_ready(self, slot, wait=False):
        return self.taken.pop(slot)


def test_overlapped_decode_songs_matches_the_synchronous_loop():
    from sheetsage2_refined_b200.shard import DecodeStats, Song, decode_songs

    import numpy as np

    rng = np.random.default_rng(6)
    targets = rng.integers(5, 150, 41).tolist()
    songs = {i: Song(memory=1000 + i, prefix=[1, 3], target=t) for i, t in enumerate(targets)}
    sync = decode_songs(FakeEngine(6), songs, poll_every=8)
    stats = DecodeStats()
    over = decode_songs(FakeAsyncEngine(6), songs, poll_every=8, stats=stats, overlap=True)
    assert over == sync and sorted(over) == list(range(41)) and stats.loads == 41
