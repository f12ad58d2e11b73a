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
