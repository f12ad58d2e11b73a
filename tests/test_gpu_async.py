"""Asynchronous polling and takes (``s2r_poll_finished_async`` / ``s2r_take_async``).

A scheduler that queues the next steps before it reads the finished flags,
takes finished slots without waiting for the device and refills them behind
the steps in flight (``shard.decode_songs(..., overlap=True)``) must produce
the same tokens and end reasons for every song as the synchronous loop (the
reference's ``finished`` / ``take``, engine.py:248-262): a window's tokens
do not depend on its slot or on when it starts.
"""

import numpy as np
import pytest
import torch

import scenarios as sc
from helpers import cuda_engine
from sheetsage2_refined_b200.shard import DecodeStats, Song, decode_songs
from sheetsage2_refined_b200.vocab_table import OUT, SOS
from sheetsage2_refined_b200.weights import memory_array

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")


def songs(n=14, seed=4):
    rng = np.random.default_rng(seed)
    out = {}
    for i in range(n):
        frames = int(rng.integers(40, sc.C1_FRAMES + 1))
        prefix = [SOS, OUT] + rng.integers(4, sc.C1.vocab_size, int(rng.integers(0, 4))).tolist()
        mem = memory_array(sc.C1_FRAMES, sc.C1.width, 900 + i)
        out[i] = Song(memory=mem, prefix=prefix, frames=frames, target=int(rng.integers(5, 90)))
    return out


@pytest.mark.parametrize("batch", [4, 16], ids=["cuda-core", "tensor-core"])
def test_overlapped_loop_matches_the_synchronous_one(batch):
    work = songs()
    sync = decode_songs(cuda_engine(sc.C1, sc.C1_SEED, sc.c1_grammar(), batch, sc.C1_FRAMES), work, poll_every=8)
    stats = DecodeStats()
    eng = cuda_engine(sc.C1, sc.C1_SEED, sc.c1_grammar(), batch, sc.C1_FRAMES)
    over = decode_songs(eng, work, poll_every=8, stats=stats, overlap=True)
    print(f"overlapped loop, batch {batch}: {len(over)} songs, {len(stats.polls)} polls, {stats.loads} loads")
    assert sorted(over) == sorted(work) and over == sync
    assert eng.free_pages == eng_pages(eng)


def eng_pages(eng):
    return eng.batch * -(-eng.max_tokens // 64)


def test_async_poll_and_take_states():
    eng = cuda_engine(sc.C1_SHORT, sc.BATCH_SEED, sc.batch_grammar(), 2, 16)
    with pytest.raises(Exception):
        eng.finished_ready()  # nothing requested
    mem = memory_array(16, sc.C1_SHORT.width, 0)
    eng.load(0, mem, [SOS, OUT], None, 16, target=10)
    eng.run(12)
    eng.finished_async()
    assert eng.finished_ready(wait=True) == [0]
    eng.take_async(0)
    assert eng.free_slots() == [0, 1]
    tokens, ended = eng.take_ready(0, wait=True)
    assert ended == "eos" and len(tokens) == 2 + 10 + 1 and tokens[-1] == 2
    with pytest.raises(Exception):
        eng.take_ready(0)  # already read
