"""Decoder token-loop throughput on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload single|batched|box|long]

Workloads (synthetic: seeded N(0, 0.02) weights, N(0, 1) encoder memory, a
seeded 8-state table grammar allowing 25% of the vocabulary per state):

* ``single`` (default): one song, 12-layer d1024/16-head/FFN4096 decoder,
  vocabulary 2048, bf16 memory [1, 1500, 1024], greedy decode of 2048 tokens
  at batch 1.  A step = load the window (cross K/V projection) and decode its
  2048 tokens.
* ``batched``: 64 slots of the same decoder, frames U[600, 3000], target
  lengths U[512, 4096], continuous batching with finished songs replaced; a
  step = 64 steps of the whole batch plus the refills they trigger.
* ``box`` (C5): 512 such songs sharded by song over the ranks (longest first
  onto the least-loaded rank); a step = the whole job.  Strong scaling.
* ``long`` (C4): 16 slots, memory [16, 6000, 1024], 8192 tokens each; a step =
  load and decode the 16 windows.

Under torchrun every rank decodes its own songs on its own GPU (no
collective on the data path; weak scaling) and ``value`` is the tokens of all
ranks divided by the slowest rank's time.  ``--impl reference`` times the
reference's CPU decode path, restated by the oracle (float32 numpy, all host
cores), on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from sheetsage2_refined_b200.grammar import TableGrammar  # noqa: E402
from sheetsage2_refined_b200.vocab_table import OUT, SOS  # noqa: E402
from sheetsage2_refined_b200.weights import DecoderConfig, DecoderWeights, synthetic_state_dict  # noqa: E402

METRIC = "decoder tokens/s per GPU and box (greedy, batch 1/64); ms/step; % HBM roofline"
CONFIG = DecoderConfig(vocab_size=2048, width=1024, layers=12, heads=16, ffn_width=4096, max_tokens=5120)
WEIGHT_SEED, MEMORY_SEED, GRAMMAR_SEED = 1, 101, 8
SINGLE_FRAMES, SINGLE_TOKENS = 1500, 2048
BATCH, BATCH_FRAMES = 64, 3000
SONGS, SONGS_SEED = 512, 2024
OVERRIDES: dict = {}  # profiling-case overrides of the workload, reported in "config"
CLASS_NAMES = ("qkv", "self_attn", "self_out", "cross_q", "cross_attn", "cross_out", "fc1", "fc2", "logits", "step")


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi SM clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.path = index, None, None

    def __enter__(self):
        import tempfile

        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.index), "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in Path(self.path).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 8 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        except OSError:
            pass
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[4:8]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def reduce_max(value: float, world: int, device) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(value: float, world: int, device) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------- CPU arm
def single_config(world: int) -> dict:
    return {"workload": "single-song decode, 12L d1024 h16 ffn4096 V2048, bf16 memory [1,1500,1024], "
                        "2048 greedy tokens per song, batch 1 per GPU",
            "global_batch": world, "seq_len": SINGLE_TOKENS, "parallelism": f"song-sharded x{world}",
            "l2": "inputs larger than L2 (352 MB of weights streamed per token)"}


class CpuDecoder:
    """The reference's CPU decode path (the oracle's float32 mode) on the single-song workload."""

    def __init__(self):
        from oracle.engine import OracleEngine
        from sheetsage2_refined_b200.weights import memory_array

        grammar = TableGrammar(CONFIG.vocab_size, states=8, density=0.25, seed=GRAMMAR_SEED)
        self.eng = OracleEngine(CONFIG, synthetic_state_dict(CONFIG, WEIGHT_SEED), grammar, batch=1,
                                frames=SINGLE_FRAMES, mode="fp32")
        self.eng.load(0, memory_array(SINGLE_FRAMES, CONFIG.width, MEMORY_SEED), [SOS, OUT], None, SINGLE_FRAMES,
                      target=SINGLE_TOKENS)
        self.eng.step()  # warm-up

    def sample(self, seconds: float, min_tokens: int = 4, threads: int | None = None):
        """Greedy tokens for ``seconds`` of decode on ``threads`` threads (default: every host core);
        returns (tokens/s, tokens, threads, seconds)."""

        from threadpoolctl import threadpool_limits

        import torch

        cores = threads or os.cpu_count() or 1
        # every host core by default, also under torchrun (which sets OMP_NUM_THREADS=1 per rank);
        # the float32 port's matrix products run on torch's CPU thread pool
        before = torch.get_num_threads()
        torch.set_num_threads(cores)
        try:
            with threadpool_limits(limits=cores):
                n, t0 = 0, time.perf_counter()
                while n < min_tokens or time.perf_counter() - t0 < seconds:
                    self.eng.step()
                    n += 1
                dt = time.perf_counter() - t0
                return n / dt, n, cores, dt
        finally:
            torch.set_num_threads(before)


def run_reference(args, world, rank):
    if rank != 0:
        return
    cpu = CpuDecoder()
    values, seconds = [], []
    tokens = 0
    for _ in range(args.warmup):
        cpu.sample(seconds=0.5, min_tokens=2)
    for _ in range(args.steps):
        v, n, cores, dt = cpu.sample(seconds=args.cpu_seconds / max(args.steps, 1), min_tokens=4)
        values.append(v)
        seconds.append(dt)
        tokens += n
    value = statistics.mean(values)
    one, one_n, _, _ = cpu.sample(seconds=max(2.0, args.cpu_seconds / 4), min_tokens=2, threads=1)
    sample = (f"single-song workload: greedy decode from position 1, {tokens} tokens over {args.steps} steps, "
              "float32 restatement of the reference CPU path (numpy, torch CPU matrix products)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * statistics.mean(seconds),
        "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": single_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample,
                         "one_thread": {"value": one, "tokens": one_n}},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm
def load_launches(eng) -> int:
    """Kernel launches of one ``load`` with the prefix [SOS, OUT] and bfloat16 memory.

    The cross K/V projection (one launch per layer), then the one-row prefill
    of position 0: a full layer but only the K/V projection in the last one
    (6 launches per layer with the attention fused with its out-projection,
    5 when the cross attention also computes its query rows, 11 on
    tensor-core engines with their LayerNorm launches); the one-kernel
    step engine prefills with one launch.
    """

    L, per_step = CONFIG.layers, eng.step_launches
    if per_step == 1:
        return L + 1
    if per_step == 11 * L + 2:
        return L + 11 * (L - 1) + 2
    if per_step == 6 * L + 1:  # attention fused with its out-projection
        return L + 6 * (L - 1) + 1
    if per_step == 5 * L + 1:  # ... and the cross attention computing its own query rows
        return L + 5 * (L - 1) + 1
    return L + 8 * (L - 1) + 1


class SingleSong:
    """One song at batch 1: load its window and decode 2048 greedy tokens (one bench step)."""

    def __init__(self, eng, torch, device, rank):
        from sheetsage2_refined_b200.weights import memory_array

        self.eng, self.torch, self.device = eng, torch, device
        mem = torch.from_numpy(memory_array(SINGLE_FRAMES, CONFIG.width, MEMORY_SEED + rank)).to(torch.bfloat16)
        self.mem_dev = mem.to(device)
        self.mem_pinned = mem.pin_memory()
        self.h2d = SINGLE_FRAMES * CONFIG.width * 2 + 2 * 8
        self.d2h = (SINGLE_TOKENS + 3) * 8 + 1
        self.launches = 0

    def config(self, world):
        return single_config(world)

    def _count(self):
        self.launches += load_launches(self.eng) + self.eng.step_launches * SINGLE_TOKENS

    def step_device(self):
        self.eng.load(0, self.mem_dev, [SOS, OUT], None, SINGLE_FRAMES, target=SINGLE_TOKENS)
        self.eng.run(SINGLE_TOKENS)
        self._count()
        return SINGLE_TOKENS

    def step_e2e(self):
        self.eng.load(0, self.mem_pinned, [SOS, OUT], None, SINGLE_FRAMES, target=SINGLE_TOKENS)
        self.eng.run(SINGLE_TOKENS)
        done = self.eng.finished()
        tokens, _ = self.eng.take(0)
        assert done == [0] and len(tokens) == SINGLE_TOKENS + 3
        return SINGLE_TOKENS

    def time_load(self, k: int = 5) -> dict:
        """CUDA-event time of one window's ``load`` (memory resident on the device)."""

        torch = self.torch
        stream = torch.cuda.current_stream(self.device)
        ms = []
        for _ in range(k):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            self.eng.load(0, self.mem_dev, [SOS, OUT], None, SINGLE_FRAMES, target=SINGLE_TOKENS)
            end.record(stream)
            torch.cuda.synchronize(self.device)
            ms.append(start.elapsed_time(end))
        flop = 2.0 * SINGLE_FRAMES * CONFIG.width * 2 * CONFIG.width * CONFIG.layers
        return {"ms": statistics.median(ms), "loads": k, "frames": SINGLE_FRAMES, "prefix_tokens": 2,
                "cross_kv_gflop": flop / 1e9,
                "what": "one window's load: memory copy, cross K/V projection of every layer on the tcgen05 GEMM, "
                        "slot state, prefill of position 0"}

    def prepare_profile(self):
        self.eng.load(0, self.mem_dev, [SOS, OUT], None, SINGLE_FRAMES, target=SINGLE_TOKENS)
        self.eng.run(SINGLE_TOKENS // 2)

    def finish_profile(self):
        self.eng.run(SINGLE_TOKENS)


class Batched:
    """64 slots with continuous refill: songs of U[600, 3000] frames and U[512, 4096] tokens.

    One bench step = 64 decode steps of the whole batch (two polls of 32, the
    reference scheduler's poll interval, transcribe.py:233,360) plus the
    take / load refills they trigger.  Tokens = position increments of the
    live slots during the step.
    """

    POLL = 32

    def __init__(self, eng, torch, device, rank):
        self.eng, self.torch, self.device = eng, torch, device
        self.rng = np.random.default_rng(1000 + rank)
        gen = torch.Generator(device=device)
        gen.manual_seed(MEMORY_SEED + rank)
        self.pool = [torch.randn(BATCH_FRAMES, CONFIG.width, generator=gen, device=device).to(torch.bfloat16)
                     for _ in range(4)]
        self.pool_pinned = [m.cpu().pin_memory() for m in self.pool]
        self.k = 0
        self.launches = 0
        self.h2d_total = 0
        self.steps_done = 0
        self.start_pos = [0] * BATCH
        for slot in range(BATCH):
            self._refill(slot, pinned=False)

    def config(self, world):
        return {"workload": "64-slot continuous batching, 12L d1024 h16 ffn4096 V2048, bf16 memory, frames "
                            "U[600,3000], targets U[512,4096], refill on finish",
                "global_batch": BATCH * world, "seq_len": 4096, "parallelism": f"song-sharded x{world}",
                "l2": "inputs larger than L2 (weights and K/V streamed every step)"}

    def _refill(self, slot, pinned):
        frames = int(self.rng.integers(600, BATCH_FRAMES + 1))
        target = int(self.rng.integers(512, 4097))
        mem = (self.pool_pinned if pinned else self.pool)[self.k % len(self.pool)][:frames]
        self.k += 1
        self.eng.load(slot, mem, [SOS, OUT], None, frames, target=target)
        self.start_pos[slot] = 1
        self.launches += load_launches(self.eng)
        if pinned:
            self.h2d_total += frames * CONFIG.width * 2 + 16

    def _positions(self):
        return self.eng.state["position"].cpu().tolist()

    def _step(self, pinned):
        tokens = 0
        for _ in range(2):
            self.eng.run(self.POLL)
            self.launches += self.eng.step_launches * self.POLL
            done = self.eng.finished()
            if done:
                pos = self._positions()
                for slot in done:
                    tokens += pos[slot] - self.start_pos[slot]
                    self.eng.take(slot)
                    self._refill(slot, pinned)
        self.steps_done += 1
        return tokens

    def step_device(self):
        return self._measure(False)

    def step_e2e(self):
        return self._measure(True)

    def _measure(self, pinned):
        tokens = self._step(pinned)
        pos = self._positions()
        tokens += sum(p - s for p, s in zip(pos, self.start_pos))
        self.start_pos = pos
        return tokens

    @property
    def h2d(self):
        return int(self.h2d_total / max(self.steps_done, 1))

    @property
    def d2h(self):
        return BATCH * 8 * 4

    def prepare_profile(self):
        pass

    def finish_profile(self):
        pass


class Box:
    """C5: 512 songs (frames U[600, 3000], targets U[512, 4096], seeded) sharded by song.

    ``shard.partition_songs`` gives every rank its songs, longest first onto
    the least-loaded rank; each rank decodes its share with 64 slots and
    continuous refill.  One bench step = the whole job (every song of the
    rank decoded to its end); the warm-up is one short batched pass.
    """

    POLL = 32
    scaling = "strong"  # the 512 songs are split over the ranks

    def __init__(self, eng, torch, device, rank, world):
        from sheetsage2_refined_b200.shard import partition_songs

        self.eng, self.torch, self.device = eng, torch, device
        rng = np.random.default_rng(SONGS_SEED)
        self.frames = rng.integers(600, BATCH_FRAMES + 1, SONGS).tolist()
        self.targets = rng.integers(512, 4097, SONGS).tolist()
        self.share = partition_songs(self.targets, world)[rank]
        gen = torch.Generator(device=device)
        gen.manual_seed(MEMORY_SEED + rank)
        self.pool = [torch.randn(BATCH_FRAMES, CONFIG.width, generator=gen, device=device).to(torch.bfloat16)
                     for _ in range(4)]
        self.pool_pinned = [m.cpu().pin_memory() for m in self.pool]
        self.launches = 0
        self.h2d_last = 0

    def config(self, world):
        return {"workload": f"{SONGS} songs sharded by song (LPT) over {world} GPU(s), 64 slots per GPU with "
                            "refill, 12L d1024 h16 ffn4096 V2048, frames U[600,3000], targets U[512,4096]",
                "global_batch": BATCH * world, "seq_len": 4096, "parallelism": f"song-sharded x{world}",
                "l2": "inputs larger than L2 (weights and K/V streamed every step)"}

    def _load(self, slot, song, pinned):
        mem = (self.pool_pinned if pinned else self.pool)[song % len(self.pool)][: self.frames[song]]
        self.eng.load(slot, mem, [SOS, OUT], None, self.frames[song], target=self.targets[song])
        self.launches += load_launches(self.eng)
        if pinned:
            self.h2d_last += self.frames[song] * CONFIG.width * 2 + 16

    def _job(self, songs, pinned):
        queue, live, tokens = list(songs), {}, 0
        self.h2d_last = 0
        for slot in range(BATCH):
            if queue:
                live[slot] = queue.pop(0)
                self._load(slot, live[slot], pinned)
        while live:
            self.eng.run(self.POLL)
            self.launches += self.eng.step_launches * self.POLL
            for slot in self.eng.finished():
                tokens += len(self.eng.take(slot)[0]) - 3  # SOS, OUT and the closing EOS are not decoded tokens
                del live[slot]
                if queue:
                    live[slot] = queue.pop(0)
                    self._load(slot, live[slot], pinned)
        return tokens

    def warm_step(self):
        return self._job(self.share[:BATCH], False)

    def step_device(self):
        return self._job(self.share, False)

    def step_e2e(self):
        return self._job(self.share, True)

    @property
    def h2d(self):
        return self.h2d_last

    @property
    def d2h(self):
        return 0

    def prepare_profile(self):
        for slot in range(BATCH):
            self._load(slot, self.share[slot % len(self.share)], False)
        self.eng.run(256)

    def finish_profile(self):
        self.eng.run(4096)
        for slot in self.eng.finished():
            self.eng.take(slot)


class LongContext:
    """C4: 16 slots, encoder memory [16, 6000, 1024], 8192 tokens each (split-K attention over long rows).

    One bench step = load the 16 windows and decode 8192 tokens in every slot.
    """

    SLOTS, FRAMES, TOKENS = 16, 6000, 8192

    def __init__(self, eng, torch, device, rank):
        self.eng, self.torch, self.device = eng, torch, device
        gen = torch.Generator(device=device)
        gen.manual_seed(MEMORY_SEED + rank)
        self.mem = torch.randn(self.FRAMES, CONFIG.width, generator=gen, device=device).to(torch.bfloat16)
        self.mem_pinned = self.mem.cpu().pin_memory()
        self.launches = 0
        self.h2d = self.SLOTS * (self.FRAMES * CONFIG.width * 2 + 16)
        self.d2h = self.SLOTS * (self.TOKENS + 3) * 8

    def config(self, world):
        return {"workload": "16 slots x 8192 tokens, encoder memory [16, 6000, 1024] bf16, 12L d1024 h16 ffn4096 "
                            "V2048 (max_tokens 8200)", "global_batch": self.SLOTS * world, "seq_len": self.TOKENS,
                "parallelism": f"song-sharded x{world}", "l2": "inputs larger than L2"}

    def _run(self, mem):
        for slot in range(self.SLOTS):
            self.eng.load(slot, mem, [SOS, OUT], None, self.FRAMES, target=self.TOKENS)
            self.launches += load_launches(self.eng)
        self.eng.run(self.TOKENS)
        self.launches += self.eng.step_launches * self.TOKENS
        return self.SLOTS * self.TOKENS

    def warm_step(self):
        for slot in range(self.SLOTS):
            self.eng.load(slot, self.mem, [SOS, OUT], None, self.FRAMES, target=64)
        self.eng.run(64)
        for slot in self.eng.finished():
            self.eng.take(slot)
        return 0

    def step_device(self):
        n = self._run(self.mem)
        for slot in self.eng.finished():
            self.eng.take(slot)
        return n

    def step_e2e(self):
        n = self._run(self.mem_pinned)
        done = self.eng.finished()
        for slot in done:
            self.eng.take(slot)
        assert len(done) == self.SLOTS
        return n

    def prepare_profile(self):
        for slot in range(self.SLOTS):
            self.eng.load(slot, self.mem, [SOS, OUT], None, self.FRAMES, target=self.TOKENS)
        self.eng.run(self.TOKENS // 2)

    def finish_profile(self):
        self.eng.run(self.TOKENS)
        for slot in self.eng.finished():
            self.eng.take(slot)


def run_b200(args, world, rank, local):
    import torch

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    from sheetsage2_refined_b200 import BatchDecoder

    grammar = TableGrammar(CONFIG.vocab_size, states=8, density=0.25, seed=GRAMMAR_SEED)
    dec = DecoderWeights(CONFIG, synthetic_state_dict(CONFIG, WEIGHT_SEED))
    # S2R_ENGINE_FLAGS (S2R_FLAG_* bits) lets a profiler run use plain launches
    flags = int(os.environ.get("S2R_ENGINE_FLAGS", "0"))
    if args.workload == "single":
        eng = BatchDecoder(dec, None, batch=1, frames=SINGLE_FRAMES, grammar=grammar, device=device, flags=flags)
        work = SingleSong(eng, torch, device, rank)
    elif args.workload == "box":
        eng = BatchDecoder(dec, None, batch=BATCH, frames=BATCH_FRAMES, grammar=grammar, device=device, flags=flags)
        work = Box(eng, torch, device, rank, world)
    elif args.workload == "long":
        eng = BatchDecoder(dec, None, batch=LongContext.SLOTS, frames=LongContext.FRAMES, grammar=grammar,
                           device=device, flags=flags)
        work = LongContext(eng, torch, device, rank)
    else:
        eng = BatchDecoder(dec, None, batch=BATCH, frames=BATCH_FRAMES, grammar=grammar, device=device, flags=flags)
        work = Batched(eng, torch, device, rank)

    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):  # warm-up (also captures the step graph)
        getattr(work, "warm_step", work.step_device)()
    torch.cuda.synchronize(device)

    # roofline: per-kernel times of one profiled step at a representative position
    work.prepare_profile()
    prof = profile(eng)
    work.finish_profile()
    torch.cuda.synchronize(device)

    def timed(fn, k):
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        tokens = 0
        start.record(stream)
        for _ in range(k):
            tokens += fn()
        end.record(stream)
        torch.cuda.synchronize(device)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        return start.elapsed_time(end), tokens

    gpu_index = local
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        try:
            gpu_index = int(visible.split(",")[local])
        except (ValueError, IndexError):
            pass
    launches0 = work.launches
    with ClockSampler(gpu_index) as clocks:
        ms, tokens = timed(work.step_device, args.steps)
    launches = work.launches - launches0
    clock_summary = clocks.summary()
    ms_e2e, tokens_e2e = timed(work.step_e2e, max(1, args.steps // 2))
    load = work.time_load() if hasattr(work, "time_load") else None

    ms_max = reduce_max(ms, world, device)
    ms_e2e_max = reduce_max(ms_e2e, world, device)
    tokens_all = reduce_sum(tokens, world, device)
    tokens_e2e_all = reduce_sum(tokens_e2e, world, device)
    value = tokens_all / (ms_max / 1000.0)
    e2e = tokens_e2e_all / (ms_e2e_max / 1000.0)

    cpu = None
    if world == 1 and not args.no_cpu:
        cpu_dec = CpuDecoder()
        v, n, cores, _ = cpu_dec.sample(seconds=args.cpu_seconds)
        one, one_n, _, _ = cpu_dec.sample(seconds=max(2.0, args.cpu_seconds / 4), min_tokens=2, threads=1)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{n} greedy tokens of the single-song workload from position 1 (load excluded), "
                         "float32 restatement of the reference CPU path (numpy, torch CPU matrix products), all host cores",
               "one_thread": {"value": one, "tokens": one_n}}

    if rank == 0:
        peak, peak_kind = peaks()
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": getattr(work, "scaling", "weak"), "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {**work.config(world), **({"profiling_overrides": OVERRIDES} if OVERRIDES else {})},
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": work.h2d, "d2h_bytes_per_step": work.d2h},
            "gpu_launches": launches,
            "clocks": clock_summary,
            "roofline": roofline(prof, peak, peak_kind, args.workload),
            "step_roofline": prof["step"],
            "kernel_classes": {k: {"us_per_launch": 1000.0 * v["ms"] / max(v["launches"], 1),
                                   "launches": v["launches"],
                                   "gbs": v["bytes_per_launch"] / max(v["ms"] / max(v["launches"], 1), 1e-9) / 1e6}
                               for k, v in prof["classes"].items()},
            "cpu_baseline": cpu,
        }
        if load is not None:
            line["load"] = load
        print(json.dumps(line), flush=True)
    eng.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def profile(eng):
    import ctypes as C

    from sheetsage2_refined_b200 import _lib

    k = len(CLASS_NAMES)
    ms = (C.c_float * k)()
    by = (C.c_double * k)()
    n = (C.c_int32 * k)()
    _lib.check(eng._lib.s2r_profile_step(eng._ctx, ms, by, n, eng._stream()))
    classes = {name: {"ms": ms[i], "launches": n[i], "bytes_per_launch": by[i]} for i, name in enumerate(CLASS_NAMES)
               if n[i] > 0}
    total_ms = sum(ms[i] for i in range(k))
    total_bytes = sum(by[i] * n[i] for i in range(k))
    return {"classes": classes, "step": {"ms_kernels": total_ms, "bytes": total_bytes,
                                         "gbs": total_bytes / (total_ms * 1e-3) / 1e9}}


# DRAM traffic of the attention launches (dram__bytes_read.sum + dram__bytes_write.sum, one ncu
# capture each; profiles/): per launch at the single-song workload's position ~1,025 (the fused
# launches: self attention + out-projection; cross attention + its query rows + out-projection),
# and as a ratio to the algorithmic bytes for the batched workload, whose launches are too large
# to capture (a one-row launch of the same kernel on the small case; traffic grows with the
# rows' keys, so the ratio carries over).
NCU_TRAFFIC = {("single", "self_attn"): 6_403_584, ("single", "cross_attn"): 10_443_520}
NCU_TRAFFIC_RATIO = {(w, k): 3_097_088 / 3_096_576 for w in ("batched", "box", "long") for k in ("cross_attn", "self_attn")}


def roofline(prof, peak, peak_kind, workload):
    name, c = max(prof["classes"].items(), key=lambda kv: kv[1]["ms"])
    per_launch_s = c["ms"] / max(c["launches"], 1) / 1000.0
    achieved = c["bytes_per_launch"] / per_launch_s / 1e9
    traffic = NCU_TRAFFIC.get((workload, name))
    if traffic is None and (workload, name) in NCU_TRAFFIC_RATIO:
        traffic = c["bytes_per_launch"] * NCU_TRAFFIC_RATIO[(workload, name)]
    return {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_kind": peak_kind, "traffic": traffic,
            "bytes_per_launch": c["bytes_per_launch"], "us_per_launch": per_launch_s * 1e6}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--workload", default="single", choices=("single", "batched", "box", "long"))
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    # smaller cases of the same kernels for ncu captures that must fit a few GB (not bench lines)
    ap.add_argument("--layers", type=int, default=None, help="override the decoder depth (profiling cases)")
    ap.add_argument("--max-tokens", type=int, default=None, help="override the context length (profiling cases)")
    ap.add_argument("--batch-frames", type=int, default=None, help="override the batched frames cap (profiling cases)")
    args = ap.parse_args()
    global CONFIG, BATCH_FRAMES, OVERRIDES
    if args.layers or args.max_tokens:
        CONFIG = dataclasses.replace(CONFIG, layers=args.layers or CONFIG.layers,
                                     max_tokens=args.max_tokens or CONFIG.max_tokens)
        OVERRIDES.update(layers=CONFIG.layers, max_tokens=CONFIG.max_tokens)
    if args.batch_frames:
        BATCH_FRAMES = args.batch_frames
        OVERRIDES.update(batch_frames=BATCH_FRAMES)
    if args.workload == "long":  # C4 decodes 8192 tokens: a longer position table
        CONFIG = dataclasses.replace(CONFIG, max_tokens=max(CONFIG.max_tokens, 8200))
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_b200(args, world, rank, local)


if __name__ == "__main__":
    main()
