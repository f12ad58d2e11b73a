"""Decoder token-loop throughput on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload all|single|batched|box|long|real]

Workloads (synthetic: seeded N(0, 0.02) weights, N(0, 1) encoder memory; the
d1024 workloads use a seeded 8-state table grammar allowing 25% of the
vocabulary per state, the product-shape ones the real vocabulary, grammar,
mode bias and frame-head rescoring):

* ``single`` (the headline): one song, 12-layer d1024/16-head/FFN4096 decoder,
  vocabulary 2048, bf16 memory [1, 1500, 1024], greedy decode of 2048 tokens
  at batch 1.  A step = load the window (cross K/V projection) and decode its
  2048 tokens.
* ``batched``: 64 slots of the same decoder, frames U[600, 3000], target
  lengths U[512, 4096], continuous batching with finished songs replaced; a
  step = 64 steps of the whole batch plus the refills they trigger.
* ``box``: 512 such songs sharded by song over the ranks (longest first onto
  the least-loaded rank), 64 slots per GPU with refill; a step = the whole
  job.  Strong scaling: the 512 songs are split over the ranks.
* ``real_b1`` / ``real_b64``: the product decoder (6 layers, d512, 8 heads,
  FFN 2048, 32,576 tokens, 7,500 frames) with the real grammar, mode bias and
  six rescoring terms; batch 1 (a step = load + 512 tokens) and 64 slots with
  refill (a step = 32 decode steps).
* ``long``: 16 slots, memory [16, 6000, 1024], 8192 tokens each (not in the
  default run; ``--workload long``).

The default run (``--workload all``) reports ``single`` as the headline
``value`` and the others under ``workloads``; ``--workload X`` runs one.
Under torchrun every rank decodes on its own GPU with no collective on the
data path; ``value`` is the tokens of all ranks over the slowest rank's time.

Reference measurements (the unmodified reference package, installed under
``baseline/_ref``): ``reference_gpu`` in the line is its own CUDA path (bf16
autocast, one CUDA graph per bucket) at the single-song and batched
workloads, and ``cpu_baseline`` / ``--impl reference`` its CPU path on every
host core over a bounded sample of the single-song workload.  Without the
install both fall back to the oracle's float32 restatement of that CPU path.
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
REAL = DecoderConfig(vocab_size=32576, width=512, layers=6, heads=8, ffn_width=2048, max_tokens=5120)
WEIGHT_SEED, MEMORY_SEED, GRAMMAR_SEED, REAL_SEED = 1, 101, 8, 6
SINGLE_FRAMES, SINGLE_TOKENS = 1500, 2048
PREFILL_LENGTHS = (512, 2048)  # prefix lengths of the load timings (overlap-primed windows)
PREFIX_SEED = 23
BATCH, BATCH_FRAMES = 64, 3000
SONGS, SONGS_SEED = 512, 2024
REAL_FRAMES, REAL_B1_TOKENS = 7500, 512
REAL_PROMPTS = ("timestamp", "downbeat_meter", "chord_detail", "key_mode", "melody_full")
REAL_MODE_BIAS = [0.0, 1.5, -0.5, 2.0, 0.25, -1.0, 3.0, 0.5, -2.0]
REAL_FRAME_WEIGHT = {"root": 0.5, "bass": 0.4, "detail": 0.3, "quality": 0.3, "downbeat": 2.0, "meter": 2.0}
OVERRIDES: dict = {}  # profiling-case overrides of the workload, reported in "config"
CLASS_NAMES = ("qkv", "self_attn", "self_out", "cross_q", "cross_attn", "cross_out", "fc1", "fc2", "logits")


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


def gather_all(value, world: int):
    """Every rank's ``value`` (a small picklable object), in rank order."""

    if world == 1:
        return [value]
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, value)
    return out


def c2_grammar() -> TableGrammar:
    return TableGrammar(CONFIG.vocab_size, states=8, density=0.25, seed=GRAMMAR_SEED)


def single_config(world: int) -> dict:
    return {"workload": "single-song decode, 12L d1024 h16 ffn4096 V2048, bf16 memory [1,1500,1024], "
                        "2048 greedy tokens per song, batch 1 per GPU",
            "global_batch": world, "seq_len": SINGLE_TOKENS, "parallelism": f"song-sharded x{world}",
            "l2": "inputs larger than L2 (352 MB of weights streamed per token)"}


# ---------------------------------------------------------------- CPU decode (reference arm, cpu_baseline)
class CpuDecoder:
    """The reference's CPU decode path on the single-song workload.

    With the reference installed (``baseline/_ref``) this is its own
    ``BatchDecoder`` on CPU (float32, eager, engine.py:69-70,244-245) driven
    through the table grammar (``kind`` "reference"); without it, the oracle's
    float32 restatement of that path (``kind`` "port").
    """

    def __init__(self):
        from reference_path import load_reference
        from sheetsage2_refined_b200.weights import memory_array

        ref = load_reference()
        memory = memory_array(SINGLE_FRAMES, CONFIG.width, MEMORY_SEED)
        if ref is not None:
            import torch

            from reference_path import ref_decoder, set_target, table_engine

            self.kind = "reference"
            decoder = ref_decoder(ref, CONFIG, WEIGHT_SEED, "cpu")
            self.eng = table_engine(ref, decoder, c2_grammar(), 1, SINGLE_FRAMES)
            with torch.inference_mode():
                self.eng.load(0, torch.from_numpy(memory), [SOS, OUT], None, SINGLE_FRAMES)
            set_target(self.eng, 0, SINGLE_TOKENS)
            self._step = self._ref_step
        else:
            from oracle.engine import OracleEngine

            self.kind = "port"
            self.eng = OracleEngine(CONFIG, synthetic_state_dict(CONFIG, WEIGHT_SEED), c2_grammar(), batch=1,
                                    frames=SINGLE_FRAMES, mode="fp32")
            self.eng.load(0, memory, [SOS, OUT], None, SINGLE_FRAMES, target=SINGLE_TOKENS)
            self._step = self.eng.step
        self._step()  # warm-up

    def _ref_step(self):
        import torch

        with torch.inference_mode():
            self.eng.run(1)

    def describe(self) -> str:
        if self.kind == "reference":
            return "the reference's own BatchDecoder on CPU (float32, eager), installed from its package"
        return "float32 restatement of the reference CPU path (numpy, torch CPU matrix products)"

    def sample(self, seconds: float, min_tokens: int = 4, threads: int | None = None):
        """Greedy tokens for ``seconds`` of decode on ``threads`` threads (default: every host core);
        returns (tokens/s, tokens, threads, seconds)."""

        from threadpoolctl import threadpool_limits

        import torch

        cores = threads or os.cpu_count() or 1
        # every host core, also under torchrun (which sets OMP_NUM_THREADS=1 per rank)
        before = torch.get_num_threads()
        torch.set_num_threads(cores)
        try:
            with threadpool_limits(limits=cores):
                n, t0 = 0, time.perf_counter()
                while n < min_tokens or time.perf_counter() - t0 < seconds:
                    self._step()
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
              + cpu.describe())
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * statistics.mean(seconds),
        "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": single_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": cpu.kind, "sample": sample,
                         "one_thread": {"value": one, "tokens": one_n}},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm: workloads
def load_launches(eng, layers: int, prefix_len: int = 2) -> int:
    """Kernel launches of one ``load`` of a bfloat16 window and a prefix of ``prefix_len`` tokens.

    The cross K/V projection (one launch for up to 32 layers), then the prefill
    of the prefix positions before the last in chunks of 128 rows: each chunk
    a full layer but only the K/V projection in the last one.  Chunks of more
    than 8 rows (and every chunk of a tensor-core engine) run the tensor-core
    layer, 11 launches; shorter ones the engine's CUDA-core decode kernels (5
    or 6 a layer; one-slot engines decode with a fused FFN, 4 launches a
    layer, but prefill with fc1 and fc2, 5).
    """

    L, per_step = layers, eng.step_launches
    n = (L + 31) // 32
    rows = max(0, prefix_len - 1)
    chunks = [128] * (rows // 128) + ([rows % 128] if rows % 128 else [])
    per_layer = (per_step - 1) // L
    if per_layer == 4:  # fused FFN in decode only
        per_layer = 5
    for r in chunks:
        if per_step == 11 * L + 2 or r > 8:
            n += 11 * (L - 1) + 2
        else:
            n += per_layer * (L - 1) + 1
    return n


class SingleSong:
    """One song at batch 1: load its window and decode 2048 greedy tokens (one bench step)."""

    name = "single"

    def __init__(self, torch, device, rank, flags):
        from sheetsage2_refined_b200 import BatchDecoder
        from sheetsage2_refined_b200.weights import memory_array

        dec = DecoderWeights(CONFIG, synthetic_state_dict(CONFIG, WEIGHT_SEED))
        self.eng = BatchDecoder(dec, None, batch=1, frames=SINGLE_FRAMES, grammar=c2_grammar(), device=device,
                                flags=flags)
        self.torch, self.device = torch, device
        mem = torch.from_numpy(memory_array(SINGLE_FRAMES, CONFIG.width, MEMORY_SEED + rank)).to(torch.bfloat16)
        self.mem_dev = mem.to(device)
        self.mem_pinned = mem.pin_memory()
        self.h2d = SINGLE_FRAMES * CONFIG.width * 2 + 2 * 8
        self.d2h = (SINGLE_TOKENS + 3) * 8 + 1
        self.launches = 0

    def config(self, world):
        return single_config(world)

    def _count(self):
        self.launches += load_launches(self.eng, CONFIG.layers) + self.eng.step_launches * SINGLE_TOKENS

    def step_device(self):
        self.eng.load(0, self.mem_dev, [SOS, OUT], None, SINGLE_FRAMES, target=SINGLE_TOKENS)
        self.eng.run(SINGLE_TOKENS)
        self._count()
        return SINGLE_TOKENS

    warm_step = step_device

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
        info = {"ms": statistics.median(ms), "loads": k, "frames": SINGLE_FRAMES, "prefix_tokens": 2,
                "cross_kv_gflop": flop / 1e9,
                "what": "one window's load: memory copy, cross K/V projection of every layer in one tcgen05 launch, "
                        "slot state, prefill of position 0"}
        # a window primed with the overlap of the window before it (transcribe.overlap_prefix): the
        # prefix's K/V are prefilled at load
        rng = np.random.default_rng(PREFIX_SEED)
        for n in PREFILL_LENGTHS:
            prefix = [SOS, OUT] + rng.integers(4, CONFIG.vocab_size, n - 2).tolist()
            ms = []
            for _ in range(3):
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record(stream)
                self.eng.load(0, self.mem_dev, prefix, None, SINGLE_FRAMES, target=SINGLE_TOKENS)
                end.record(stream)
                torch.cuda.synchronize(self.device)
                ms.append(start.elapsed_time(end))
            t = statistics.median(ms)
            info.setdefault("prefill", []).append(
                {"prefix_tokens": n, "load_ms": t, "prefill_us_per_token": 1000.0 * (t - info["ms"]) / (n - 1)})
        return info

    def prepare_profile(self):
        self.eng.load(0, self.mem_dev, [SOS, OUT], None, SINGLE_FRAMES, target=SINGLE_TOKENS)
        self.eng.run(SINGLE_TOKENS // 2)

    def finish_profile(self):
        self.eng.run(SINGLE_TOKENS)


def random_pool(torch, device, frames, width, seed, n=4):
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    pool = [torch.randn(frames, width, generator=gen, device=device).to(torch.bfloat16) for _ in range(n)]
    return pool, [m.cpu().pin_memory() for m in pool]


class Batched:
    """64 slots with continuous refill: songs of U[600, 3000] frames and U[512, 4096] tokens.

    One bench step = 64 decode steps of the whole batch (two polls of 32, the
    reference scheduler's poll interval, transcribe.py:233,360) plus the
    take / load refills they trigger.  Tokens = position increments of the
    live slots during the step.
    """

    name = "batched"
    POLL = 32
    POLLS = 2

    def __init__(self, torch, device, rank, flags):
        from sheetsage2_refined_b200 import BatchDecoder

        dec = DecoderWeights(CONFIG, synthetic_state_dict(CONFIG, WEIGHT_SEED))
        self.eng = BatchDecoder(dec, None, batch=BATCH, frames=BATCH_FRAMES, grammar=c2_grammar(), device=device,
                                flags=flags)
        self.layers = CONFIG.layers
        self.torch, self.device = torch, device
        self.rng = np.random.default_rng(1000 + rank)
        self.pool, self.pool_pinned = random_pool(torch, device, BATCH_FRAMES, CONFIG.width, MEMORY_SEED + rank)
        self._init_slots()

    def _init_slots(self):
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

    def _window(self):
        return int(self.rng.integers(600, BATCH_FRAMES + 1)), int(self.rng.integers(512, 4097))

    def _load(self, slot, frames, target, mem):
        self.eng.load(slot, mem, [SOS, OUT], None, frames, target=target)
        return [SOS, OUT]

    def _refill(self, slot, pinned):
        frames, target = self._window()
        mem = (self.pool_pinned if pinned else self.pool)[self.k % len(self.pool)][:frames]
        self.k += 1
        prefix = self._load(slot, frames, target, mem)
        self.start_pos[slot] = len(prefix) - 1
        self.launches += load_launches(self.eng, self.layers, len(prefix))
        if pinned:
            self.h2d_total += mem.numel() * mem.element_size() + 16

    def _positions(self):
        return self.eng.state["position"].cpu().tolist()

    def _done(self):
        return self.eng.finished()

    def _step(self, pinned):
        tokens = 0
        for _ in range(self.POLLS):
            self.eng.run(self.POLL)
            self.launches += self.eng.step_launches * self.POLL
            done = self._done()
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

    warm_step = step_device

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
    """512 songs (frames U[600, 3000], targets U[512, 4096], seeded) sharded by song.

    ``shard.decode_box`` gives every rank its songs, longest first onto the
    least-loaded rank, and decodes them with 64 slots and continuous refill
    (``shard.decode_songs``); the token lists are gathered on rank 0 after the
    timed region.  One bench step = the whole job; the warm-up loads every
    slot once and runs 64 steps.
    """

    name = "box"
    POLL = 32
    scaling = "strong"  # the 512 songs are split over the ranks

    def __init__(self, torch, device, rank, flags, world):
        from sheetsage2_refined_b200 import BatchDecoder
        from sheetsage2_refined_b200.shard import Song, partition_songs

        dec = DecoderWeights(CONFIG, synthetic_state_dict(CONFIG, WEIGHT_SEED))
        self.eng = BatchDecoder(dec, None, batch=BATCH, frames=BATCH_FRAMES, grammar=c2_grammar(), device=device,
                                flags=flags)
        self.torch, self.device, self.world = torch, device, world
        rng = np.random.default_rng(SONGS_SEED)
        self.frames = rng.integers(600, BATCH_FRAMES + 1, SONGS).tolist()
        self.targets = rng.integers(512, 4097, SONGS).tolist()
        self.share = partition_songs(self.targets, world)[rank]
        self.pool, self.pool_pinned = random_pool(torch, device, BATCH_FRAMES, CONFIG.width, MEMORY_SEED + rank)
        self.songs = {
            pinned: {i: Song(memory=(self.pool_pinned if pinned else self.pool)[i % 4][: self.frames[i]],
                             prefix=[SOS, OUT], frames=self.frames[i], target=self.targets[i]) for i in self.share}
            for pinned in (False, True)}
        self.launches = 0
        self.h2d = sum(self.frames[i] * CONFIG.width * 2 + 16 for i in self.share)
        self.d2h = sum((t + 3) * 8 for t in (self.targets[i] for i in self.share)) + BATCH
        self.stats = None
        self.results = None

    def config(self, world):
        return {"workload": f"{SONGS} songs sharded by song (LPT) over {world} GPU(s), 64 slots per GPU with "
                            "refill, 12L d1024 h16 ffn4096 V2048, frames U[600,3000], targets U[512,4096]",
                "global_batch": BATCH * world, "seq_len": 4096, "parallelism": f"song-sharded x{world}",
                "l2": "inputs larger than L2 (weights and K/V streamed every step)"}

    def _job(self, pinned):
        from sheetsage2_refined_b200.shard import DecodeStats, decode_songs

        self.stats = DecodeStats()
        steps_before = 0
        self.results = decode_songs(self.eng, self.songs[pinned], self.POLL, self.stats)
        polls = len(self.stats.polls)
        self.launches += self.stats.loads * load_launches(self.eng, CONFIG.layers) + \
            self.eng.step_launches * self.POLL * polls + steps_before
        return sum(len(tokens) - 3 for tokens, _ in self.results.values())  # SOS, OUT, closing EOS

    def warm_step(self):
        for slot, i in enumerate(self.share[:BATCH]):
            self.eng.load(slot, self.pool[i % 4][: self.frames[i]], [SOS, OUT], None, self.frames[i],
                          target=self.targets[i])
        self.eng.run(64)
        for slot in range(BATCH):
            if self.eng.loaded[slot]:
                self.eng.take(slot)
        return 0

    def step_device(self):
        return self._job(False)

    def step_e2e(self):
        return self._job(True)

    def job_summary(self) -> dict:
        st = self.stats
        return {"songs": len(self.share), "occupancy": st.occupancy(BATCH), "tail_s": st.tail_seconds(),
                "job_s": st.polls[-1][0] if st.polls else 0.0, "loads": st.loads}

    def prepare_profile(self):
        for slot in range(BATCH):
            i = self.share[slot % len(self.share)]
            self.eng.load(slot, self.pool[i % 4][: self.frames[i]], [SOS, OUT], None, self.frames[i],
                          target=self.targets[i])
        self.eng.run(256)

    def finish_profile(self):
        for slot in range(BATCH):
            if self.eng.loaded[slot]:
                self.eng.take(slot)


class LongContext:
    """16 slots, encoder memory [16, 6000, 1024], 8192 tokens each (split-K attention over long rows).

    One bench step = load the 16 windows and decode 8192 tokens in every slot.
    """

    name = "long"
    SLOTS, FRAMES, TOKENS = 16, 6000, 8192

    def __init__(self, torch, device, rank, flags):
        from sheetsage2_refined_b200 import BatchDecoder

        cfg = dataclasses.replace(CONFIG, max_tokens=max(CONFIG.max_tokens, 8200))
        self.cfg = cfg
        dec = DecoderWeights(cfg, synthetic_state_dict(cfg, WEIGHT_SEED))
        self.eng = BatchDecoder(dec, None, batch=self.SLOTS, frames=self.FRAMES, grammar=c2_grammar(), device=device,
                                flags=flags)
        self.torch, self.device = torch, device
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
            self.launches += load_launches(self.eng, CONFIG.layers)
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


def real_engine(torch, device, batch, flags):
    from sheetsage2_refined_b200 import BatchDecoder, VocabTable

    vocab = VocabTable()
    dec = DecoderWeights(REAL, synthetic_state_dict(REAL, REAL_SEED))
    eng = BatchDecoder(dec, vocab, batch=batch, frames=REAL_FRAMES, prompts=REAL_PROMPTS, mode_bias=REAL_MODE_BIAS,
                       frame_weight=REAL_FRAME_WEIGHT, device=device, flags=flags)
    return eng, vocab


def real_tables(torch, device, rows, seed):
    """Per-frame rescoring tables of one window (``transcribe.frame_tables`` shapes), on ``device``."""

    import scenarios as sc

    return {name: torch.from_numpy(t).to(device) for name, t in sc.rescore_tables(rows, seed).items()
            if name in REAL_FRAME_WEIGHT}


def real_config(world, batch, what):
    return {"workload": f"product decoder shape, {what}: 6L d512 h8 ffn2048 V32576, memory [{REAL_FRAMES},512] bf16, "
                        "real grammar, mode bias, 6 frame-head rescoring terms",
            "global_batch": batch * world, "seq_len": 5120, "parallelism": f"song-sharded x{world}",
            "l2": "inputs larger than L2 (cross K/V and rescoring tables streamed every step)"}


class RealSong:
    """Product shape at batch 1: load a 7,500-frame window and decode 512 greedy tokens."""

    name = "real_b1"

    def __init__(self, torch, device, rank, flags):
        self.torch, self.device = torch, device
        self.eng, vocab = real_engine(torch, device, 1, flags)
        self.prefix = vocab.prompt_prefix(REAL_PROMPTS)
        self.pool, self.pool_pinned = random_pool(torch, device, REAL_FRAMES, REAL.width, MEMORY_SEED + rank, n=1)
        self.tables = real_tables(torch, device, REAL_FRAMES, 91 + rank)
        self.tables_pinned = {k: v.cpu().pin_memory() for k, v in self.tables.items()}
        self.launches = 0
        self.h2d = REAL_FRAMES * REAL.width * 2 + sum(t.numel() * 4 for t in self.tables.values())
        self.d2h = (REAL_B1_TOKENS + len(self.prefix) + 1) * 8 + 1

    def config(self, world):
        return real_config(world, 1, f"batch 1, {REAL_B1_TOKENS} greedy tokens per window")

    def _run(self, mem, tables):
        self.eng.load(0, mem, self.prefix, None, REAL_FRAMES, tables)
        self.eng.run(REAL_B1_TOKENS)
        self.launches += load_launches(self.eng, REAL.layers, len(self.prefix)) + \
            self.eng.step_launches * REAL_B1_TOKENS

    def step_device(self):
        self._run(self.pool[0], self.tables)
        return int(self.eng.state["position"][0].item()) - (len(self.prefix) - 1)

    warm_step = step_device

    def step_e2e(self):
        self._run(self.pool_pinned[0], self.tables_pinned)
        self.eng.finished()
        tokens, _ = self.eng.take(0)
        return len(tokens) - len(self.prefix) - (1 if tokens[-1] == 2 else 0)

    def prepare_profile(self):
        self.eng.load(0, self.pool[0], self.prefix, None, REAL_FRAMES, self.tables)
        self.eng.run(REAL_B1_TOKENS // 2)

    def finish_profile(self):
        self.eng.take(0)


class RealBatched(Batched):
    """Product shape, 64 slots with refill: 7,500-frame windows, one bench step = 32 decode steps.

    Random-init weights rarely end a window by themselves, so each window gets
    a length drawn from U[512, 4096] tokens (the batched workload's targets):
    once a slot has generated that many tokens it is taken and refilled like
    a finished one.
    """

    name = "real_b64"
    POLLS = 1

    def __init__(self, torch, device, rank, flags):
        self.torch, self.device = torch, device
        self.eng, vocab = real_engine(torch, device, BATCH, flags)
        self.layers = REAL.layers
        self.prefix = vocab.prompt_prefix(REAL_PROMPTS)
        self.rng = np.random.default_rng(2000 + rank)
        self.pool, self.pool_pinned = random_pool(torch, device, REAL_FRAMES, REAL.width, MEMORY_SEED + rank)
        self.tables = [real_tables(torch, device, REAL_FRAMES, 93 + i) for i in range(2)]
        self.tables_pinned = [{k: v.cpu().pin_memory() for k, v in t.items()} for t in self.tables]
        self.ends = [0] * BATCH
        self._init_slots()

    def config(self, world):
        return real_config(world, BATCH, "64 slots with refill, real frames U[3000, 7500]")

    def _window(self):
        frames, length = int(self.rng.integers(3000, REAL_FRAMES + 1)), int(self.rng.integers(512, 4097))
        if self.k < BATCH:  # the first windows start part-way through, as in a batch that has been running
            length = max(16, int(length * self.rng.random()))
        return frames, length

    def _load(self, slot, frames, target, mem):
        tables = (self.tables_pinned if mem.device.type == "cpu" else self.tables)[self.k % 2]
        self.eng.load(slot, mem, self.prefix, None, frames, tables)
        if mem.device.type == "cpu":
            self.h2d_total += sum(t.numel() * 4 for t in tables.values())
        self.ends[slot] = len(self.prefix) - 1 + target
        return self.prefix

    def _done(self):
        done = set(self.eng.finished())
        pos = self._positions()
        return sorted(done | {s for s in range(BATCH) if self.eng.loaded[s] and pos[s] >= self.ends[s]})


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
# and as a ratio to the algorithmic bytes for the batched workloads, whose launches are too large
# to capture (a one-row launch of the same kernel on the small case; traffic grows with the
# rows' keys, so the ratio carries over).  The single-song cross attention also asks the L2 for
# the next FFN's 16,777,216 bytes of weights (that kernel cannot start beside it), which a
# serialised capture counts against the cross attention: 27,206,144 = its own 10,428,928 plus
# the FFN's; nothing is read twice.
NCU_TRAFFIC = {("single", "self_attn"): 6_397_440, ("single", "cross_attn"): 27_206_144}
NCU_TRAFFIC_NOTE = {("single", "cross_attn"): "includes the L2 prefetch of the next FFN's 16,777,216 bytes of weights"}
NCU_TRAFFIC_RATIO = {(w, k): 3_097_088 / 3_096_576 for w in ("batched", "box", "long") for k in ("cross_attn", "self_attn")}


def roofline(prof, peak, peak_kind, workload, kernel=None):
    if kernel is None:
        name, c = max(prof["classes"].items(), key=lambda kv: kv[1]["ms"])
    else:
        name, c = kernel, prof["classes"][kernel]
    per_launch_s = c["ms"] / max(c["launches"], 1) / 1000.0
    achieved = c["bytes_per_launch"] / per_launch_s / 1e9
    traffic = NCU_TRAFFIC.get((workload, name))
    if traffic is None and (workload, name) in NCU_TRAFFIC_RATIO:
        traffic = c["bytes_per_launch"] * NCU_TRAFFIC_RATIO[(workload, name)]
    out = {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
           "frac": achieved / peak, "peak_kind": peak_kind, "traffic": traffic,
           "bytes_per_launch": c["bytes_per_launch"], "us_per_launch": per_launch_s * 1e6}
    if (workload, name) in NCU_TRAFFIC_NOTE:
        out["traffic_note"] = NCU_TRAFFIC_NOTE[(workload, name)]
    return out


def kernel_classes(prof):
    return {k: {"us_per_launch": 1000.0 * v["ms"] / max(v["launches"], 1), "launches": v["launches"],
                "gbs": v["bytes_per_launch"] / max(v["ms"] / max(v["launches"], 1), 1e-9) / 1e6}
            for k, v in prof["classes"].items()}


def measure(work, args, steps, warmup, e2e_steps, world, device, gpu_index, torch):
    """Warm-up, one profiled step (roofline), then ``steps`` timed steps (memory resident) and
    ``e2e_steps`` through the public API from pinned host memory, max over ranks."""

    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        work.warm_step()
    torch.cuda.synchronize(device)
    work.prepare_profile()
    prof = profile(work.eng)
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

    launches0 = work.launches
    with ClockSampler(gpu_index) as clocks:
        ms, tokens = timed(work.step_device, steps)
    launches = work.launches - launches0
    job = work.job_summary() if hasattr(work, "job_summary") else None
    ms_e2e, tokens_e2e = timed(work.step_e2e, e2e_steps)
    ms_max = reduce_max(ms, world, device)
    ms_e2e_max = reduce_max(ms_e2e, world, device)
    tokens_all = reduce_sum(tokens, world, device)
    tokens_e2e_all = reduce_sum(tokens_e2e, world, device)
    per_rank = gather_all({"ms": ms, "tokens": tokens, **(job or {})}, world)
    peak, peak_kind = peaks()
    out = {
        "value": tokens_all / (ms_max / 1000.0), "unit": "tokens/s", "steps": steps, "warmup": warmup,
        "ms_per_step": ms_max / steps, "scaling": getattr(work, "scaling", "weak"),
        "config": work.config(world),
        "e2e": {"value": tokens_e2e_all / (ms_e2e_max / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": int(work.h2d), "d2h_bytes_per_step": int(work.d2h), "steps": e2e_steps},
        "gpu_launches": int(reduce_sum(launches, world, device)),
        "clocks": clocks.summary(),
        "roofline": roofline(prof, peak, peak_kind, work.name),
        "step_roofline": prof["step"],
        "kernel_classes": kernel_classes(prof),
    }
    if "logits" in prof["classes"] and work.name.startswith("real"):
        out["roofline_logits"] = roofline(prof, peak, peak_kind, work.name, "logits")
    if world > 1 or job is not None:
        out["per_rank"] = per_rank
    return out


# ---------------------------------------------------------------- the reference's own CUDA path
def reference_gpu(torch, device, seconds: float = 20.0):
    """The unmodified reference engine on this GPU (bf16 autocast, per-bucket CUDA graphs) at the
    single-song workload (one 2048-token song after a warm-up song that captures its graphs) and the
    batched workload (64 slots, 2 timed bench steps of 64 decode steps with refill)."""

    from reference_path import load_reference, ref_decoder, set_target, table_engine
    from sheetsage2_refined_b200.weights import memory_array

    ref = load_reference()
    if ref is None:
        return {"unavailable": "the reference package is not installed under baseline/_ref"}
    out = {"what": "the reference's own BatchDecoder on cuda: bf16 autocast, one CUDA graph per cache bucket "
                   "(engine.py:234-281), same weights, memory and grammar as this arm"}
    stream = torch.cuda.current_stream(device)

    def timed(fn):
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        n = fn()
        end.record(stream)
        torch.cuda.synchronize(device)
        return start.elapsed_time(end), n

    # the decoder's parameters are ordinary tensors (the engine reads their version counters, engine.py:151-153);
    # the decode itself runs under inference mode, as transcribe_many runs it (transcribe.py:225)
    decoder = ref_decoder(ref, CONFIG, WEIGHT_SEED, device)
    with torch.inference_mode():
        eng = table_engine(ref, decoder, c2_grammar(), 1, SINGLE_FRAMES)
        mem = torch.from_numpy(memory_array(SINGLE_FRAMES, CONFIG.width, MEMORY_SEED)).to(device)

        def song():
            eng.load(0, mem, [SOS, OUT], None, SINGLE_FRAMES)
            set_target(eng, 0, SINGLE_TOKENS)
            eng.run(SINGLE_TOKENS)
            assert eng.finished() == [0]
            eng.take(0)
            return SINGLE_TOKENS

        t0 = time.perf_counter()
        song()  # captures the bucket graphs
        capture_s = time.perf_counter() - t0
        ms, n = timed(song)
        out["single"] = {"value": n / (ms / 1000.0), "unit": "tokens/s", "ms_per_token": ms / n,
                         "ms_per_step": ms, "warmup_s": capture_s, "config": single_config(1)["workload"]}
        del eng
        torch.cuda.empty_cache()

        eng = table_engine(ref, decoder, c2_grammar(), BATCH, BATCH_FRAMES)
        rng = np.random.default_rng(1000)
        gen = torch.Generator(device=device)
        gen.manual_seed(MEMORY_SEED)
        pool = [torch.randn(1, BATCH_FRAMES, CONFIG.width, generator=gen, device=device) for _ in range(4)]
        start_pos = [1] * BATCH
        count = [0]

        def load(slot):
            frames, target = int(rng.integers(600, BATCH_FRAMES + 1)), int(rng.integers(512, 4097))
            memory = torch.zeros_like(pool[0])
            memory[:, :frames] = pool[count[0] % 4][:, :frames]
            count[0] += 1
            eng.load(slot, memory, [SOS, OUT], None, frames)
            set_target(eng, slot, target)
            start_pos[slot] = 1

        def bench_step():
            tokens = 0
            for _ in range(2):
                eng.run(32)
                done = eng.finished()
                pos = eng.state["position"].tolist()
                for slot in done:
                    tokens += pos[slot] - start_pos[slot]
                    eng.take(slot)
                    load(slot)
            pos = eng.state["position"].tolist()
            tokens += sum(p - s for p, s in zip(pos, start_pos))
            start_pos[:] = pos
            return tokens

        for slot in range(BATCH):
            load(slot)
        t0 = time.perf_counter()
        for _ in range(2):  # warm-up: graphs of the buckets these positions reach
            bench_step()
        warm_s = time.perf_counter() - t0
        total_ms, total_tokens, steps = 0.0, 0, 0
        while steps < 2 or (total_ms < seconds * 1000.0 * 0.25 and steps < 8):
            ms, n = timed(bench_step)
            total_ms, total_tokens, steps = total_ms + ms, total_tokens + n, steps + 1
        out["batched"] = {"value": total_tokens / (total_ms / 1000.0), "unit": "tokens/s", "steps": steps,
                          "ms_per_step": total_ms / steps, "warmup_s": warm_s,
                          "config": "64 slots with refill, frames U[600,3000], targets U[512,4096], "
                                    "bench step = 64 decode steps"}
        del eng
        torch.cuda.empty_cache()
    return out


def run_prefill(args):
    """One GPU: ``load`` of a single-song window (12L d1024, 1,500 frames, memory on the device)
    with an ``args.prefill``-token prefix, timed with CUDA events (the case the prefill profiles
    capture)."""

    import torch

    from sheetsage2_refined_b200 import BatchDecoder
    from sheetsage2_refined_b200.weights import memory_array

    device = torch.device("cuda", 0)
    flags = int(os.environ.get("S2R_ENGINE_FLAGS", "0"))
    dec = DecoderWeights(CONFIG, synthetic_state_dict(CONFIG, WEIGHT_SEED))
    eng = BatchDecoder(dec, None, batch=1, frames=SINGLE_FRAMES, grammar=c2_grammar(), device=device, flags=flags)
    mem = torch.from_numpy(memory_array(SINGLE_FRAMES, CONFIG.width, MEMORY_SEED)).to(torch.bfloat16).to(device)
    n = args.prefill
    prefix = [SOS, OUT] + np.random.default_rng(PREFIX_SEED).integers(4, CONFIG.vocab_size, n - 2).tolist()
    for _ in range(args.warmup):
        eng.load(0, mem, prefix, None, SINGLE_FRAMES, target=SINGLE_TOKENS)
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        eng.load(0, mem, prefix, None, SINGLE_FRAMES, target=SINGLE_TOKENS)
    end.record()
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / max(1, args.steps)
    print(json.dumps({"case": "prefill", "prefix_tokens": n, "ms_per_load": ms,
                      "prefill_tokens_per_s": (n - 1) / (ms / 1000.0), "flags": flags}))
    eng.close()


def run_b200(args, world, rank, local):
    import torch

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    # S2R_ENGINE_FLAGS (S2R_FLAG_* bits) lets a profiler run use plain launches
    flags = int(os.environ.get("S2R_ENGINE_FLAGS", "0"))
    gpu_index = local
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        try:
            gpu_index = int(visible.split(",")[local])
        except (ValueError, IndexError):
            pass

    K, W = args.steps, args.warmup
    # (factory, timed steps, warm-up steps, e2e steps) per workload; the headline keeps K and W
    plans = {
        "single": (lambda: SingleSong(torch, device, rank, flags), K, W, max(1, K // 2)),
        "batched": (lambda: Batched(torch, device, rank, flags), max(3, min(K, 10)), max(3, W), 3),
        "box": (lambda: Box(torch, device, rank, flags, world), 1, max(3, W), 1),
        "real_b1": (lambda: RealSong(torch, device, rank, flags), max(3, min(K, 10)), max(3, W), 3),
        "real_b64": (lambda: RealBatched(torch, device, rank, flags), max(3, min(K, 10)), max(3, W), 3),
        "long": (lambda: LongContext(torch, device, rank, flags), K, W, max(1, K // 2)),
    }
    names = {"all": ["single", "batched", "box", "real_b1", "real_b64"], "real": ["real_b1", "real_b64"]}.get(
        args.workload, [args.workload])
    results, load_info = {}, None
    for name in names:
        factory, steps, warmup, e2e_steps = plans[name]
        work = factory()
        results[name] = measure(work, args, steps, warmup, e2e_steps, world, device, gpu_index, torch)
        if name == "single":
            load_info = work.time_load()
        work.eng.close()
        del work
        torch.cuda.synchronize(device)
        torch.cuda.empty_cache()

    cpu = None
    if world == 1 and not args.no_cpu:
        cpu_dec = CpuDecoder()
        v, n, cores, _ = cpu_dec.sample(seconds=args.cpu_seconds)
        one, one_n, _, _ = cpu_dec.sample(seconds=max(2.0, args.cpu_seconds / 4), min_tokens=2, threads=1)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": cpu_dec.kind,
               "sample": f"{n} greedy tokens of the single-song workload from position 1 (load excluded), "
                         + cpu_dec.describe() + ", all host cores",
               "one_thread": {"value": one, "tokens": one_n}}
    ref_gpu = None
    if world == 1 and not args.no_reference_gpu and args.workload in ("all", "single", "batched"):
        try:
            ref_gpu = reference_gpu(torch, device)
        except Exception as exc:  # noqa: BLE001 - reported, never fatal for this arm
            ref_gpu = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
        for key in ("single", "batched"):
            if ref_gpu and key in ref_gpu and key in results:
                ref_gpu[key]["this_arm_over_reference"] = results[key]["value"] / ref_gpu[key]["value"]

    if rank == 0:
        head_name = names[0]
        head = results[head_name]
        line = {
            "metric": METRIC, "value": head["value"], "unit": "tokens/s", "n_gpus": world, "steps": head["steps"],
            "warmup": head["warmup"], "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": head["scaling"], "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {**head["config"], **({"profiling_overrides": OVERRIDES} if OVERRIDES else {})},
            "e2e": {k: v for k, v in head["e2e"].items() if k != "steps"},
            "gpu_launches": head["gpu_launches"],
            "clocks": head["clocks"],
            "roofline": head["roofline"],
            "step_roofline": head["step_roofline"],
            "kernel_classes": head["kernel_classes"],
            "cpu_baseline": cpu,
        }
        if load_info is not None:
            line["load"] = load_info
        others = {k: v for k, v in results.items() if k != head_name}
        if others:
            line["workloads"] = others
        if ref_gpu is not None:
            line["reference_gpu"] = ref_gpu
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--workload", default="all", choices=("all", "single", "batched", "box", "long", "real",
                                                           "real_b1", "real_b64"))
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true", help="skip timing the reference's own CUDA path")
    # smaller cases of the same kernels for ncu captures that must fit a few GB (not bench lines)
    ap.add_argument("--layers", type=int, default=None, help="override the decoder depth (profiling cases)")
    ap.add_argument("--max-tokens", type=int, default=None, help="override the context length (profiling cases)")
    ap.add_argument("--batch-frames", type=int, default=None, help="override the batched frames cap (profiling cases)")
    ap.add_argument("--prefill", type=int, default=None, metavar="TOKENS",
                    help="profiling case: only `load` a single-song window with a prefix of TOKENS tokens, "
                         "--warmup + --steps times, and print its prefill rate (not a bench line)")
    args = ap.parse_args()
    global CONFIG, REAL, BATCH_FRAMES, OVERRIDES
    if args.layers or args.max_tokens:
        CONFIG = dataclasses.replace(CONFIG, layers=args.layers or CONFIG.layers,
                                     max_tokens=args.max_tokens or CONFIG.max_tokens)
        REAL = dataclasses.replace(REAL, layers=args.layers or REAL.layers)
        OVERRIDES.update(layers=CONFIG.layers, max_tokens=CONFIG.max_tokens)
    if args.batch_frames:
        BATCH_FRAMES = args.batch_frames
        OVERRIDES.update(batch_frames=BATCH_FRAMES)
    world, rank, local = dist_env()
    if args.prefill:
        run_prefill(args)
        return
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_b200(args, world, rank, local)


if __name__ == "__main__":
    main()
