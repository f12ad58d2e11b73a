"""Generate the golden fixtures of this directory by running the reference itself.

Run where the reference package is importable from a checkout or an
install directory (read only), given as the first argument or as
``S2R_REFERENCE``::

    python tests/golden/make_golden.py /path/to/reference [fixture ...]

With fixture names (``trace c1 batch real c2 rescore real_full``) only those
files are rewritten.

The reference package is imported from that checkout with a stub for
``soundfile`` (only ``transcribe.load_waveform`` uses it).  Its CPU path is
float32 and eager (``engine.py:69-70,244-245``), so the files hold the
reference's own float32 results: greedy tokens and end reasons from
``BatchDecoder`` and teacher-forced logits from ``TokenDecoder.forward``.
For the synthetic vocabularies a table grammar (the rule documented in
``sheetsage2_refined_b200.grammar.TableGrammar``) is put into the reference
engine through its grammar duck type (``engine.grammar`` and extra state).

Files:

* ``c1_table.npz``      — 2L/d256/V512 decoder, one slot, 128 greedy steps.
* ``c2_head.npz``       — 12L/d1024/V2048 decoder, F=1500, first 128 steps.
* ``batch_table.npz``   — three slots with prefill, masking, limit, refill.
* ``real_grammar.npz``  — real 32,576-token vocabulary and ``TokenGrammar``,
  two prompt sets, stop seconds and a mode bias.
* ``grammar_trace.npz`` — ``TokenGrammar`` state after every token of seeded
  random walks through the allowed tokens (EOS included), per prompt set.
* ``rescore.npz``       — real vocabulary with every frame-head rescoring
  term switched on: seeded per-frame tables, two slots (one with a prefix
  that states a time, a meter and a key), greedy tokens and end reasons.
* ``real_full.npz``     — the product decoder shape (6L/d512/8 heads/FFN 2048,
  32,576 tokens, 7,500 frames) with the real grammar, the mode bias or the
  key terms, and frame-head rescoring: per case and slot the greedy tokens of
  160 steps, the top 8 (value, token) of the masked logits the reference's
  argmax saw at every step, and teacher-forced logits of the first 64 steps
  at 1,024 seeded vocabulary columns.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests"))
sys.modules.setdefault("soundfile", types.ModuleType("soundfile"))
_ARGS = [a for a in sys.argv[1:] if "/" in a or Path(a).is_dir()]
REFERENCE = _ARGS[0] if _ARGS else os.environ.get("S2R_REFERENCE")
if not REFERENCE:
    sys.exit("make_golden.py: give the reference package's directory (argument or S2R_REFERENCE)")

import scenarios as sc  # noqa: E402
from reference_path import load_reference  # noqa: E402
from reference_path import ref_decoder as _ref_decoder  # noqa: E402
from reference_path import table_engine as _table_engine  # noqa: E402
from sheetsage2_refined_b200.weights import memory_array  # noqa: E402

REF = load_reference(REFERENCE)
if REF is None:
    sys.exit(f"make_golden.py: no sheetsage2_refined package under {REFERENCE}")
BatchDecoder = REF.engine.BatchDecoder
TokenGrammar = REF.grammar.TokenGrammar
Vocab = REF.vocab.Vocab


def ref_decoder(config, seed):
    return _ref_decoder(REF, config, seed)


def table_engine(decoder, desc, batch, frames):
    return _table_engine(REF, decoder, desc, batch, frames)


def ref_loader(engine, width, frames_engine):
    def load(slot, memory_seed, prefix, stop, frames, target):
        memory = torch.from_numpy(memory_array(frames_engine, width, memory_seed))
        engine.load(slot, memory, prefix, stop, frames)
        if target is not None:
            engine.state["target"][slot] = target
    return load


def teacher_forced(decoder, memory_seed, frames_engine, frames, tokens, first):
    """Logits predicting ``tokens[first+1:]`` from the full prefix (decoder.py:98-151)."""

    memory = torch.from_numpy(memory_array(frames_engine, decoder.config.width, memory_seed))
    cache = decoder.new_cache(memory, torch.tensor([frames]))
    logits = decoder(torch.tensor([tokens[:-1]]), cache)[0]
    return logits[first:].numpy().astype(np.float32)


@torch.no_grad()
def make_single(name, config, seed, desc, memory_seed, frames, steps):
    decoder = ref_decoder(config, seed)
    engine = table_engine(decoder, desc, 1, frames)
    tokens, ended = sc.single(engine, ref_loader(engine, config.width, frames), steps, memory_seed, frames,
                              target=steps)
    logits = teacher_forced(decoder, memory_seed, frames, frames, tokens[: steps + 2], 1)
    np.savez_compressed(HERE / name, tokens=np.array(tokens), ended=np.array(ended), logits=logits)
    print(name, len(tokens), ended, logits.shape)


@torch.no_grad()
def make_batch():
    decoder = ref_decoder(sc.C1_SHORT, sc.BATCH_SEED)
    engine = table_engine(decoder, sc.batch_grammar(), 3, sc.BATCH_FRAMES)
    taken = sc.continuous_batch(engine, ref_loader(engine, sc.C1_SHORT.width, sc.BATCH_FRAMES))
    slots = np.array([s for s, _, _ in taken])
    ended = np.array([e for _, _, e in taken])
    lengths = np.array([len(t) for _, t, _ in taken])
    flat = np.concatenate([np.array(t) for _, t, _ in taken])
    np.savez_compressed(HERE / "batch_table.npz", slots=slots, ended=ended, lengths=lengths, tokens=flat)
    print("batch_table", list(zip(slots.tolist(), lengths.tolist(), ended.tolist())))


def mode_bias_values():
    return [0.0, 1.5, -0.5, 2.0, 0.25, -1.0, 3.0, 0.5, -2.0]


@torch.no_grad()
def make_real():
    vocab = Vocab()
    decoder = ref_decoder(sc.REAL_TINY, sc.REAL_SEED)
    out = {}
    for i, prompts in enumerate(sc.REAL_PROMPT_SETS):
        bias = mode_bias_values() if "key_mode" in prompts else None
        engine = BatchDecoder(decoder, vocab, batch=2, frames=sc.REAL_FRAMES, prompts=prompts, mode_bias=bias)
        prefix = vocab.prompt_prefix(prompts)
        load = ref_loader(engine, sc.REAL_TINY.width, sc.REAL_FRAMES)
        load(0, 31 + i, prefix, 2.5, sc.REAL_FRAMES, None)
        load(1, 41 + i, prefix + [vocab.start["shift"] + 3], None, 50, None)
        for _ in range(40):
            engine.run(5)
            if len(engine.finished()) == 2:
                break
        for slot in (0, 1):
            finished = bool(engine.state["finished"][slot])
            length = int(engine.state["position"][slot]) + 1
            out[f"p{i}_s{slot}_tokens"] = engine.out[slot, :length].numpy().copy()
            out[f"p{i}_s{slot}_ended"] = np.array(int(engine.state["ended"][slot]))
            out[f"p{i}_s{slot}_finished"] = np.array(finished)
            print("real", i, slot, length, finished, int(engine.state["ended"][slot]))
    np.savez_compressed(HERE / "real_grammar.npz", **out)


@torch.no_grad()
def make_rescore():
    vocab = Vocab()
    decoder = ref_decoder(sc.REAL_TINY, sc.REAL_SEED)
    out = {}
    for case, weights in sc.RESCORE_CASES.items():
        engine = BatchDecoder(decoder, vocab, batch=2, frames=sc.REAL_FRAMES, prompts=sc.RESCORE_PROMPTS,
                              frame_weight=weights)
        for slot, (prefix, stop, frames, rows, seed) in enumerate(sc.rescore_windows(vocab)):
            tables = {k: torch.from_numpy(v) for k, v in sc.rescore_tables(rows, seed).items()}
            memory = torch.from_numpy(memory_array(sc.REAL_FRAMES, sc.REAL_TINY.width, 61 + slot))
            engine.load(slot, memory, prefix, stop, frames, frame_logp=tables)
        for _ in range(60):
            engine.run(4)
            if len(engine.finished()) == 2:
                break
        for slot in (0, 1):
            length = int(engine.state["position"][slot]) + 1
            out[f"{case}_s{slot}_tokens"] = engine.out[slot, :length].numpy().copy()
            out[f"{case}_s{slot}_ended"] = np.array(int(engine.state["ended"][slot]))
            out[f"{case}_s{slot}_finished"] = np.array(bool(engine.state["finished"][slot]))
            print("rescore", case, slot, length, bool(engine.state["finished"][slot]), int(engine.state["ended"][slot]))
    np.savez_compressed(HERE / "rescore.npz", **out)


@torch.no_grad()
def make_trace():
    vocab = Vocab()
    out = {}
    names = ("in_shift", "shift_run", "payload", "last_field", "incomplete", "finished", "ended")
    for i, prompts in enumerate(sc.REAL_PROMPT_SETS):
        grammar = TokenGrammar(vocab, "cpu", prompts)
        rng = np.random.default_rng(1000 + i)
        state = TokenGrammar.new_state(1, "cpu")
        stop = torch.tensor([120.0], dtype=torch.float64)
        tokens, states, masks = [], [], []
        for step in range(600):
            allowed = grammar.allowed(state)[0].numpy()
            masks.append(np.packbits(allowed))
            choices = np.nonzero(allowed)[0]
            eos_ok = allowed[2]
            if eos_ok and rng.random() < 0.02:
                token = 2
            else:
                # prefer non-time tokens so that events get several fields
                non_time = choices[(choices < vocab.start["time"]) | (choices >= vocab.end["time"])]
                pool = non_time if len(non_time) and rng.random() < 0.8 else choices
                token = int(rng.choice(pool))
            at_limit = torch.tensor([step == 599])
            grammar.update(state, torch.tensor([token]), torch.tensor([True]), stop, at_limit)
            tokens.append(token)
            states.append([int(state[n][0]) for n in names])
            if bool(state["finished"][0]):
                state = TokenGrammar.new_state(1, "cpu")
        out[f"p{i}_tokens"] = np.array(tokens)
        out[f"p{i}_states"] = np.array(states)
        out[f"p{i}_masks"] = np.stack(masks)
        prefix = vocab.prompt_prefix(prompts) + tokens[:25]
        ps = grammar.prefix_state(prefix, prefix.index(3), "cpu")
        out[f"p{i}_prefix_state"] = np.array([int(ps[n][0]) for n in names])
    np.savez_compressed(HERE / "grammar_trace.npz", **out)
    print("grammar_trace written")


class ArgmaxTap(torch.overrides.TorchFunctionMode):
    """Records the input of every ``[rows, vocab]`` argmax: the reference engine's masked logits
    (engine.py:350), as its CPU path evaluates them eagerly."""

    def __init__(self, vocab_size):
        super().__init__()
        self.vocab_size, self.seen = vocab_size, []

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func in (torch.Tensor.argmax, torch.argmax) and args and args[0].dim() == 2 \
                and args[0].shape[-1] == self.vocab_size:
            self.seen.append(args[0].detach().clone())
        return func(*args, **kwargs)


@torch.no_grad()
def make_real_full():
    vocab = Vocab()
    decoder = ref_decoder(sc.REAL, sc.REAL_FULL_SEED)
    cols = sc.real_logit_columns(vocab.size)
    out = {"columns": cols}
    for case, spec in sc.REAL_CASES.items():
        engine = BatchDecoder(decoder, vocab, batch=2, frames=sc.REAL_FULL_FRAMES, prompts=spec["prompts"],
                              mode_bias=spec["mode_bias"], frame_weight=spec["frame_weight"])
        windows = sc.real_windows(vocab, case)
        for slot, (seed, prefix, stop, frames, rows, table_seed) in enumerate(windows):
            tables = {k: torch.from_numpy(v) for k, v in sc.rescore_tables(rows, table_seed).items()}
            memory = torch.from_numpy(memory_array(sc.REAL_FULL_FRAMES, sc.REAL.width, seed))
            engine.load(slot, memory, prefix, stop, frames, frame_logp=tables)
        tap = ArgmaxTap(vocab.size)
        steps = 0
        with tap:
            for _ in range(sc.REAL_STEPS):
                engine.run(1)
                steps += 1
                if len(engine.finished()) == 2:
                    break
        masked = torch.stack(tap.seen)  # [steps, 2, vocab]
        assert masked.shape[0] == steps, (masked.shape, steps)
        top = torch.topk(masked, 8, dim=-1)
        for slot, (seed, prefix, stop, frames, rows, table_seed) in enumerate(windows):
            length = int(engine.state["position"][slot]) + 1
            tokens = engine.out[slot, :length].numpy().copy()
            out[f"{case}_s{slot}_tokens"] = tokens
            out[f"{case}_s{slot}_ended"] = np.array(int(engine.state["ended"][slot]))
            out[f"{case}_s{slot}_top_values"] = top.values[:, slot].numpy().astype(np.float32)
            out[f"{case}_s{slot}_top_tokens"] = top.indices[:, slot].numpy().astype(np.int32)
            n = len(prefix)
            forced = min(sc.REAL_LOGIT_STEPS, length - n)
            logits = teacher_forced(decoder, seed, sc.REAL_FULL_FRAMES, frames, tokens[: n + forced].tolist(), n - 1)
            out[f"{case}_s{slot}_logits"] = logits[:, cols]
            print("real_full", case, slot, length, int(engine.state["ended"][slot]), logits.shape)
    np.savez_compressed(HERE / "real_full.npz", **out)


FIXTURES = {
    "trace": make_trace,
    "c1": lambda: make_single("c1_table.npz", sc.C1, sc.C1_SEED, sc.c1_grammar(), sc.C1_MEMORY_SEED, sc.C1_FRAMES,
                              sc.C1_STEPS),
    "batch": make_batch,
    "real": make_real,
    "c2": lambda: make_single("c2_head.npz", sc.C2, sc.C2_SEED, sc.c2_grammar(), sc.C2_MEMORY_SEED, sc.C2_FRAMES, 128),
    "rescore": make_rescore,
    "real_full": make_real_full,
}


if __name__ == "__main__":
    torch.manual_seed(0)
    chosen = [a for a in sys.argv[1:] if a in FIXTURES] or list(FIXTURES)
    for name in chosen:
        FIXTURES[name]()
