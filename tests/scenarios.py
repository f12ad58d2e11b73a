"""Decode scenarios shared by the golden generator and the parity tests.

Each scenario drives an engine through the reference engine's public surface
(``load / run / finished / take``, ``sheetsage2_refined/engine.py:176-262``),
so the same protocol runs on the reference ``BatchDecoder`` (golden files),
on the numpy oracle and on the CUDA engine.  ``load`` is passed in as a
callable ``load(slot, memory_seed, prefix, stop_seconds, frames, target)``
because the three engines take the memory tensor and the table-grammar
target differently.
"""

from __future__ import annotations

from sheetsage2_refined_b200.grammar import TableGrammar
from sheetsage2_refined_b200.vocab_table import FULL_PROMPTS, OUT, SOS
from sheetsage2_refined_b200.weights import DecoderConfig

# Workload shapes (seeds fixed here; the golden files were made with them).
C1 = DecoderConfig(vocab_size=512, width=256, layers=2, heads=4, ffn_width=1024, max_tokens=5120)
C1_SHORT = DecoderConfig(vocab_size=512, width=256, layers=2, heads=4, ffn_width=1024, max_tokens=256)
C2 = DecoderConfig(vocab_size=2048, width=1024, layers=12, heads=16, ffn_width=4096, max_tokens=5120)
REAL_TINY = DecoderConfig(vocab_size=32576, width=128, layers=2, heads=2, ffn_width=256, max_tokens=5120)
# The product decoder's shape (decoder.py:12-21 with the real vocabulary, model.py:22) and its
# 300 s window of 7,500 encoder frames (model.py:15, encoder.py:37-39).
REAL = DecoderConfig(vocab_size=32576, width=512, layers=6, heads=8, ffn_width=2048, max_tokens=5120)
REAL_FULL_SEED, REAL_FULL_FRAMES, REAL_STEPS, REAL_LOGIT_STEPS = 6, 7500, 160, 64

C1_SEED, C1_MEMORY_SEED, C1_GRAMMAR_SEED, C1_FRAMES, C1_STEPS = 0, 100, 7, 256, 128
C2_SEED, C2_MEMORY_SEED, C2_GRAMMAR_SEED, C2_FRAMES = 1, 101, 8, 1500
BATCH_SEED, BATCH_GRAMMAR_SEED, BATCH_FRAMES = 3, 9, 256
REAL_SEED, REAL_FRAMES = 5, 64


def c1_grammar() -> TableGrammar:
    return TableGrammar(C1.vocab_size, states=8, density=0.25, seed=C1_GRAMMAR_SEED)


def c2_grammar() -> TableGrammar:
    return TableGrammar(C2.vocab_size, states=8, density=0.25, seed=C2_GRAMMAR_SEED)


def batch_grammar() -> TableGrammar:
    return TableGrammar(C1_SHORT.vocab_size, states=8, density=0.25, seed=BATCH_GRAMMAR_SEED)


def single(engine, load, steps: int, memory_seed: int, frames: int, prefix=(SOS, OUT), target=None, stop=None):
    """One slot, ``steps`` steps: the workload of a single-song decode."""

    load(0, memory_seed, list(prefix), stop, frames, target)
    engine.run(steps)
    return engine.take(0)


def continuous_batch(engine, load) -> list[tuple[int, list[int], str]]:
    """Three slots that start, end and are refilled at different steps.

    Covers the prefix prefill (a prefix with tokens after ``<out>``), masked
    cross-attention (real frames below the engine's), the context limit
    (slot 1 runs into ``max_tokens``), a slot loaded mid-run and a slot
    refilled after ``take``.  Returns ``(slot, tokens, ended)`` in take order.
    """

    taken = []
    load(0, 11, [SOS, OUT], None, 256, 40)
    load(1, 12, [SOS, 5, OUT, 17, 200, 301], None, 100, 10_000)
    engine.run(10)
    load(2, 13, [SOS, OUT, 9], None, 37, 25)
    refilled = False
    for _ in range(64):
        engine.run(8)
        for slot in engine.finished():
            tokens, ended = engine.take(slot)
            taken.append((slot, tokens, ended))
            if slot == 0 and not refilled:
                load(0, 14, [SOS, OUT], None, 200, 30)
                refilled = True
        if refilled and not any(engine.loaded):
            break
    return taken


REAL_PROMPT_SETS = (
    FULL_PROMPTS,
    ("timestamp", "downbeat_meter", "chord_detail", "key_mode", "melody_vocal"),
)


# Frame-head rescoring: a prompt set that emits every rescored span (chord
# detail, key, downbeat/meter) and two weight sets -- chord and key terms,
# then meter and downbeat terms -- with seeded per-frame tables shaped as
# transcribe.frame_tables makes them.
RESCORE_PROMPTS = ("timestamp", "downbeat_meter", "key", "chord_detail")
RESCORE_CASES = {
    "chords": {"root": 0.5, "bass": 0.4, "detail": 0.3, "quality": 0.3, "key": 0.5, "key_boundary": 0.6},
    "meters": {"downbeat": 2.0, "meter": 2.0, "key_boundary": 0.6},
}


def rescore_tables(rows: int, seed: int) -> dict:
    """Seeded per-frame tables of every term, ``[rows, width]`` (``[rows]`` for the scalar terms).

    Scores ~N(0, 3) rather than normalised log-probabilities, so that the
    rescored spans outscore the rest of the vocabulary under random weights
    and every term decides tokens; the meter table prefers long bars (16+
    beats) so that meter changes happen.
    """

    import numpy as np

    rng = np.random.default_rng(seed)
    widths = {"root": 12, "bass": 12, "detail": 744, "quality": 744, "key": 24, "key_boundary": 0, "downbeat": 0,
              "meter": 16}
    tables = {name: (rng.standard_normal((rows, w) if w else rows) * 3.0).astype(np.float32)
              for name, w in widths.items()}
    tables["meter"][:, 15] += 6.0
    return tables


def rescore_windows(vocab):
    """(prefix, stop_seconds, frames, table rows, table seed) per slot.

    Slot 1's prefix states a time (1.5 s), a 4/4 meter, bar position 0 and a
    key, so the rescoring state starts from the prefix (engine.py:225-232).
    """

    prefix = vocab.prompt_prefix(RESCORE_PROMPTS)
    stated = prefix + [vocab.start["time"] + 150, vocab.start["meter"] + 3 * 6 + 2, vocab.start["eighth_position"],
                       vocab.start["key"] + 5]
    return [(prefix, None, REAL_FRAMES, REAL_FRAMES, 71), (stated, None, 50, 40, 72)]


def rescore_forced(engine, vocab, golden: dict, case: str, load, masks: list | None = None) -> list[tuple[int, int, int]]:
    """Force the reference's greedy tokens of a rescoring case through ``engine``.

    Loads both windows of the case with their frame tables (``load(slot,
    memory_seed, prefix, stop, frames, frame_logp)``), then at every step
    forces each slot's next reference token and records ``(slot, engine's
    greedy choice, reference's choice)`` while the slot is running.  With
    ``masks`` (an oracle engine only) the masked logits of every recorded
    choice are appended to it as well.
    """

    import numpy as np

    windows = rescore_windows(vocab)
    seqs = [golden[f"{case}_s{slot}_tokens"].tolist() for slot in (0, 1)]
    for slot, (prefix, stop, frames, rows, seed) in enumerate(windows):
        load(slot, 61 + slot, prefix, stop, frames, rescore_tables(rows, seed))
    starts = [len(w[0]) for w in windows]
    steps = max(len(s) - p for s, p in zip(seqs, starts))
    record = []
    for k in range(steps):
        forced = np.full(getattr(engine, "batch", 2), -1, np.int64)
        live = []
        for slot in (0, 1):
            if starts[slot] + k < len(seqs[slot]):
                forced[slot] = seqs[slot][starts[slot] + k]
                live.append(slot)
        _, greedy = engine.step_debug(forced, want_logits=False) if hasattr(engine, "step_debug") else \
            engine.step(forced=forced)
        for slot in live:
            record.append((slot, int(greedy[slot]), int(forced[slot])))
            if masks is not None:
                masks.append(engine.last_masked[slot].copy())
    return record


# Product-shape cases: the real vocabulary and TokenGrammar, mode bias or the key terms, and the
# frame-head rescoring terms each prompt set can use (engine.py:29-38: key and key_mode share a
# prompt group, so the key terms and the mode bias never meet).
REAL_CASES = {
    "mode": {"prompts": ("timestamp", "downbeat_meter", "chord_detail", "key_mode", "melody_full"),
             "mode_bias": [0.0, 1.5, -0.5, 2.0, 0.25, -1.0, 3.0, 0.5, -2.0],
             "frame_weight": {"root": 0.5, "bass": 0.4, "detail": 0.3, "quality": 0.3, "downbeat": 2.0,
                              "meter": 2.0}},
    "key": {"prompts": ("timestamp", "downbeat_meter", "key", "chord_detail", "melody_full"),
            "mode_bias": None,
            "frame_weight": {"root": 0.5, "bass": 0.4, "detail": 0.3, "quality": 0.3, "key": 0.5,
                             "key_boundary": 0.6, "downbeat": 2.0, "meter": 2.0}},
}

# Columns of the teacher-forced logits kept in the product-shape fixture (the full rows would be
# 130 KB each): a seeded sample of the vocabulary.
REAL_LOGIT_COLUMNS = 1024


def real_logit_columns(vocab_size: int):
    import numpy as np

    return np.sort(np.random.default_rng(77).choice(vocab_size, REAL_LOGIT_COLUMNS, replace=False))


def real_windows(vocab, case: str):
    """(memory seed, prefix, stop seconds, real frames, table rows, table seed) of the case's two slots.

    Slot 0 starts from the prompt prefix and sees every frame; slot 1's prefix
    states a time, a meter, bar position 0 and a key (or key-and-mode) token,
    and it sees 6,000 of the 7,500 frames.
    """

    prompts = REAL_CASES[case]["prompts"]
    prefix = vocab.prompt_prefix(prompts)
    key = vocab.start["key"] + 5 if "key" in prompts else vocab.start["key_mode"] + 17
    stated = prefix + [vocab.start["time"] + 150, vocab.start["meter"] + 3 * 6 + 2, vocab.start["eighth_position"], key]
    return [(201, prefix, None, REAL_FULL_FRAMES, REAL_FULL_FRAMES, 81),
            (202, stated, None, 6000, 5000, 82)]


def real_forced(engine, vocab, golden: dict, case: str, load, masks: list | None = None,
                logits: list | None = None) -> list[tuple[int, int, int, int]]:
    """Force the reference's greedy tokens of a product-shape case through ``engine``.

    Loads both windows of the case with their frame tables (``load(slot,
    memory_seed, prefix, stop, frames, frame_logp)``), then at every step
    forces each slot's next reference token and records ``(slot, step,
    engine's greedy choice, reference's choice)`` while the slot has
    reference tokens left.  ``masks`` (an oracle engine only) receives the
    masked logits of every record; ``logits`` receives ``(slot, step, raw
    logits row)`` of every record.
    """

    import numpy as np

    windows = real_windows(vocab, case)
    seqs = [golden[f"{case}_s{slot}_tokens"].tolist() for slot in (0, 1)]
    for slot, (seed, prefix, stop, frames, rows, table_seed) in enumerate(windows):
        load(slot, seed, prefix, stop, frames, rescore_tables(rows, table_seed))
    starts = [len(w[1]) for w in windows]
    steps = max(len(s) - p for s, p in zip(seqs, starts))
    record = []
    for k in range(steps):
        forced = np.full(getattr(engine, "batch", 2), -1, np.int64)
        live = [slot for slot in (0, 1) if starts[slot] + k < len(seqs[slot])]
        for slot in live:
            forced[slot] = seqs[slot][starts[slot] + k]
        if hasattr(engine, "step_debug"):
            raw, greedy = engine.step_debug(forced, want_logits=logits is not None)
        else:
            raw, greedy = engine.step(forced=forced)
        for slot in live:
            record.append((slot, k, int(greedy[slot]), int(forced[slot])))
            if masks is not None:
                masks.append(engine.last_masked[slot].copy())
            if logits is not None:
                logits.append((slot, k, raw[slot].copy()))
    return record
