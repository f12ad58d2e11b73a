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
