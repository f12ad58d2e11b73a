"""Pin the numpy oracle against the reference's own outputs (golden files).

The golden files were produced by ``tests/golden/make_golden.py``, which runs
the reference ``BatchDecoder`` / ``TokenDecoder`` / ``TokenGrammar`` on CPU
(float32).  The oracle's ``fp32`` mode must reproduce them: greedy tokens and
grammar states bit-exactly, logits within 1e-4 (float32 summation order).
The ``bf16`` mode (the reference's CUDA numerics) must stay within the
parity tolerance of 2e-2 of the float32 logits.
"""

from pathlib import Path

import numpy as np
import pytest

import scenarios as sc
from oracle.engine import OracleEngine
from oracle.grammar import ClassGrammarOracle
from sheetsage2_refined_b200.grammar import ClassGrammar
from sheetsage2_refined_b200.vocab_table import VocabTable
from sheetsage2_refined_b200.weights import memory_array, synthetic_state_dict

GOLDEN = Path(__file__).resolve().parent / "golden"
LOGIT_TOL_FP32 = 1e-4
LOGIT_TOL_BF16 = 2e-2  # parity tolerance for teacher-forced bf16 logits


def oracle_loader(engine, width, frames_engine):
    def load(slot, memory_seed, prefix, stop, frames, target):
        engine.load(slot, memory_array(frames_engine, width, memory_seed), prefix, stop, frames, target=target)
    return load


def teacher_forced_run(engine, tokens, prefix_len, steps):
    """Run ``steps`` steps forcing ``tokens[prefix_len:]``; returns logits [steps, V] and greedy choices."""

    logits, greedy = [], []
    for k in range(steps):
        forced = np.array([tokens[prefix_len + k]])
        lg, ch = engine.step(forced=forced)
        logits.append(lg[0])
        greedy.append(int(ch[0]))
    return np.stack(logits), np.array(greedy)


def test_grammar_trace_bit_exact():
    g = np.load(GOLDEN / "grammar_trace.npz")
    vocab = VocabTable()
    names = ("in_shift", "shift_run", "payload", "last_field", "incomplete", "finished", "ended")
    for i, prompts in enumerate(sc.REAL_PROMPT_SETS):
        grammar = ClassGrammarOracle(ClassGrammar(vocab, prompts))
        state = grammar.new_state(1)
        tokens, states, masks = g[f"p{i}_tokens"], g[f"p{i}_states"], g[f"p{i}_masks"]
        for step, token in enumerate(tokens):
            allowed = grammar.allowed(state)[0]
            assert np.array_equal(np.packbits(allowed), masks[step]), (i, step)
            grammar.update(state, np.array([token]), np.array([True]), np.array([120.0]), np.array([step == 599]))
            got = [int(state[n][0]) for n in names]
            assert got == states[step].tolist(), (i, step, got, states[step])
            if state["finished"][0]:
                state = grammar.new_state(1)
        prefix = vocab.prompt_prefix(prompts) + tokens[:25].tolist()
        ps = grammar.prefix_state(prefix, prefix.index(3))
        assert [int(ps[n][0]) for n in names] == g[f"p{i}_prefix_state"].tolist()


def test_trace_covers_every_end_reason_and_class():
    g = np.load(GOLDEN / "grammar_trace.npz")
    ended = np.concatenate([g[f"p{i}_states"][:, 6] for i in range(len(sc.REAL_PROMPT_SETS))])
    assert {1, 2, 3} <= set(ended.tolist())  # eos, stop and limit all occur


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_c1_single_slot(mode):
    g = np.load(GOLDEN / "c1_table.npz")
    engine = OracleEngine(sc.C1, synthetic_state_dict(sc.C1, sc.C1_SEED), sc.c1_grammar(), batch=1,
                          frames=sc.C1_FRAMES, mode=mode)
    tokens = g["tokens"].tolist()
    if mode == "fp32":
        got, ended = sc.single(engine, oracle_loader(engine, sc.C1.width, sc.C1_FRAMES), sc.C1_STEPS,
                               sc.C1_MEMORY_SEED, sc.C1_FRAMES, target=sc.C1_STEPS)
        assert got == tokens and ended == str(g["ended"])
    engine2 = OracleEngine(sc.C1, synthetic_state_dict(sc.C1, sc.C1_SEED), sc.c1_grammar(), batch=1,
                           frames=sc.C1_FRAMES, mode=mode)
    oracle_loader(engine2, sc.C1.width, sc.C1_FRAMES)(0, sc.C1_MEMORY_SEED, tokens[:2], None, sc.C1_FRAMES,
                                                       sc.C1_STEPS)
    logits, greedy = teacher_forced_run(engine2, tokens, 2, sc.C1_STEPS)
    err = np.abs(logits - g["logits"]).max()
    assert err <= (LOGIT_TOL_FP32 if mode == "fp32" else LOGIT_TOL_BF16), err
    same = (greedy == np.array(tokens[2 : 2 + sc.C1_STEPS])).mean()
    assert same >= (1.0 if mode == "fp32" else 0.98), same


def test_continuous_batch_fp32():
    g = np.load(GOLDEN / "batch_table.npz")
    engine = OracleEngine(sc.C1_SHORT, synthetic_state_dict(sc.C1_SHORT, sc.BATCH_SEED), sc.batch_grammar(),
                          batch=3, frames=sc.BATCH_FRAMES, mode="fp32")
    taken = sc.continuous_batch(engine, oracle_loader(engine, sc.C1_SHORT.width, sc.BATCH_FRAMES))
    assert [s for s, _, _ in taken] == g["slots"].tolist()
    assert [e for _, _, e in taken] == g["ended"].tolist()
    assert [len(t) for _, t, _ in taken] == g["lengths"].tolist()
    assert np.concatenate([np.array(t) for _, t, _ in taken]).tolist() == g["tokens"].tolist()


def real_grammar_run(mode):
    from sheetsage2_refined_b200.vocab_table import NO_KEY

    vocab = VocabTable()
    sd = synthetic_state_dict(sc.REAL_TINY, sc.REAL_SEED)
    results = {}
    for i, prompts in enumerate(sc.REAL_PROMPT_SETS):
        bias = None
        if "key_mode" in prompts:
            bias = np.zeros(vocab.size, np.float32)
            start = vocab.start["key_mode"]
            bias[start : start + NO_KEY] = np.repeat(np.array(
                [0.0, 1.5, -0.5, 2.0, 0.25, -1.0, 3.0, 0.5, -2.0], np.float32), 12)
        engine = OracleEngine(sc.REAL_TINY, sd, ClassGrammar(vocab, prompts), batch=2, frames=sc.REAL_FRAMES,
                              mode=mode, logit_bias=bias)
        prefix = vocab.prompt_prefix(prompts)
        load = oracle_loader(engine, sc.REAL_TINY.width, sc.REAL_FRAMES)
        load(0, 31 + i, prefix, 2.5, sc.REAL_FRAMES, None)
        load(1, 41 + i, prefix + [vocab.start["shift"] + 3], None, 50, None)
        for _ in range(40):
            engine.run(5)
            if len(engine.finished()) == 2:
                break
        for slot in (0, 1):
            length = int(engine.state["position"][slot]) + 1
            results[(i, slot)] = (engine.out[slot, :length].tolist(), int(engine.state["ended"][slot]),
                                  bool(engine.state["finished"][slot]))
    return results


def test_real_grammar_fp32():
    g = np.load(GOLDEN / "real_grammar.npz")
    for (i, slot), (tokens, ended, finished) in real_grammar_run("fp32").items():
        assert tokens == g[f"p{i}_s{slot}_tokens"].tolist(), (i, slot)
        assert ended == int(g[f"p{i}_s{slot}_ended"]) and finished == bool(g[f"p{i}_s{slot}_finished"])


def test_c2_head_fp32():
    g = np.load(GOLDEN / "c2_head.npz")
    sd = synthetic_state_dict(sc.C2, sc.C2_SEED)
    engine = OracleEngine(sc.C2, sd, sc.c2_grammar(), batch=1, frames=sc.C2_FRAMES, mode="fp32")
    tokens = g["tokens"].tolist()
    steps = len(g["logits"])
    oracle_loader(engine, sc.C2.width, sc.C2_FRAMES)(0, sc.C2_MEMORY_SEED, tokens[:2], None, sc.C2_FRAMES, steps)
    logits, greedy = teacher_forced_run(engine, tokens, 2, steps)
    assert np.abs(logits - g["logits"]).max() <= LOGIT_TOL_FP32
    assert greedy.tolist() == tokens[2:2 + steps]


@pytest.mark.parametrize("case", list(sc.RESCORE_CASES))
def test_rescore_oracle_vs_reference(case):
    """Frame-head rescoring: the oracle (fp32) picks the reference's greedy token at every forced step."""

    g = np.load(GOLDEN / "rescore.npz")
    vocab = VocabTable()
    from oracle.engine import FRAME_TERM_NAMES

    weights = tuple(float(sc.RESCORE_CASES[case].get(n, 0.0)) for n in FRAME_TERM_NAMES)
    eng = OracleEngine(sc.REAL_TINY, synthetic_state_dict(sc.REAL_TINY, sc.REAL_SEED),
                       ClassGrammar(vocab, sc.RESCORE_PROMPTS), batch=2, frames=sc.REAL_FRAMES, mode="fp32",
                       frame_weight=weights, vocab=vocab)

    def load(slot, memory_seed, prefix, stop, frames, tables):
        eng.load(slot, memory_array(sc.REAL_FRAMES, sc.REAL_TINY.width, memory_seed), prefix, stop, frames,
                 frame_logp=tables)

    record = sc.rescore_forced(eng, vocab, g, case, load)
    same = sum(int(a == b) for _, a, b in record)
    print(f"rescoring ({case}) oracle fp32 vs reference: {same}/{len(record)}")
    assert same == len(record)


@pytest.mark.parametrize("case", list(sc.REAL_CASES))
def test_real_full_oracle_vs_reference(case):
    """Product decoder shape: the oracle (fp32) picks the reference's greedy token at every forced
    step, its masked maximum equals the one the reference's argmax saw, and its teacher-forced
    logits match the reference's at the fixture's columns."""

    from oracle.engine import FRAME_TERM_NAMES
    from sheetsage2_refined_b200.engine import frame_terms

    g = np.load(GOLDEN / "real_full.npz")
    vocab = VocabTable()
    spec = sc.REAL_CASES[case]
    bias = None
    if spec["mode_bias"] is not None:
        bias = np.zeros(vocab.size, np.float32)
        bias[vocab.start["key_mode"]: vocab.start["key_mode"] + 108] = np.repeat(np.float32(spec["mode_bias"]), 12)
    eng = OracleEngine(sc.REAL, synthetic_state_dict(sc.REAL, sc.REAL_FULL_SEED), ClassGrammar(vocab, spec["prompts"]),
                       batch=2, frames=sc.REAL_FULL_FRAMES, mode="fp32", logit_bias=bias,
                       frame_weight=frame_terms(spec["frame_weight"], spec["prompts"]), vocab=vocab)
    assert len(FRAME_TERM_NAMES) == 8

    def load(slot, memory_seed, prefix, stop, frames, tables):
        eng.load(slot, memory_array(sc.REAL_FULL_FRAMES, sc.REAL.width, memory_seed), prefix, stop, frames,
                 frame_logp=tables)

    masks, logits = [], []
    record = sc.real_forced(eng, vocab, g, case, load, masks, logits)
    cols = g["columns"]
    for (slot, k, greedy, ref), m in zip(record, masks):
        assert greedy == ref, (slot, k, greedy, ref)
        assert abs(float(m[ref]) - float(g[f"{case}_s{slot}_top_values"][k, 0])) <= LOGIT_TOL_FP32, (slot, k)
    worst = 0.0
    for slot, k, row in logits:
        if k < sc.REAL_LOGIT_STEPS:
            worst = max(worst, float(np.abs(row[cols] - g[f"{case}_s{slot}_logits"][k]).max()))
    print(f"real_full {case}: {len(record)} forced steps, greedy equal; max |dlogit| {worst:.2e}")
    assert worst <= LOGIT_TOL_FP32


def test_bf16_rounding_matches_the_bit_rule():
    """The oracle's bfloat16 rounding (torch's conversion) equals round-to-nearest-even on the bits,
    ties, subnormals, infinities and NaN included."""

    from oracle.numerics import bf16, bf16_rule

    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2 ** 32, 1 << 20, dtype=np.uint64).astype(np.uint32)
    ties = (rng.integers(0, 2 ** 16, 4096, dtype=np.uint64).astype(np.uint32) << 16) | np.uint32(0x8000)
    x = np.concatenate([bits, ties]).view(np.float32)
    x = np.concatenate([x, np.float32([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-40, 3.4e38])])
    a, b = bf16(x), bf16_rule(x)
    nan = np.isnan(x)
    assert np.array_equal(np.isnan(a), nan) and np.array_equal(np.isnan(b), nan)
    assert np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))
