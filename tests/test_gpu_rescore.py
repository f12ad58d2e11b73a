"""Frame-head rescoring on the CUDA engine (engine.py:81-116,218-232,318-347,358-369).

Every rescoring term is on in one of two weight sets (chord and key terms;
meter, downbeat and key-boundary terms).  The reference's greedy tokens of
both windows (golden ``rescore.npz``) are forced through the engine step by
step; at every step the engine's own greedy choice -- logits + mode bias +
rescoring terms, grammar mask, argmax -- is compared with the reference's
choice and with the oracle's bf16 choice on the same forced prefix.  The
rescoring state (current frame, key stated, active meter, meter change)
advances on the device from the forced tokens, so a wrong state shows up as
a wrong choice later on.  Runs on the step as a CUDA graph, as plain launches
and on a 16-slot engine (tensor-core logits).
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import scenarios as sc
from helpers import TOKEN_AGREEMENT, near_tie, weights
from oracle.engine import FRAME_TERM_NAMES, OracleEngine
from sheetsage2_refined_b200.grammar import ClassGrammar
from sheetsage2_refined_b200.vocab_table import VocabTable
from sheetsage2_refined_b200.weights import DecoderWeights, memory_array

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")


@pytest.mark.parametrize("flags,batch", [(0, 2), (3, 2), (0, 16)], ids=["graph", "plain-launches", "tensor-core"])
def test_rescore_vs_reference_and_oracle(flags, batch):
    """Both weight sets; agreement is counted over every forced step of both."""

    from sheetsage2_refined_b200 import BatchDecoder

    g = np.load(GOLDEN / "rescore.npz")
    vocab = VocabTable()
    dec = DecoderWeights(sc.REAL_TINY, weights(sc.REAL_TINY, sc.REAL_SEED))

    def loader(engine):
        def load(slot, memory_seed, prefix, stop, frames, tables):
            mem = memory_array(sc.REAL_FRAMES, sc.REAL_TINY.width, memory_seed)
            engine.load(slot, mem, prefix, stop, frames, frame_logp=tables)
        return load

    steps = vs_ref = vs_oracle = 0
    divergences = []
    for case, weight in sc.RESCORE_CASES.items():
        eng = BatchDecoder(dec, vocab, batch=batch, frames=sc.REAL_FRAMES, prompts=sc.RESCORE_PROMPTS,
                           frame_weight=weight, flags=flags)
        assert eng.rescore
        frame_weight = tuple(float(weight.get(n, 0.0)) for n in FRAME_TERM_NAMES)
        oracles = [OracleEngine(sc.REAL_TINY, weights(sc.REAL_TINY, sc.REAL_SEED), ClassGrammar(vocab, sc.RESCORE_PROMPTS),
                                batch=batch, frames=sc.REAL_FRAMES, mode=mode, frame_weight=frame_weight, vocab=vocab)
                   for mode in ("bf16", "fp32")]
        got = sc.rescore_forced(eng, vocab, g, case, loader(eng))
        want = sc.rescore_forced(oracles[0], vocab, g, case, loader(oracles[0]))
        # the reference's masked logits at every step (the oracle's float32 mode reproduces its
        # rescored greedy choices exactly), to judge each divergence from the reference
        masks: list = []
        ref32 = sc.rescore_forced(oracles[1], vocab, g, case, loader(oracles[1]), masks)
        assert [(s, r) for s, _, r in got] == [(s, r) for s, _, r in want] == [(s, r) for s, _, r in ref32]
        steps += len(got)
        vs_ref += sum(int(a == r) for _, a, r in got)
        vs_oracle += sum(int(a == b) for (_, a, _), (_, b, _) in zip(got, want))
        divergences += [(case, i, a, r, near_tie(m, a, r)) for i, ((_, a, r), m) in enumerate(zip(got, masks))
                        if a != r]
        eng.close()
    print(f"rescoring: vs reference fp32 {vs_ref}/{steps}, vs oracle bf16 {vs_oracle}/{steps}, "
          f"divergences from the reference {divergences}")
    assert vs_oracle / steps >= TOKEN_AGREEMENT
    assert all(t for *_, t in divergences), divergences
    assert vs_ref / steps >= TOKEN_AGREEMENT
