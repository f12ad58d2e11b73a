"""The product decoder shape on the CUDA engine against the reference (golden ``real_full.npz``).

6 layers, width 512, 8 heads, FFN 2048, the real 32,576-token vocabulary and
``TokenGrammar``, a 7,500-frame window, the mode bias or the key terms, and
frame-head rescoring (engine.py:77-116,316-369).  The reference's greedy tokens
of two windows per case are forced through the engine step by step; at every
step the engine's own greedy choice (logits, bias, rescoring, grammar mask,
argmax) must be the reference's, or a near-tie of the masked logits the
reference's argmax saw (the fixture keeps their top 8).  The raw logits of the
first 64 steps are compared at the fixture's 1,024 vocabulary columns.  Runs
on the CUDA-core path (2 slots) and the tensor-core path (16 slots, tcgen05
logits over the whole vocabulary).
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import scenarios as sc
from helpers import (LOGIT_WITHIN_FRACTION, NEAR_TIE_ULPS, TOKEN_AGREEMENT, bf16_ulp, logit_error, logit_within,
                     weights)
from sheetsage2_refined_b200.vocab_table import VocabTable
from sheetsage2_refined_b200.weights import DecoderWeights, memory_array

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")


def golden_near_tie(g, case: str, slot: int, k: int, token: int) -> bool:
    """``token`` is among the reference's 8 best masked values at step ``k`` and within
    NEAR_TIE_ULPS bf16 ulps of the best."""

    values, tokens = g[f"{case}_s{slot}_top_values"][k], g[f"{case}_s{slot}_top_tokens"][k]
    hit = np.nonzero(tokens == token)[0]
    if len(hit) == 0 or not np.isfinite(values[0]):
        return False
    return float(values[0] - values[hit[0]]) <= NEAR_TIE_ULPS * bf16_ulp(values[0])


@pytest.mark.parametrize("batch", [2, 16], ids=["cuda-core", "tensor-core"])
def test_real_shape_vs_reference_golden(batch):
    from sheetsage2_refined_b200 import BatchDecoder

    g = np.load(GOLDEN / "real_full.npz")
    vocab = VocabTable()
    dec = DecoderWeights(sc.REAL, weights(sc.REAL, sc.REAL_FULL_SEED))
    cols = g["columns"]
    steps = same = within = count = 0
    err = 0.0
    divergences = []
    for case, spec in sc.REAL_CASES.items():
        eng = BatchDecoder(dec, vocab, batch=batch, frames=sc.REAL_FULL_FRAMES, prompts=spec["prompts"],
                           mode_bias=spec["mode_bias"], frame_weight=spec["frame_weight"])
        assert eng.rescore

        def load(slot, memory_seed, prefix, stop, frames, tables):
            mem = memory_array(sc.REAL_FULL_FRAMES, sc.REAL.width, memory_seed)
            eng.load(slot, mem, prefix, stop, frames, frame_logp=tables)

        logits: list = []
        record = sc.real_forced(eng, vocab, g, case, load, logits=logits)
        for slot, k, got, ref in record:
            steps += 1
            if got == ref:
                same += 1
            else:
                divergences.append((case, slot, k, got, ref, golden_near_tie(g, case, slot, k, got)))
        for slot, k, row in logits:
            if k < sc.REAL_LOGIT_STEPS:
                want = g[f"{case}_s{slot}_logits"][k]
                err = max(err, logit_error(row[cols], want))
                w, n = logit_within(row[cols], want)
                within, count = within + w, count + n
        eng.close()
    print(f"product shape, batch {batch}: greedy {same}/{steps} equal to the reference, logit error {err:.3f}, "
          f"within 2e-2 {within}/{count}, divergences {divergences}")
    assert all(t for *_, t in divergences), divergences
    assert same / steps >= TOKEN_AGREEMENT
    assert err <= 1.0 and within / count >= LOGIT_WITHIN_FRACTION
