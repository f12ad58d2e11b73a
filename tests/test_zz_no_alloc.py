"""The allocation-free masked argmax entry point against the engine's own selection.

``s2r_masked_argmax_noalloc`` is for callers that cannot call cudaMalloc
while decoding (a host whose pool allocator reserves all device memory up
front, or a serving loop that must not stall the device, which cudaFree
synchronises).  It must pick exactly the token the
engine's fused logits kernel picks: this test runs the engine one step at a
time through ``s2r_step_debug`` (which returns the raw logits and the greedy
choice), rebuilds the grammar mask from the slots' state before the step, and
calls the entry point through the C ABI on the same logits, mask and mode
bias, twice in a row.  The file sorts last so that a run stopping at the
first failure has already run every other test.
"""

import ctypes as C

import numpy as np
import pytest
import torch

import scenarios as sc
from helpers import loader, weights
from oracle.grammar import ClassGrammarOracle
from sheetsage2_refined_b200 import _lib
from sheetsage2_refined_b200.grammar import ClassGrammar
from sheetsage2_refined_b200.vocab_table import VocabTable
from sheetsage2_refined_b200.weights import DecoderWeights

pytestmark = pytest.mark.gpu

GRAMMAR_STATE = ("in_shift", "shift_run", "payload", "last_field", "incomplete", "finished", "ended")


def ptr(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def test_noalloc_argmax_matches_engine_selection_twice():
    if not torch.cuda.is_available():
        pytest.fail("needs a CUDA device")
    from sheetsage2_refined_b200 import BatchDecoder

    vocab = VocabTable()
    prompts = sc.REAL_PROMPT_SETS[1]  # includes key_mode, so the mode bias is live
    bias_values = [0.0, 1.5, -0.5, 2.0, 0.25, -1.0, 3.0, 0.5, -2.0]
    dec = DecoderWeights(sc.REAL_TINY, weights(sc.REAL_TINY, sc.REAL_SEED))
    eng = BatchDecoder(dec, vocab, batch=2, frames=sc.REAL_FRAMES, prompts=prompts, mode_bias=bias_values)
    load = loader(eng, sc.REAL_TINY.width, sc.REAL_FRAMES)
    prefix = vocab.prompt_prefix(prompts)
    load(0, 51, prefix, None, sc.REAL_FRAMES, None)
    load(1, 52, prefix + [vocab.start["shift"] + 5], None, 40, None)
    grammar = ClassGrammarOracle(ClassGrammar(vocab, prompts))
    lib = _lib.load()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    bias = torch.from_numpy(eng._bias).cuda()
    for call in range(2):
        state = {name: eng.state[name].cpu().numpy().copy() for name in GRAMMAR_STATE}
        # row-major [rows, vocab] as the C ABI expects (the oracle's mask comes out column-major)
        allowed = np.ascontiguousarray(grammar.allowed(state), dtype=np.uint8)
        logits, greedy = eng.step_debug(None)  # the engine's fused selection
        d_logits = torch.from_numpy(np.ascontiguousarray(logits)).cuda()
        d_allowed = torch.from_numpy(allowed).cuda()
        assert d_allowed.is_contiguous() and d_logits.is_contiguous()
        out = torch.full((2,), -1, dtype=torch.int64, device="cuda")
        rc = lib.s2r_masked_argmax_noalloc(ptr(d_logits), ptr(bias), ptr(d_allowed), 2, vocab.size, ptr(out), stream)
        assert rc == _lib.S2R_OK, lib.s2r_last_error()
        torch.cuda.synchronize()
        assert out.cpu().tolist() == greedy.tolist(), (call, out.cpu().tolist(), greedy.tolist())


def _edge_case_inputs(rows: int, vocab: int, seed: int):
    """Seeded logits and masks with the cases where a selection can go wrong.

    Row 0 has nothing allowed; row 1 allows only tokens whose value is -inf;
    rows 2-3 plant equal maxima in different CTAs' vocabulary ranges (256
    tokens per CTA); row 4's maximum is a signed zero at two indices, -0.0 at
    the lower one; row 5 has NaNs; row 6 ties its maximum with a token whose
    bias is -inf.  The other rows are random, with random ties.
    """

    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(rows, vocab, generator=g)
    # coarse values so that random ties happen in every row
    logits = torch.round(logits * 4) / 4
    allowed = torch.rand(rows, vocab, generator=g) < 0.3
    allowed[0] = False
    logits[1] = float("-inf")
    allowed[1, ::7] = True
    logits[2, 300] = logits[2, 2900] = 50.0
    allowed[2, 300] = allowed[2, 2900] = True
    logits[3, 700] = logits[3, 1100] = logits[3, 2999] = 60.0
    allowed[3, [700, 1100, 2999]] = True
    logits[4] = -torch.rand(vocab, generator=g) - 1.0
    logits[4, 40], logits[4, 2000] = -0.0, 0.0
    allowed[4, 40] = allowed[4, 2000] = True
    logits[5, 77] = logits[5, 1500] = float("nan")
    allowed[5, [77, 1500]] = True
    logits[6, 5] = logits[6, 2500] = 70.0
    allowed[6, [5, 2500]] = True
    bias = torch.randn(vocab, generator=g).round()
    bias[5] = float("-inf")
    return logits.contiguous(), allowed.to(torch.uint8).contiguous(), bias.contiguous()


def test_noalloc_argmax_edge_cases_match_torch_twice():
    """Synthetic rows against torch.argmax of the reference's masked logits (engine.py:349-350).

    Covers the index-0 rule (nothing allowed, or a best allowed value of -inf),
    ties split across CTAs, signed zeros, NaNs, a -inf bias, ``bias=NULL`` and
    the largest row count the static scratch holds.  Two different inputs are
    selected in a row so that the second call sees the scratch the first left.
    """

    if not torch.cuda.is_available():
        pytest.fail("needs a CUDA device")
    lib = _lib.load()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rows, vocab = 1024, 3000
    for call, (seed, use_bias) in enumerate(((1, True), (2, False))):
        logits, allowed, bias = _edge_case_inputs(rows, vocab, seed)
        x = logits + bias if use_bias else logits
        want = torch.where(allowed.bool(), x, torch.tensor(float("-inf"))).argmax(-1)
        d_logits, d_allowed, d_bias = logits.cuda(), allowed.cuda(), bias.cuda()
        out = torch.full((rows,), -1, dtype=torch.int64, device="cuda")
        rc = lib.s2r_masked_argmax_noalloc(ptr(d_logits), ptr(d_bias) if use_bias else None, ptr(d_allowed), rows,
                                           vocab, ptr(out), stream)
        assert rc == _lib.S2R_OK, lib.s2r_last_error()
        torch.cuda.synchronize()
        got = out.cpu()
        assert got[:7].tolist() == want[:7].tolist(), (call, got[:7].tolist(), want[:7].tolist())
        assert got[0] == 0 and got[1] == 0, call
        assert torch.equal(got, want), (call, int((got != want).sum()))


def test_noalloc_argmax_rejects_more_rows_than_its_scratch():
    lib = _lib.load()
    rc = lib.s2r_masked_argmax_noalloc(C.c_void_p(16), None, C.c_void_p(16), 1025, 8, C.c_void_p(16), None)
    assert rc == _lib.S2R_EINVAL
    assert b"1024" in lib.s2r_last_error()
