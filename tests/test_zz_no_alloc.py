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


def test_noalloc_argmax_rejects_more_rows_than_its_scratch():
    lib = _lib.load()
    rc = lib.s2r_masked_argmax_noalloc(C.c_void_p(16), None, C.c_void_p(16), 1025, 8, C.c_void_p(16), None)
    assert rc == _lib.S2R_EINVAL
    assert b"1024" in lib.s2r_last_error()
