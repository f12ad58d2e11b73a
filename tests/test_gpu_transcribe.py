"""``transcribe_many`` end to end with this engine as the reference's ``BatchDecoder``.

The reference's whole-song scheduler (transcribe.py:225-398: windowing,
encoder, continuous batching of windows of different songs, overlap priming,
stop and limit endings, resume after a full window, detokenisation) runs
unchanged on a small random-init ``SheetSage`` with the real vocabulary
(``reference_path.tiny_sheetsage``) over two seeded songs of 40 s and 330 s
(one window; two windows, the second primed with the first's accepted events
and resumed once after filling the context).  It runs twice on the same GPU
with the same encoder: once with the reference's own engine (bf16 autocast,
CUDA graphs) and once with ``transcribe.BatchDecoder`` rebound to
``sheetsage2_refined_b200.BatchDecoder``, the binding INTEGRATION.md gives.

Every window's tokens are compared up to its first divergence: at least 99.5%
must be equal, and at a divergence the engine's own choice and the
reference's token must be an argmax near-tie of the engine's logits along
the reference's history (the window is replayed into a fresh engine and the
reference's tokens are forced).  With no divergence the event lists must be
equal.

The reference package comes from ``baseline/_ref`` (its unmodified install);
without it the test is skipped.
"""

import numpy as np
import pytest
import torch

from helpers import NEAR_TIE_ULPS, TOKEN_AGREEMENT, bf16_ulp
from reference_path import load_reference, seeded_waveforms, tiny_sheetsage

pytestmark = pytest.mark.gpu

PROMPT_CASES = {
    "full": (None, None),
    "mode_bias": (("timestamp", "downbeat_meter", "chord_detail", "key_mode", "melody_full"),
                  [-3.0, -1.5, -2.5, -2.0, -2.75, -4.0, -0.5, -2.5, -5.0]),
}


@pytest.fixture(autouse=True)
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")


def recording(base):
    """``base`` (an engine class) that also records every window: load arguments and taken tokens."""

    class Recording(base):
        windows: list = []

        def load(self, slot, memory, prefix, stop_seconds, frames=None, frame_logp=None, **kw):
            self._pending = getattr(self, "_pending", {})
            self._pending[slot] = (memory.detach().clone(), list(prefix), stop_seconds, frames)
            return super().load(slot, memory, prefix, stop_seconds, frames, frame_logp, **kw)

        def take(self, slot):
            tokens, ended = super().take(slot)
            Recording.windows.append((self._pending.pop(slot), tokens, ended))
            return tokens, ended

    Recording.windows = []
    return Recording


def run(ref, model, engine_class, prompts, mode_bias):
    ref.transcribe.BatchDecoder = engine_class
    model._batch_decoder = None
    kwargs = {"prompts": prompts} if prompts is not None else {}
    stats = {}
    events = ref.transcribe.transcribe_many(model, seeded_waveforms([40.0, 330.0]), batch_size=2, stats=stats,
                                            mode_bias=mode_bias, **kwargs)
    model._batch_decoder = None
    torch.cuda.synchronize()
    return events, list(engine_class.windows), stats


def near_tie_replay(model, window, ref_tokens, k, prompts, mode_bias):
    """Replay ``window`` in a fresh engine along the reference's tokens; near-tie at step k?"""

    from oracle.grammar import ClassGrammarOracle
    from sheetsage2_refined_b200 import BatchDecoder
    from sheetsage2_refined_b200.grammar import ClassGrammar

    from sheetsage2_refined_b200.vocab_table import FULL_PROMPTS

    (memory, prefix, stop, frames), _, _ = window
    prompts = prompts or FULL_PROMPTS
    eng = BatchDecoder(model.decoder, model.vocab, batch=1, frames=memory.shape[-2], prompts=prompts,
                       mode_bias=mode_bias)
    eng.load(0, memory, prefix, stop, frames)
    grammar = ClassGrammarOracle(ClassGrammar(model.vocab, prompts))
    names = ("in_shift", "shift_run", "payload", "last_field", "incomplete", "finished", "ended")
    for i in range(len(prefix), k + 1):
        state = {n: eng.state[n].cpu().numpy().copy() for n in names}
        logits, greedy = eng.step_debug(np.array([ref_tokens[i]]))
    bias = getattr(eng, "_bias", None)
    x = logits[0] + (bias if bias is not None else 0.0)
    masked = np.where(grammar.allowed(state)[0], x, -np.inf)
    a, b = int(greedy[0]), int(ref_tokens[k])
    eng.close()
    return abs(float(masked[a]) - float(masked[b])) <= NEAR_TIE_ULPS * bf16_ulp(max(abs(masked[a]), abs(masked[b])))


@pytest.mark.parametrize("case", list(PROMPT_CASES))
def test_transcribe_many_with_the_b200_engine(case):
    ref = load_reference()
    if ref is None:
        pytest.skip("the reference package is not installed under baseline/_ref")
    from sheetsage2_refined_b200 import BatchDecoder

    prompts, mode_bias = PROMPT_CASES[case]
    model = tiny_sheetsage(ref).to("cuda")
    original = ref.transcribe.BatchDecoder
    try:
        ev_ref, win_ref, st_ref = run(ref, model, recording(original), prompts, mode_bias)
        ev_new, win_new, st_new = run(ref, model, recording(BatchDecoder), prompts, mode_bias)
    finally:
        ref.transcribe.BatchDecoder = original
    assert len(win_ref) >= 3, len(win_ref)
    same = compared = 0
    divergences = []
    for w, (wn, wr) in enumerate(zip(win_new, win_ref)):
        (_, prefix_n, _, _), tok_n, end_n = wn
        (_, prefix_r, _, _), tok_r, end_r = wr
        assert prefix_n == prefix_r, w  # the same window, primed the same way
        start = len(prefix_r)
        n = min(len(tok_n), len(tok_r))
        k = next((i for i in range(start, n) if tok_n[i] != tok_r[i]), None)
        if k is None:
            assert len(tok_n) == len(tok_r) and end_n == end_r, (w, len(tok_n), len(tok_r), end_n, end_r)
            same += n - start
            compared += n - start
            continue
        same += k - start
        compared += k - start + 1
        divergences.append((w, k, tok_n[k], tok_r[k], near_tie_replay(model, wr, tok_r, k, prompts, mode_bias)))
        break  # later windows are primed by different events
    print(f"transcribe_many ({case}): {len(win_ref)} windows, {same}/{compared} generated tokens equal, "
          f"divergences {divergences}; windows {[(w['song'], w['start'], w['generated'], w['ended']) for w in st_new['windows']]}")
    assert all(t for *_, t in divergences), divergences
    assert same / compared >= TOKEN_AGREEMENT
    if not divergences:
        assert len(win_new) == len(win_ref) and ev_new == ev_ref
