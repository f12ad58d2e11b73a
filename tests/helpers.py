"""Engine factories and comparison rules shared by the parity tests."""

from __future__ import annotations

import numpy as np

import scenarios as sc
from oracle.engine import OracleEngine
from sheetsage2_refined_b200.weights import DecoderWeights, memory_array, synthetic_state_dict

# Parity tolerances against the reference decoder: teacher-forced logits within 2e-2 (bf16), greedy tokens
# equal on at least 99.5% of steps, every divergence an argmax near-tie.
LOGIT_TOL = 2e-2
LOGIT_MAX = 3e-2  # bound on every logit (see logit_error)
TOKEN_AGREEMENT = 0.995
# A near-tie: the two candidates' logits differ by at most this many bfloat16
# ulps of the larger one (2^-7 relative per ulp for values in [1, 2)).
NEAR_TIE_ULPS = 2

_WEIGHTS: dict = {}


def weights(config, seed):
    key = (config, seed)
    if key not in _WEIGHTS:
        _WEIGHTS[key] = synthetic_state_dict(config, seed)
    return _WEIGHTS[key]


def cuda_engine(config, seed, grammar, batch, frames, **kw):
    from sheetsage2_refined_b200 import BatchDecoder

    return BatchDecoder(DecoderWeights(config, weights(config, seed)), None, batch=batch, frames=frames,
                        grammar=grammar, **kw)


def oracle_engine(config, seed, grammar, batch, frames, mode="bf16", **kw):
    return OracleEngine(config, weights(config, seed), grammar, batch=batch, frames=frames, mode=mode, **kw)


def loader(engine, width, frames_engine):
    def load(slot, memory_seed, prefix, stop, frames, target):
        engine.load(slot, memory_array(frames_engine, width, memory_seed), prefix, stop, frames, target=target)
    return load


def logit_error(a: np.ndarray, b: np.ndarray) -> float:
    """Largest logit difference in units of ``3e-2 + ulp_bf16(max(|a|, |b|))``.

    Logits are bfloat16 values widened to float32 (engine.py:315).  The
    reference's own CUDA arithmetic (the oracle's bf16 mode) differs from its
    float32 path by up to 0.0254 at the 12-layer workload (0.014% of the
    logits beyond 2e-2): bf16 rounding noise accumulated through 12 layers is
    absolute, whatever the logit's size, and large logits add one rounding
    step.  A result <= 1 bounds every logit (the reference's own bf16 path
    scores 0.56 on this scale); ``logit_within`` counts the fraction within
    2e-2, which must stay >= 99.9%.
    """

    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    mag = np.maximum(np.abs(a), np.abs(b))
    ulp = np.exp2(np.floor(np.log2(np.maximum(mag, 2.0 ** -126))) - 7)
    return float((np.abs(a - b) / (LOGIT_MAX + ulp)).max())


def logit_within(a: np.ndarray, b: np.ndarray) -> tuple[int, int]:
    """(entries within 2e-2, entries)."""

    d = np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))
    return int((d <= LOGIT_TOL).sum()), int(d.size)


# Fraction of logits that must lie within 2e-2 (the rest within 3e-2 + 1 bf16 ulp).
LOGIT_WITHIN_FRACTION = 0.999


def bf16_ulp(x: float) -> float:
    x = abs(float(x))
    if x == 0.0:
        return 2.0 ** -133
    return 2.0 ** (np.floor(np.log2(x)) - 7)


def near_tie(masked_logits: np.ndarray, a: int, b: int) -> bool:
    """True if tokens ``a`` and ``b`` are within NEAR_TIE_ULPS bf16 ulps in ``masked_logits``."""

    va, vb = float(masked_logits[a]), float(masked_logits[b])
    if not (np.isfinite(va) and np.isfinite(vb)):
        return False
    return abs(va - vb) <= NEAR_TIE_ULPS * bf16_ulp(max(abs(va), abs(vb)))


def masked(logits: np.ndarray, allowed: np.ndarray, bias=None) -> np.ndarray:
    x = logits if bias is None else logits + bias
    return np.where(allowed, x, -np.inf)


def window_agreement(pairs, tie_at):
    """Greedy agreement of free-running windows with the reference's tokens.

    ``pairs`` holds ``(got, ref, start)`` per window: both token lists and the
    index of the first generated token.  Tokens are compared from ``start`` up
    to the window's first divergence; after it the two histories differ, so
    later tokens of that window are not compared.  ``tie_at(window, k)``
    returns the reference-side masked logits (bias and rescoring included) of
    the step that chose token ``k``, to judge the divergence a near-tie.

    Returns ``(same, compared, divergences)``; every divergence is ``(window,
    k, engine token, reference token, is_near_tie)``.
    """

    same = compared = 0
    divergences = []
    for w, (got, ref, start) in enumerate(pairs):
        n = min(len(got), len(ref))
        k = next((i for i in range(start, n) if got[i] != ref[i]), None)
        if k is None:
            assert len(got) == len(ref), (w, len(got), len(ref))
            same += n - start
            compared += n - start
            continue
        same += k - start
        compared += k - start + 1
        divergences.append((w, k, int(got[k]), int(ref[k]), near_tie(tie_at(w, k), int(got[k]), int(ref[k]))))
    return same, compared, divergences


def masked_logits_at(oracle, load_args, ref, k):
    """The oracle's masked logits for the step that chose ``ref[k]`` in slot 0.

    ``load_args`` = ``(load, memory_seed, prefix, stop, frames, target)``: the
    window is loaded into slot 0, the reference tokens after its prefix are
    forced one by one up to position ``k``, and the masked logits of the
    step predicting ``ref[k]`` are returned.
    """

    load, seed, prefix, stop, frames, target = load_args
    load(0, seed, prefix, stop, frames, target)
    for i in range(len(prefix), k):
        oracle.step(forced=np.array([ref[i]]))
    oracle.step(forced=np.array([ref[k]]))
    return oracle.last_masked[0]


def teacher_forced_compare(engine, oracle, tokens, prefix_len, steps, slot=0):
    """Force ``tokens[prefix_len:]`` through both engines (slot ``slot``); compare per step.

    Returns ``(max_abs_logit_diff, max_logit_error, fraction_within_2e-2,
    agreement, mismatches)``; every mismatch
    is ``(step, engine_choice, oracle_choice, is_near_tie)``.
    """

    B = engine.batch
    max_diff, same, mismatches = 0.0, 0, []
    max_err, within, count = 0.0, 0, 0
    for k in range(steps):
        forced = np.full(B, -1, np.int64)
        forced[slot] = tokens[prefix_len + k]
        allowed = oracle.grammar.allowed(oracle.state)[slot]
        lg_e, gr_e = engine.step_debug(forced)
        lg_o, gr_o = oracle.step(forced=forced)
        max_diff = max(max_diff, float(np.abs(lg_e[slot] - lg_o[slot]).max()))
        max_err = max(max_err, logit_error(lg_e[slot], lg_o[slot]))
        w, n = logit_within(lg_e[slot], lg_o[slot])
        within, count = within + w, count + n
        if gr_e[slot] == gr_o[slot]:
            same += 1
        else:
            bias = oracle.logit_bias
            ml = masked(lg_o[slot], allowed, bias)
            mismatches.append((k, int(gr_e[slot]), int(gr_o[slot]), near_tie(ml, int(gr_e[slot]), int(gr_o[slot]))))
    return max_diff, max_err, within / count, same / steps, mismatches


def prefill_compare(la: np.ndarray, lb: np.ndarray, ga: int, gb: int, exact: bool, what) -> None:
    """A decode step after a prefilled prefix (``la``, ``ga``) against the same step after the prefix
    was forced token by token (``lb``, ``gb``).

    ``exact``: the prefill ran on the decode step's kernels, so logits and choice are bit-identical.
    Otherwise the prefill ran on tensor cores (float32 sums in another order than the decode step's):
    logits within the parity tolerance, and a different choice only at a near-tie.
    """

    if exact:
        assert np.array_equal(la, lb) and ga == gb, what
        return
    assert logit_error(la, lb) <= 1.0, (what, float(np.abs(la - lb).max()))
    w, n = logit_within(la, lb)
    assert w / n >= LOGIT_WITHIN_FRACTION, (what, w, n)
    assert ga == gb or near_tie(la, int(ga), int(gb)), (what, ga, gb)


__all__ = ["sc"]
