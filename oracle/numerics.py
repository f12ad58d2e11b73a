"""Scalar arithmetic of the reference step, restated in numpy (test infrastructure).

``bf16`` is IEEE round-to-nearest-even from float32 to bfloat16 (the rule of
``torch.Tensor.to(torch.bfloat16)``), returned as float32 so that later
arithmetic stays in float32.
"""

from __future__ import annotations

import math

import numpy as np
import torch

LN_EPS = 1e-5  # torch.nn.LayerNorm default, decoder.py:63-68,95

_erf = np.vectorize(math.erf, otypes=[np.float64])
try:  # scipy is faster; math.erf is the fallback
    from scipy.special import erf as _scipy_erf

    def _erf64(x):
        return _scipy_erf(np.asarray(x, np.float64))

except ImportError:  # pragma: no cover
    def _erf64(x):
        return _erf(np.asarray(x, np.float64))


def bf16(a) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest, ties to even), widened back to float32.

    This is the conversion the reference's autocast performs, evaluated by
    torch's own CPU kernel (several threads; the numpy rule below is ~10x
    slower on large arrays).  ``bf16_rule`` restates the same rounding on
    the bits and a CPU test checks that the two agree bit for bit.
    """

    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return t.to(torch.bfloat16).to(torch.float32).numpy()


def bf16_rule(a) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest, ties to even) on the bits; NaN stays NaN."""

    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32).reshape(a.shape)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def layer_norm(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray) -> np.ndarray:
    """``torch.nn.functional.layer_norm`` over the last axis (biased variance), float32 out."""

    x64 = np.asarray(x, np.float64)
    mean = x64.mean(axis=-1, keepdims=True)
    var = ((x64 - mean) ** 2).mean(axis=-1, keepdims=True)
    y = (x64 - mean) / np.sqrt(var + LN_EPS) * gamma + beta
    return y.astype(np.float32)


def gelu(x: np.ndarray) -> np.ndarray:
    """Exact (erf) GELU, ``F.gelu`` default (decoder.py:83, engine.py:314), float32 out."""

    x64 = np.asarray(x, np.float64)
    return (x64 * 0.5 * (1.0 + _erf64(x64 * (1.0 / math.sqrt(2.0))))).astype(np.float32)


def softmax(s: np.ndarray) -> np.ndarray:
    """Softmax over the last axis, float32 out; ``-inf`` entries get probability 0."""

    s64 = np.asarray(s, np.float64)
    m = s64.max(axis=-1, keepdims=True)
    e = np.exp(s64 - m)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
