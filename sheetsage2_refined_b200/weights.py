"""Decoder shape, parameter layout and seeded synthetic weights.

``DecoderConfig`` mirrors ``sheetsage2_refined/decoder.py:12-21`` (dropout and
the pad token play no part in decoding).  ``param_layout`` lists the
parameters under the reference's ``TokenDecoder.state_dict()`` names, in
``TokenDecoder.parameters()`` order (decoder.py:28-96), so a reference
decoder and a ``DecoderWeights`` object are interchangeable inputs of
``BatchDecoder``.

Synthetic weights: every Linear weight and bias and both embeddings are drawn
from N(0, 0.02) in float32 with ``numpy.random.default_rng(seed)``, one
parameter after another in layout order; LayerNorm parameters keep PyTorch's
initialisation (weight 1, bias 0).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

POSITION_OFFSET = 2  # decoder.py:24-25: position p uses row p + 2


@dataclass(frozen=True)
class DecoderConfig:
    vocab_size: int = 31_678
    width: int = 512
    layers: int = 6
    heads: int = 8
    ffn_width: int = 2048
    max_tokens: int = 5120

    @property
    def head_dim(self) -> int:
        return self.width // self.heads


def param_layout(config: DecoderConfig) -> list[tuple[str, tuple[int, ...]]]:
    """``(state_dict name, shape)`` of every decoder parameter, in order."""

    d, f = config.width, config.ffn_width
    out = [
        ("token_embedding.weight", (config.vocab_size, d)),
        ("position_embedding.weight", (config.max_tokens + POSITION_OFFSET, d)),
        ("embedding_norm.weight", (d,)),
        ("embedding_norm.bias", (d,)),
    ]
    for i in range(config.layers):
        p = f"layers.{i}."
        for attn in ("self_attn", "cross_attn"):
            for proj in ("q", "k", "v", "out"):
                out += [(f"{p}{attn}.{proj}.weight", (d, d)), (f"{p}{attn}.{proj}.bias", (d,))]
            out += [(f"{p}{attn}_norm.weight", (d,)), (f"{p}{attn}_norm.bias", (d,))]
        out += [
            (f"{p}fc1.weight", (f, d)),
            (f"{p}fc1.bias", (f,)),
            (f"{p}fc2.weight", (d, f)),
            (f"{p}fc2.bias", (d,)),
            (f"{p}final_norm.weight", (d,)),
            (f"{p}final_norm.bias", (d,)),
        ]
    return out


def is_norm(name: str) -> bool:
    return "_norm." in name or name.startswith("embedding_norm.")


def synthetic_state_dict(config: DecoderConfig, seed: int, std: float = 0.02) -> dict[str, np.ndarray]:
    """Seeded float32 weights (see the module docstring for the rule)."""

    rng = np.random.default_rng(seed)
    state = {}
    for name, shape in param_layout(config):
        if is_norm(name):
            state[name] = np.ones(shape, np.float32) if name.endswith("weight") else np.zeros(shape, np.float32)
        else:
            state[name] = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
    return state


class DecoderWeights:
    """A decoder's configuration and weights without the torch module.

    Duck-types the two things ``BatchDecoder`` reads from the reference
    ``TokenDecoder``: ``.config`` and ``.state_dict()``.
    """

    def __init__(self, config: DecoderConfig, state: dict):
        missing = [name for name, _ in param_layout(config) if name not in state]
        if missing:
            raise ValueError(f"missing decoder parameters: {missing[:4]}{'...' if len(missing) > 4 else ''}")
        self.config = config
        self._state = state

    @classmethod
    def synthetic(cls, config: DecoderConfig, seed: int, std: float = 0.02) -> "DecoderWeights":
        return cls(config, synthetic_state_dict(config, seed, std))

    def state_dict(self) -> dict:
        return self._state

    def parameters(self):
        return iter(self._state[name] for name, _ in param_layout(self.config))


def memory_array(frames: int, width: int, seed: int) -> np.ndarray:
    """Synthetic encoder memory ``[1, frames, width]`` ~ N(0, 1), float32."""

    return np.random.default_rng(seed).standard_normal((1, frames, width), dtype=np.float32)
