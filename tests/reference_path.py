"""Drive the installed reference package (SheetSage2-Refined) on its own code path.

The reference is pure Python over PyTorch.  ``python -m pip install
--no-index --no-build-isolation --no-deps --target baseline/_ref <checkout>``
puts an unmodified copy of it under ``baseline/_ref``; this module imports it
from there (or from a directory given explicitly, such as a read-only
checkout) and builds its ``TokenDecoder`` / ``BatchDecoder`` with the seeded
synthetic weights of this repository, so that the golden generator, the
benchmark's reference measurements and the drop-in tests run the reference's
own engine, on CPU (float32, eager) or on CUDA (bf16 autocast, one CUDA graph
per cache-length bucket; engine.py:1-16,234-281).

The reference's package ``__init__`` imports ``soundfile`` (only
``transcribe.load_waveform`` uses it); a stub module stands in for it.

For the synthetic vocabularies the table grammar
(``sheetsage2_refined_b200.grammar.TableGrammar``) enters the reference
engine through its grammar duck type (``allowed / update / prefix_state /
time_seconds / prompts``, engine.py:74,211,349,355) with three extra state
entries (``g``, ``count``, ``target``).
"""

from __future__ import annotations

import importlib
import sys
import types
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
INSTALLED = ROOT / "baseline" / "_ref"


def load_reference(path: str | Path | None = None):
    """The reference package's modules as a namespace, or None when it is not installed.

    ``path`` is a directory that contains ``sheetsage2_refined/`` (default:
    ``baseline/_ref``).  Returns an object with the attributes ``engine``,
    ``decoder``, ``grammar``, ``vocab``, ``transcribe``, ``model``,
    ``encoder`` (the reference's modules) and ``path``.
    """

    where = Path(path) if path is not None else INSTALLED
    if not (where / "sheetsage2_refined" / "engine.py").exists():
        return None
    sys.modules.setdefault("soundfile", types.ModuleType("soundfile"))
    if str(where) not in sys.path:
        sys.path.insert(0, str(where))
    ns = types.SimpleNamespace(path=where)
    for name in ("engine", "decoder", "grammar", "vocab", "transcribe", "model", "encoder"):
        setattr(ns, name, importlib.import_module(f"sheetsage2_refined.{name}"))
    return ns


class TableGrammarRef:
    """The table grammar in the reference engine's grammar duck type, on ``device``."""

    def __init__(self, desc, device="cpu"):
        self.device = torch.device(device)
        self.table = torch.tensor(np.asarray(desc.table, bool), device=self.device)
        self.states, self.multiplier = desc.states, desc.multiplier
        self.time_seconds = torch.tensor(desc.time_seconds, device=self.device)
        self.prompts = desc.prompts

    def allowed(self, state):
        return self.table[state["g"]]

    def update(self, state, tokens, active, stop, at_limit):
        g = (self.multiplier * state["g"] + tokens) % self.states
        count = state["count"] + 1
        done = count >= state["target"]
        ended = torch.where(done, 1, torch.where(at_limit, 3, 0))
        finished = done | at_limit
        state["g"].copy_(torch.where(active, g, state["g"]))
        state["count"].copy_(torch.where(active, count, state["count"]))
        state["ended"].copy_(torch.where(active & finished, ended, state["ended"]))
        state["finished"].copy_(state["finished"] | (active & finished))

    def prefix_state(self, tokens, out_index, device):
        g = 0
        for token in tokens[out_index + 1:]:
            g = (self.multiplier * g + token) % self.states
        z = lambda v: torch.tensor([v], dtype=torch.long)  # noqa: E731
        return {"g": z(g), "count": z(0), "finished": torch.tensor([False]), "ended": z(0)}


def ref_decoder(ref, config, seed: int, device="cpu"):
    """The reference ``TokenDecoder`` with this repository's seeded synthetic weights."""

    from sheetsage2_refined_b200.weights import synthetic_state_dict

    dc = ref.decoder.DecoderConfig(vocab_size=config.vocab_size, width=config.width, layers=config.layers,
                                   heads=config.heads, ffn_width=config.ffn_width, max_tokens=config.max_tokens)
    decoder = ref.decoder.TokenDecoder(dc)
    state = {k: torch.from_numpy(v) for k, v in synthetic_state_dict(config, seed).items()}
    decoder.load_state_dict(state, strict=True)
    return decoder.to(device).eval()


def table_engine(ref, decoder, desc, batch: int, frames: int):
    """The reference ``BatchDecoder`` driven by the table grammar ``desc``."""

    engine = ref.engine.BatchDecoder(decoder, ref.vocab.Vocab(), batch=batch, frames=frames)
    device = engine.device
    engine.grammar = TableGrammarRef(desc, device)
    engine.state["g"] = torch.zeros(batch, dtype=torch.long, device=device)
    engine.state["count"] = torch.zeros(batch, dtype=torch.long, device=device)
    engine.state["target"] = torch.full((batch,), np.iinfo(np.int64).max, dtype=torch.long, device=device)
    return engine


def set_target(engine, slot: int, target: int | None) -> None:
    """The table grammar's generated-token count of ``slot`` (after ``engine.load``)."""

    if target is not None:
        engine.state["target"][slot] = target


def tiny_sheetsage(ref, seed: int = 0, decoder_seed: int = 5):
    """A small random-init ``SheetSage`` (model.py:18-51) with the real 32,576-token vocabulary.

    The encoder keeps the reference's structure (mel front end, three
    ConvNeXt stages with strides 1-2-2, Conformer blocks; 960 samples per
    frame) at width 128 with two blocks; its mel filterbank buffer gets seeded
    positive values so that the memory varies over time.  The decoder (2
    layers, width 128, 2 heads, FFN 256) takes this repository's seeded
    synthetic weights, with the token-embedding rows of the shift tokens
    scaled by 4: the reference's ``Vocab.decode`` (vocab.py:322-349) rejects a
    window whose first event has no subbeat shift, which the grammar allows
    but a trained decoder never emits, so untrained weights must prefer
    shifts.  Windows are encoded at their own length (``pad_encoder = False``,
    as for the fine-tuned decoders).
    """

    from sheetsage2_refined_b200.weights import DecoderConfig, synthetic_state_dict

    torch.manual_seed(seed)
    enc = ref.encoder.EncoderConfig(n_mels=32, stage_channels=(32, 64, 128), stage_depths=(1, 1, 1), width=128,
                                    ffn_width=256, layers=2, heads=2, conv_kernel=7)
    vocab_size = ref.vocab.Vocab().size
    config = DecoderConfig(vocab_size=vocab_size, width=128, layers=2, heads=2, ffn_width=256, max_tokens=5120)
    dc = ref.decoder.DecoderConfig(vocab_size=vocab_size, width=128, layers=2, heads=2, ffn_width=256, max_tokens=5120)
    model = ref.model.SheetSage(enc, dc)
    with torch.no_grad():
        fb = model.encoder.frontend.mel_fb
        fb.copy_(torch.rand(fb.shape, generator=torch.Generator().manual_seed(seed + 1)) * 1e-3)
        state = {k: torch.from_numpy(v) for k, v in synthetic_state_dict(config, decoder_seed).items()}
        model.decoder.load_state_dict(state, strict=True)
        vocab = ref.vocab.Vocab()
        model.decoder.token_embedding.weight[vocab.start["shift"]:vocab.end["shift"]] *= 4.0
    model.pad_encoder = False
    return model.eval()


def seeded_waveforms(seconds, seed: int = 0, rate: int = 24_000):
    """Seeded noise bursts as mono 24 kHz waveforms, one per length in ``seconds``."""

    gen = torch.Generator().manual_seed(seed)
    out = []
    for s in seconds:
        n = int(s * rate)
        env = (torch.sin(torch.arange(n) * (2 * np.pi * 2.0 / rate)) > 0).float()  # 2 Hz on/off
        out.append((torch.randn(n, generator=gen) * 0.1 * (0.2 + env)).float())
    return out
