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
