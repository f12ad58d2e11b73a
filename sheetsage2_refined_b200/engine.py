"""``BatchDecoder``: drop-in for ``sheetsage2_refined.engine.BatchDecoder`` on B200.

Same constructor, methods and attributes as the reference
(``sheetsage2_refined/engine.py:52-262``): ``load``, ``run``, ``finished``,
``take``, ``free_slots``, ``is_current`` and the ``frames``, ``rescore``,
``state``, ``out``, ``stop``, ``loaded``, ``bound``, ``grammar`` attributes.
Behind it every step runs in the CUDA engine of ``libs2r.so``; ``state`` and
``out`` are zero-copy torch views of the engine's device buffers.

There is no CPU path: without a CUDA device, or without the built library,
construction raises ``RuntimeError``.

Differences from the reference, all outside the numerics of a step:

* ``frame_weight`` rescoring (engine.py:81-116,318-347,358-369) needs the
  class grammar (the real vocabulary); ``load``'s ``frame_logp`` tables are
  copied into the engine per slot.
* ``grammar=`` accepts a grammar descriptor (``ClassGrammar`` or
  ``TableGrammar``) instead of building ``TokenGrammar(vocab, prompts)``;
  ``load(..., target=n)`` sets the table grammar's target length.
* ``load`` rejects ``frames < 1`` (the reference produces NaN there) and a
  prefix that does not leave room for one more token (the reference indexes
  past ``out``).
* ``BUCKETS`` is kept for callers that read it; the engine attends over each
  slot's exact length, so it plays no part.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from .grammar import ENDED, ClassGrammar
from .vocab_table import FULL_PROMPTS, NO_CHORD, NO_KEY, OUT, meter_tables
from .weights import DecoderConfig, param_layout

# Width of each frame table row (engine.py:97).
FRAME_WIDTHS = {"root": 12, "bass": 12, "detail": NO_CHORD, "quality": NO_CHORD, "key": 24, "key_boundary": 1,
                "downbeat": 1, "meter": 16}

# Terms a frame head can rescore (engine.py:29-38).
FRAME_TERMS = {
    "root": "chord_detail",
    "bass": "chord_detail",
    "detail": "chord_detail",
    "quality": "chord_detail",
    "key": "key",
    "key_boundary": "key",
    "downbeat": "downbeat_meter",
    "meter": "downbeat_meter",
}

_TORCH_DTYPES = {0: torch.float32, 2: torch.int64, 3: torch.uint8, 4: torch.float64, 5: torch.int32}
_TYPESTR = {0: "<f4", 2: "<i8", 3: "|u1", 4: "<f8", 5: "<i4"}


def frame_terms(weights, prompts) -> tuple[float, ...]:
    """engine.py:41-49: weights as a tuple in FRAME_TERMS order; ValueError for unknown terms."""

    weights = weights or {}
    unknown = set(weights) - set(FRAME_TERMS)
    if unknown:
        raise ValueError(f"unknown frame terms {sorted(unknown)}; known: {list(FRAME_TERMS)}")
    return tuple(float(weights.get(name, 0.0)) if prompt in prompts else 0.0 for name, prompt in FRAME_TERMS.items())


class _DeviceArray:
    """A raw device buffer described through ``__cuda_array_interface__``."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _config_of(decoder) -> DecoderConfig:
    cfg = decoder.config
    return DecoderConfig(vocab_size=cfg.vocab_size, width=cfg.width, layers=cfg.layers, heads=cfg.heads,
                         ffn_width=cfg.ffn_width, max_tokens=cfg.max_tokens)


def _f32(value, keep: list, device: torch.device | None = None):
    """A float32 contiguous tensor of ``value`` (torch or numpy) kept alive in ``keep``; its address."""

    t = value.detach() if isinstance(value, torch.Tensor) else torch.from_numpy(np.asarray(value))
    t = t.to(dtype=torch.float32).contiguous()
    keep.append(t)
    return t.data_ptr()


class BatchDecoder:
    BUCKETS = (256, 512, 1024, 2048, 4096)

    def __init__(self, decoder, vocab, *, batch: int, frames: int, prompts=FULL_PROMPTS, mode_bias=None,
                 frame_weight=None, dtype=torch.bfloat16, grammar=None, kv_pages: int = 0, flags: int = 0,
                 device=None):
        if not torch.cuda.is_available():
            raise RuntimeError("the B200 decode engine needs a CUDA device; it has no CPU path")
        lib = _lib.load()
        if lib.s2r_abi_version() != 1:
            raise RuntimeError("libs2r.so ABI version mismatch")
        self._lib = lib
        self.decoder, self.dtype, self.batch, self.frames = decoder, dtype, batch, frames
        config = _config_of(decoder)
        self.config = config
        self.max_tokens = config.max_tokens
        weight = decoder.state_dict()["token_embedding.weight"]
        if device is None:
            device = weight.device if isinstance(weight, torch.Tensor) and weight.is_cuda else torch.device(
                "cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        self.versions = self._versions(decoder)
        self.grammar = grammar if grammar is not None else ClassGrammar(vocab, prompts)
        self.prompts = tuple(sorted(set(prompts)))
        self.mode_bias = mode_bias if "key_mode" in prompts else None
        self.frame_weight = frame_terms(frame_weight, prompts)
        self.rescore = any(self.frame_weight)

        keep: list = []
        state = decoder.state_dict()
        missing = [n for n, _ in param_layout(config) if n not in state]
        if missing:
            raise ValueError(f"decoder state_dict lacks {missing[:3]}")
        layers = (_lib.LayerWeights * config.layers)()
        names = {
            "self_q": "self_attn.q", "self_k": "self_attn.k", "self_v": "self_attn.v", "self_out": "self_attn.out",
            "self_norm": "self_attn_norm", "cross_q": "cross_attn.q", "cross_k": "cross_attn.k",
            "cross_v": "cross_attn.v", "cross_out": "cross_attn.out", "cross_norm": "cross_attn_norm",
            "fc1": "fc1", "fc2": "fc2", "final_norm": "final_norm",
        }
        for i in range(config.layers):
            for field in _lib.LAYER_FIELDS:
                stem, kind = field.rsplit("_", 1)
                key = f"layers.{i}.{names[stem]}.{'weight' if kind == 'w' else 'bias'}"
                setattr(layers[i], field, _f32(state[key], keep))
        w = _lib.Weights(
            token_embedding=_f32(state["token_embedding.weight"], keep),
            position_embedding=_f32(state["position_embedding.weight"], keep),
            embedding_norm_w=_f32(state["embedding_norm.weight"], keep),
            embedding_norm_b=_f32(state["embedding_norm.bias"], keep),
            layers=layers,
        )
        g = self.grammar
        gd = _lib.GrammarDesc(kind=g.kind)
        if g.table is not None:
            table = np.ascontiguousarray(g.table, dtype=np.uint8)
            keep.append(table)
            gd.table, gd.states, gd.multiplier = table.ctypes.data, g.states, g.multiplier
            if g.vocab_size != config.vocab_size:
                raise ValueError(f"grammar vocabulary {g.vocab_size} != decoder vocabulary {config.vocab_size}")
        else:
            if g.vocab_size != config.vocab_size:
                raise ValueError(f"vocabulary has {g.vocab_size} tokens, decoder expects {config.vocab_size}")
            arrays = (np.ascontiguousarray(g.token_class, np.int8), np.ascontiguousarray(g.field_of_class, np.int32),
                      np.ascontiguousarray(g.time_seconds, np.float64))
            keep.extend(arrays)
            gd.token_class, gd.field_of_class, gd.time_seconds = (a.ctypes.data for a in arrays)
        cfg = _lib.Config(vocab_size=config.vocab_size, width=config.width, layers=config.layers,
                          heads=config.heads, ffn_width=config.ffn_width, max_tokens=config.max_tokens,
                          batch=batch, frames=frames, kv_pages=kv_pages, flags=flags)
        ctx = C.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(lib.s2r_create(C.byref(cfg), C.byref(w), C.byref(gd), self.device.index or 0, C.byref(ctx)))
        self._ctx = ctx
        del keep
        if self.mode_bias is not None:
            start = vocab.start["key_mode"]
            bias = np.zeros(config.vocab_size, np.float32)
            bias[start : start + NO_KEY] = np.repeat(np.asarray(self.mode_bias, np.float32), 12)  # engine.py:79-80
            self._bias = bias
            _lib.check(lib.s2r_set_logit_bias(ctx, bias.ctypes.data))
        if self.rescore:
            self._set_rescore(vocab)

        self.state = {name: self._view(name) for name in (
            "in_shift", "shift_run", "payload", "last_field", "incomplete", "finished", "ended", "token",
            "position", "g", "count", "target")}
        self.state["in_shift"] = self.state["in_shift"].view(torch.bool)
        self.state["finished"] = self.state["finished"].view(torch.bool)
        self.stop = self._view("stop")
        self.out = self._view("out").view(batch, self.max_tokens)
        self.bound = [0] * batch
        self.loaded = [False] * batch
        self._inflight: list = []  # (event, sources) of loads whose copies may still be pending

    def _set_rescore(self, vocab) -> None:
        """The rescoring configuration of engine.py:81-116 for the C ABI."""

        if vocab is None or self.grammar.kind != 0:
            raise ValueError("frame-head rescoring needs the real vocabulary and its class grammar")
        beats, units = meter_tables()
        self._meter = (np.ascontiguousarray(beats, np.int32), np.ascontiguousarray(units, np.int32))
        rs = _lib.Rescore()
        for i, w in enumerate(self.frame_weight):
            rs.weight[i] = w
        spans = {"bass_span": "chord_bass", "key_span": "key", "eighth_span": "eighth_position", "meter_span": "meter"}
        for field, block in spans.items():
            getattr(rs, field)[0], getattr(rs, field)[1] = vocab.start[block], vocab.end[block]
        rs.detail_span[0] = vocab.start["chord_detail"]
        rs.detail_span[1] = vocab.start["chord_detail"] + NO_CHORD
        rs.meter_beats, rs.meter_unit = self._meter[0].ctypes.data, self._meter[1].ctypes.data
        rs.time_hz = int(vocab.time_hz)
        _lib.check(self._lib.s2r_set_rescore(self._ctx, C.byref(rs)))

    def _load_frame_tables(self, slot: int, frame_logp) -> None:
        """Copy the window's frame tables (engine.py:218-224) into the engine."""

        frame_logp = frame_logp or {}
        ptrs = (C.c_void_p * len(FRAME_TERMS))()
        rows = (C.c_int32 * len(FRAME_TERMS))()
        keep = []
        for i, name in enumerate(FRAME_TERMS):
            if name not in frame_logp:
                continue
            t = frame_logp[name]
            t = t.detach() if isinstance(t, torch.Tensor) else torch.from_numpy(np.asarray(t))
            t = t.to(dtype=torch.float32)
            if t.is_cuda and t.device != self.device:
                t = t.to(self.device)
            t = t.contiguous()
            width = FRAME_WIDTHS[name]
            if tuple(t.shape[1:]) != ((width,) if width > 1 else ()):
                raise ValueError(f"frame table {name!r} has shape {tuple(t.shape)}; expected [frames{', %d' % width if width > 1 else ''}]")
            keep.append(t)
            ptrs[i], rows[i] = t.data_ptr(), t.shape[0]
        _lib.check(self._lib.s2r_load_frame_tables(self._ctx, slot, ptrs, rows, self._stream()))
        return keep

    # ------------------------------------------------------------ plumbing
    def _retain(self, sources) -> None:
        """Keep a load's source tensors alive until the stream has run the copies that read them.

        The engine copies ``memory`` and the frame tables asynchronously on the
        current stream, so a pinned host or device tensor that the caller drops
        right after ``load`` could otherwise be handed out again before the copy
        reads it.  Sources whose copies have completed are released here.
        """

        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream(self.device))
        self._inflight = [(e, s) for e, s in self._inflight if not e.query()]
        self._inflight.append((done, sources))

    def _view(self, name: str) -> torch.Tensor:
        ptr, numel, dtype = C.c_void_p(), C.c_int64(), C.c_int32()
        _lib.check(self._lib.s2r_get_buffer(self._ctx, name.encode(), C.byref(ptr), C.byref(numel), C.byref(dtype)))
        arr = _DeviceArray(ptr.value, (numel.value,), _TYPESTR[dtype.value])
        return torch.as_tensor(arr, device=self.device)

    def _stream(self) -> C.c_void_p:
        return C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def close(self) -> None:
        ctx = getattr(self, "_ctx", None)
        if ctx is not None and ctx.value:
            self._lib.s2r_destroy(ctx)
            self._ctx = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    @staticmethod
    def _versions(decoder) -> tuple:
        params = decoder.parameters()
        return tuple(getattr(p, "_version", 0) for p in params)

    def is_current(self, decoder, batch: int, frames: int, prompts, mode_bias=None, frame_weight=None) -> bool:
        """engine.py:155-174."""

        return (
            decoder is self.decoder
            and (mode_bias if "key_mode" in prompts else None) == self.mode_bias
            and frame_terms(frame_weight, prompts) == self.frame_weight
            and batch == self.batch
            and frames == self.frames
            and tuple(sorted(set(prompts))) == self.prompts
            and self._versions(decoder) == self.versions
        )

    # --------------------------------------------------------------- slots
    def free_slots(self) -> list[int]:
        return [slot for slot in range(self.batch) if not self.loaded[slot]]

    def load(self, slot: int, memory, prefix: list[int], stop_seconds: float | None, frames: int | None = None,
             frame_logp=None, target: int | None = None) -> None:
        """Start ``slot`` on a window (engine.py:180-232): ``memory`` ``[1, F, D]`` or ``[F, D]``."""

        frames = self.frames if frames is None else frames
        if isinstance(memory, np.ndarray):
            memory = torch.from_numpy(memory)
        mem = memory.detach().reshape(-1, self.config.width)
        if mem.dtype not in (torch.float32, torch.bfloat16):
            mem = mem.float()
        if mem.is_cuda and mem.device != self.device:
            mem = mem.to(self.device)
        mem = mem.contiguous()
        dtype = _lib.S2R_F32 if mem.dtype == torch.float32 else _lib.S2R_BF16
        if OUT not in prefix:
            raise ValueError("prefix must contain <out>")
        toks = (C.c_int64 * len(prefix))(*[int(t) for t in prefix])
        stop = float("inf") if stop_seconds is None else float(stop_seconds)
        tgt = _lib.S2R_NO_TARGET if target is None else int(target)
        tables = self._load_frame_tables(slot, frame_logp) if self.rescore else None
        _lib.check(self._lib.s2r_load_slot(self._ctx, slot, C.c_void_p(mem.data_ptr()), dtype, mem.shape[0], frames,
                                           toks, len(prefix), stop, tgt, self._stream()))
        self._retain((mem, tables))
        self.bound[slot], self.loaded[slot] = len(prefix) - 1, True

    def run(self, steps: int) -> None:
        """Advance every slot by ``steps`` tokens (engine.py:234-246)."""

        _lib.check(self._lib.s2r_step(self._ctx, int(steps), self._stream()))
        self.bound = [min(b + steps, self.max_tokens - 1) if on else b for b, on in zip(self.bound, self.loaded)]

    def step_debug(self, forced=None, want_logits: bool = True):
        """One step with teacher forcing; returns ``(raw logits [B, V], greedy [B])`` as numpy arrays."""

        logits = np.zeros((self.batch, self.config.vocab_size), np.float32) if want_logits else None
        greedy = np.zeros(self.batch, np.int64)
        f = None
        if forced is not None:
            f = np.ascontiguousarray(forced, np.int64)
        _lib.check(self._lib.s2r_step_debug(self._ctx, None if f is None else f.ctypes.data,
                                            None if logits is None else logits.ctypes.data, greedy.ctypes.data,
                                            self._stream()))
        self.bound = [min(b + 1, self.max_tokens - 1) if on else b for b, on in zip(self.bound, self.loaded)]
        return logits, greedy

    def finished(self) -> list[int]:
        """Loaded slots whose sequence has ended (synchronises; engine.py:248-252)."""

        done = np.zeros(self.batch, np.uint8)
        _lib.check(self._lib.s2r_poll_finished(self._ctx, done.ctypes.data, self._stream()))
        return [slot for slot in range(self.batch) if self.loaded[slot] and done[slot]]

    def take(self, slot: int) -> tuple[list[int], str]:
        """A finished slot's tokens (ending in <eos>) and why it ended; frees the slot (engine.py:254-262)."""

        cap = self.max_tokens + 1
        buf = (C.c_int64 * cap)()
        length, ended = C.c_int32(), C.c_int32()
        _lib.check(self._lib.s2r_take(self._ctx, slot, buf, cap, C.byref(length), C.byref(ended), self._stream()))
        self.loaded[slot] = False
        return list(buf[: length.value]), ENDED[ended.value]

    # ------------------------------------------------- asynchronous polling
    def finished_async(self) -> None:
        """Queue a copy of the finished flags behind the steps already queued; returns at once.

        ``finished_ready`` reads it.  A scheduler can queue the next steps in
        between, so the device never waits for the host's poll (the
        reference's ``finished`` synchronises, engine.py:248-252).
        """

        _lib.check(self._lib.s2r_poll_finished_async(self._ctx, self._stream()))

    def finished_ready(self, wait: bool = False) -> list[int] | None:
        """Loaded slots finished as of the last ``finished_async``, or None while its copy is queued.

        With ``wait`` it blocks until that copy lands (not for later steps).
        """

        done = np.zeros(self.batch, np.uint8)
        ready = C.c_int32()
        _lib.check(self._lib.s2r_poll_finished_ready(self._ctx, done.ctypes.data, int(wait), C.byref(ready)))
        if not ready.value:
            return None
        return [slot for slot in range(self.batch) if self.loaded[slot] and done[slot]]

    def take_async(self, slot: int) -> None:
        """Queue the copy of a slot's tokens and free the slot at once (``take_ready`` reads them).

        A ``load`` of the slot issued afterwards on the same stream runs after the copy.
        """

        _lib.check(self._lib.s2r_take_async(self._ctx, slot, self._stream()))
        self.loaded[slot] = False

    def take_ready(self, slot: int, wait: bool = False) -> tuple[list[int], str] | None:
        """The ``(tokens, ended)`` of the slot's ``take_async``, or None while its copy is queued."""

        cap = self.max_tokens + 1
        buf = (C.c_int64 * cap)()
        length, ended, ready = C.c_int32(), C.c_int32(), C.c_int32()
        _lib.check(self._lib.s2r_take_ready(self._ctx, slot, buf, cap, C.byref(length), C.byref(ended), int(wait),
                                            C.byref(ready)))
        if not ready.value:
            return None
        return list(buf[: length.value]), ENDED[ended.value]

    # ------------------------------------------------------------ extras
    @property
    def step_launches(self) -> int:
        """Kernel launches one step issues."""

        return int(self._lib.s2r_step_launches(self._ctx))

    @property
    def free_pages(self) -> int:
        return int(self._lib.s2r_free_pages(self._ctx))
