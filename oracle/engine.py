"""The batched greedy decode engine restated in numpy (test infrastructure).

The ``fp32`` mode (the reference CPU path) runs its matrix products through
torch's CPU kernels, as that path does; everything else, and the whole
``bf16`` mode, is numpy.

``OracleEngine`` mirrors ``sheetsage2_refined/engine.py:52-369``:
construction (55-149), ``load`` (180-232), ``run`` (234-246), ``finished``
(248-252), ``take`` (254-262), the step ``_forward`` (294-357) and the
frame-head rescoring terms and state (81-116, 218-232, 318-347, 358-369).  ``step(forced=...)`` additionally lets a test force the
committed token per slot (teacher forcing) and returns the raw logits.

The decoder forward is ``TokenDecoder`` (decoder.py:58-151) evaluated one
token per row against the per-slot caches; the prefix prefill of ``load``
(engine.py:199-207, decoder.py:118-151) is evaluated as the same single-token
forward over the prefix positions in order, which equals the reference's
causal forward up to float32 summation order.
"""

from __future__ import annotations

import numpy as np
import torch

from sheetsage2_refined_b200.grammar import ENDED
from sheetsage2_refined_b200.vocab_table import EOS, NO_CHORD, OUT, meter_tables
from sheetsage2_refined_b200.weights import POSITION_OFFSET

from .grammar import make_grammar_oracle
from .numerics import bf16, gelu, layer_norm, softmax


# FRAME_TERMS order (engine.py:29-38)
FRAME_TERM_NAMES = ("root", "bass", "detail", "quality", "key", "key_boundary", "downbeat", "meter")
AFTER_METER = 1  # incomplete-field state after a meter token (grammar.py, AFTER_METER)


class OracleEngine:
    # prefixes with at least this many tokens before the last are prefilled with batched products
    BATCHED_PREFILL = 16

    def __init__(self, config, state_dict: dict, grammar, *, batch: int, frames: int, mode: str = "bf16",
                 logit_bias: np.ndarray | None = None, frame_weight: tuple | None = None, vocab=None):
        if mode not in ("fp32", "bf16"):
            raise ValueError(mode)
        self.config, self.mode, self.batch, self.frames = config, mode, batch, frames
        self.max_tokens = config.max_tokens
        self.heads, self.head_dim = config.heads, config.width // config.heads
        rnd = bf16 if mode == "bf16" else (lambda a: np.asarray(a, np.float32))
        self._round = rnd
        sd = {k: np.asarray(v, np.float32) for k, v in state_dict.items()}
        # Linear weights as the engine holds them (engine.py:118-123): bf16 copies on CUDA.
        self.lin = {}
        for i in range(config.layers):
            p = f"layers.{i}."
            for name in ("self_attn.q", "self_attn.k", "self_attn.v", "self_attn.out",
                         "cross_attn.q", "cross_attn.k", "cross_attn.v", "cross_attn.out", "fc1", "fc2"):
                w, b = sd[f"{p}{name}.weight"], sd[f"{p}{name}.bias"]
                self.lin[(i, name)] = (np.ascontiguousarray(rnd(w).T), rnd(b))
            for norm in ("self_attn_norm", "cross_attn_norm", "final_norm"):
                self.lin[(i, norm)] = (sd[f"{p}{norm}.weight"], sd[f"{p}{norm}.bias"])
        self.tok_emb = sd["token_embedding.weight"]  # the lookup stays fp32 (engine.py:298-301)
        self.pos_emb = sd["position_embedding.weight"]
        self.emb_norm = (sd["embedding_norm.weight"], sd["embedding_norm.bias"])
        self.out_emb_t = np.ascontiguousarray(rnd(self.tok_emb).T)  # tied logits (engine.py:123,315)
        # fp32 mode runs its matrix products through torch's CPU kernels, as the
        # reference CPU path does (one thread pool for every product)
        self._t = None
        if mode == "fp32":
            self._t = {key: (torch.from_numpy(wt), torch.from_numpy(b)) for key, (wt, b) in self.lin.items()
                       if not key[1].endswith("_norm")}
            self._t["logits"] = torch.from_numpy(self.out_emb_t)
        # bf16 mode: the same bf16 weights as torch tensors, for the products of many rows at once
        self._tw = {key: torch.from_numpy(wt) for key, (wt, b) in self.lin.items() if not key[1].endswith("_norm")}
        self.grammar = make_grammar_oracle(grammar)
        self.logit_bias = None if logit_bias is None else np.asarray(logit_bias, np.float32)

        H, hd, L = self.heads, self.head_dim, config.layers
        self.self_k = [np.zeros((batch, H, self.max_tokens, hd), np.float32) for _ in range(L)]
        self.self_v = [np.zeros((batch, H, self.max_tokens, hd), np.float32) for _ in range(L)]
        self.cross_k = [np.zeros((batch, H, frames, hd), np.float32) for _ in range(L)]
        self.cross_v = [np.zeros((batch, H, frames, hd), np.float32) for _ in range(L)]
        self.frames_real = np.full(batch, frames, np.int64)
        self.out = np.zeros((batch, self.max_tokens), np.int64)
        self.state = self.grammar.new_state(batch)
        self.state["finished"][:] = True
        self.state["token"] = np.full(batch, EOS, np.int64)
        self.state["position"] = np.zeros(batch, np.int64)
        self.stop = np.full(batch, np.inf, np.float64)
        self.loaded = [False] * batch
        # frame-head rescoring (engine.py:81-116): weights in FRAME_TERMS order
        self.frame_weight = tuple(frame_weight) if frame_weight is not None else (0.0,) * 8
        self.rescore = any(self.frame_weight)
        if self.rescore:
            sizes = {"root": 12, "bass": 12, "detail": NO_CHORD, "quality": NO_CHORD, "key": 24, "meter": 16}
            self.frame = {name: np.zeros((batch, frames) + ((sizes[name],) if name in sizes else ()), np.float32)
                          for name in FRAME_TERM_NAMES}
            self.frame_now = np.zeros(batch, np.int64)
            self.key_seen = np.zeros(batch, bool)
            self.root_of_detail = np.arange(NO_CHORD) % 12
            self.key_span = (vocab.start["key"], vocab.end["key"])
            self.eighth_span = (vocab.start["eighth_position"], vocab.end["eighth_position"])
            self.meter_span = (vocab.start["meter"], vocab.end["meter"])
            beats, units = meter_tables()
            self.meter_beats, self.meter_unit = np.array(beats), np.array(units)
            self.active_meter = np.full(batch, -1, np.int64)
            self.meter_changed = np.zeros(batch, bool)
            self.meter_index = np.arange(len(beats))
            self.time_hz = vocab.time_hz
            self.bass_span = (vocab.start["chord_bass"], vocab.end["chord_bass"])
            self.detail_span = (vocab.start["chord_detail"], vocab.start["chord_detail"] + NO_CHORD)

    # ------------------------------------------------------------ numerics
    def _linear(self, layer: int, name: str, x: np.ndarray) -> np.ndarray:
        if self._t is not None:
            wt, b = self._t[(layer, name)]
            return (torch.from_numpy(np.ascontiguousarray(x, np.float32)) @ wt + b).numpy()
        wt, b = self.lin[(layer, name)]
        xr = self._round(x)
        if xr.ndim == 2 and xr.shape[0] > 8:  # many rows: torch's threaded product (float32 accumulation)
            return self._round((torch.from_numpy(xr) @ self._tw[(layer, name)]).numpy() + b)
        return self._round(xr @ wt + b)

    def _split(self, y: np.ndarray) -> np.ndarray:
        return y.reshape(self.heads, self.head_dim)

    def _attend(self, q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
        """engine.py:286-292 for one row: q ``[H, hd]``, k/v ``[H, n, hd]`` (only the visible keys)."""

        scale = np.float32(self.head_dim ** -0.5)
        if self.mode == "fp32":
            # the reference CPU path's batched matmuls (bmm over the heads)
            q_t = torch.from_numpy(np.ascontiguousarray(q, np.float32))
            scores = torch.bmm(torch.from_numpy(k), q_t[:, :, None])[..., 0].numpy() * scale
            p_t = torch.from_numpy(softmax(scores))
            return torch.bmm(p_t[:, None, :], torch.from_numpy(v))[:, 0, :].numpy().reshape(-1)
        rnd = self._round
        scores = rnd(np.einsum("hd,hnd->hn", q, k)) * scale
        p = rnd(softmax(scores))
        return rnd(np.einsum("hn,hnd->hd", p, v)).reshape(-1)

    def _row_forward(self, slot: int, token: int, position: int) -> np.ndarray:
        """Final hidden state (fp32) of one token at ``position`` of ``slot``; writes its K/V."""

        x = self.tok_emb[token] + self.pos_emb[position + POSITION_OFFSET]
        x = layer_norm(x, *self.emb_norm)
        n_cross = int(self.frames_real[slot])
        for i in range(self.config.layers):
            k = self._split(self._linear(i, "self_attn.k", x))
            v = self._split(self._linear(i, "self_attn.v", x))
            self.self_k[i][slot, :, position] = k
            self.self_v[i][slot, :, position] = v
            q = self._split(self._linear(i, "self_attn.q", x))
            a = self._attend(q, self.self_k[i][slot, :, : position + 1], self.self_v[i][slot, :, : position + 1])
            x = layer_norm(x + self._linear(i, "self_attn.out", a), *self.lin[(i, "self_attn_norm")])
            q = self._split(self._linear(i, "cross_attn.q", x))
            a = self._attend(q, self.cross_k[i][slot, :, :n_cross], self.cross_v[i][slot, :, :n_cross])
            x = layer_norm(x + self._linear(i, "cross_attn.out", a), *self.lin[(i, "cross_attn_norm")])
            h = self._round(gelu(self._linear(i, "fc1", x)))
            x = layer_norm(x + self._linear(i, "fc2", h), *self.lin[(i, "final_norm")])
        return x

    def _attend_rows(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, first: int | None) -> np.ndarray:
        """engine.py:286-292 for many query rows: q ``[H, n, hd]``, k/v ``[H, m, hd]``.

        ``first`` is the position of the first query row of a causal block
        (row i sees keys ``0 .. first + i``), or None for cross-attention
        (every row sees every key).  The same arithmetic as ``_attend`` (the
        softmax in float64, rounded to float32), evaluated with torch's CPU
        kernels on blocks of rows so that the score matrix stays small.
        Returns ``[n, H * hd]``.
        """

        H, n, hd = q.shape
        scale = hd ** -0.5
        bf = self.mode == "bf16"

        def rnd(t):
            return t.to(torch.bfloat16).to(torch.float32) if bf else t

        out = np.empty((n, H * hd), np.float32)
        qt, kt, vt = (torch.from_numpy(np.ascontiguousarray(a, np.float32)) for a in (q, k, v))
        block = 512
        for r0 in range(0, n, block):
            r1 = min(n, r0 + block)
            m = kt.shape[1] if first is None else first + r1
            scores = rnd(torch.bmm(qt[:, r0:r1], kt[:, :m].transpose(1, 2))) * np.float32(scale)
            if first is not None:
                rows = torch.arange(r0, r1)[:, None] + first
                scores = scores.masked_fill(torch.arange(m)[None, :] > rows, float("-inf"))
            p = torch.softmax(scores.double(), dim=-1).float()
            o = rnd(torch.bmm(rnd(p), vt[:, :m]))
            out[r0:r1] = o.transpose(0, 1).reshape(r1 - r0, H * hd).numpy()
        return out

    def _prefill_rows(self, slot: int, tokens: list[int]) -> None:
        """The prefix prefill of ``load`` (engine.py:199-205, decoder.py:118-151) for positions
        ``0 .. len(tokens)-1`` of ``slot`` at once: the same arithmetic as ``_row_forward`` per
        row, with the rows' matrix products batched (float32 summation order aside)."""

        n, H, hd = len(tokens), self.heads, self.head_dim
        x = self.tok_emb[np.asarray(tokens)] + self.pos_emb[np.arange(n) + POSITION_OFFSET]
        x = layer_norm(x, *self.emb_norm)
        n_cross = int(self.frames_real[slot])

        def heads(y):
            return np.ascontiguousarray(y.reshape(n, H, hd).transpose(1, 0, 2))

        for i in range(self.config.layers):
            k, v = heads(self._linear(i, "self_attn.k", x)), heads(self._linear(i, "self_attn.v", x))
            self.self_k[i][slot, :, :n] = k
            self.self_v[i][slot, :, :n] = v
            q = heads(self._linear(i, "self_attn.q", x))
            a = self._attend_rows(q, self.self_k[i][slot], self.self_v[i][slot], first=0)
            x = layer_norm(x + self._linear(i, "self_attn.out", a), *self.lin[(i, "self_attn_norm")])
            q = heads(self._linear(i, "cross_attn.q", x))
            a = self._attend_rows(q, self.cross_k[i][slot, :, :n_cross], self.cross_v[i][slot, :, :n_cross], None)
            x = layer_norm(x + self._linear(i, "cross_attn.out", a), *self.lin[(i, "cross_attn_norm")])
            h = self._round(gelu(self._linear(i, "fc1", x)))
            x = layer_norm(x + self._linear(i, "fc2", h), *self.lin[(i, "final_norm")])

    def _logits(self, x: np.ndarray) -> np.ndarray:
        if self._t is not None:
            return (torch.from_numpy(np.ascontiguousarray(x, np.float32)) @ self._t["logits"]).numpy()
        return self._round(self._round(x) @ self.out_emb_t).astype(np.float32)

    # --------------------------------------------------------------- slots
    def free_slots(self) -> list[int]:
        return [s for s in range(self.batch) if not self.loaded[s]]

    def load(self, slot: int, memory, prefix: list[int], stop_seconds, frames: int | None = None,
             target: int | None = None, frame_logp: dict | None = None) -> None:
        """engine.py:180-232; ``target`` feeds the table grammar."""

        memory = np.asarray(memory, np.float32).reshape(-1, self.config.width)
        frames = self.frames if frames is None else frames
        n = len(prefix)
        for i in range(self.config.layers):
            # decoder.py:108-113 — cross K/V of every memory frame, projected once per window
            k = self._linear(i, "cross_attn.k", memory[: self.frames])
            v = self._linear(i, "cross_attn.v", memory[: self.frames])
            f = k.shape[0]
            self.cross_k[i][slot] = 0.0
            self.cross_v[i][slot] = 0.0
            self.cross_k[i][slot, :, :f] = k.reshape(f, self.heads, self.head_dim).transpose(1, 0, 2)
            self.cross_v[i][slot, :, :f] = v.reshape(f, self.heads, self.head_dim).transpose(1, 0, 2)
        self.frames_real[slot] = frames
        if n - 1 >= self.BATCHED_PREFILL:  # prefix prefill (engine.py:200-205)
            self._prefill_rows(slot, list(prefix[: n - 1]))
        else:
            for pos in range(n - 1):
                self._row_forward(slot, prefix[pos], pos)
        self.out[slot, :n] = prefix
        for name, value in self.grammar.prefix_state(prefix, prefix.index(OUT)).items():
            self.state[name][slot] = value[0]
        if target is not None and "target" in self.state:
            self.state["target"][slot] = target
        self.state["token"][slot] = prefix[-1]
        self.state["position"][slot] = n - 1
        self.stop[slot] = np.inf if stop_seconds is None else stop_seconds
        self.loaded[slot] = True
        if self.rescore:  # engine.py:218-232
            frame_logp = frame_logp or {}
            for name, table in self.frame.items():
                table[slot] = 0.0
                if name in frame_logp:
                    count = min(len(frame_logp[name]), self.frames)
                    table[slot, :count] = np.asarray(frame_logp[name], np.float32)[:count]
            seconds = self.grammar.time_seconds
            times = [float(seconds[t]) for t in prefix if seconds[t] > float("-inf")]
            self.frame_now[slot] = (min(int(times[-1] * self.time_hz) * 25 // self.time_hz, self.frames - 1)
                                    if times else 0)
            self.key_seen[slot] = any(self.key_span[0] <= t < self.key_span[1] for t in prefix)
            m0, m1 = self.meter_span
            meters = [t - m0 for t in prefix if m0 <= t < m1]
            self.active_meter[slot] = meters[-1] if meters else -1
            self.meter_changed[slot] = False

    def _rescore_logits(self, logits: np.ndarray) -> None:
        """engine.py:318-347 in place: the frame-head terms of every row."""

        st, rows = self.state, np.arange(self.batch)
        (b0, b1), (d0, d1), (k0, k1) = self.bass_span, self.detail_span, self.key_span
        w, now, frame = dict(zip(FRAME_TERM_NAMES, self.frame_weight)), self.frame_now, self.frame
        if w["root"]:
            logits[:, d0:d1] += w["root"] * frame["root"][rows, now][:, self.root_of_detail]
        if w["detail"]:
            logits[:, d0:d1] += w["detail"] * frame["detail"][rows, now]
        if w["quality"]:
            logits[:, d0:d1] += w["quality"] * frame["quality"][rows, now]
        if w["bass"]:
            logits[:, b0:b1] += w["bass"] * frame["bass"][rows, now]
        if w["key"]:
            logits[:, k0:k1] += w["key"] * frame["key"][rows, now]
        if w["key_boundary"]:
            stated = self.key_seen.astype(np.float32)
            logits[:, k0:k1] += (w["key_boundary"] * frame["key_boundary"][rows, now] * stated)[:, None]
        if w["downbeat"]:
            logits[:, self.eighth_span[0]] += w["downbeat"] * frame["downbeat"][rows, now]
        if w["meter"]:
            (m0, m1), (e0, e1) = self.meter_span, self.eighth_span
            table = frame["meter"][rows, now]
            active = np.maximum(self.active_meter, 0)
            change = (self.active_meter >= 0)[:, None] & (self.meter_index[None] != active[:, None])
            current = np.take_along_axis(table, self.meter_beats[active][:, None], axis=1)
            same_unit = self.meter_unit[None] == self.meter_unit[active][:, None]
            logits[:, m0:m1] += w["meter"] * (table[:, self.meter_beats] - current) * (change & same_unit)
            if w["downbeat"]:
                logits[:, m0:m1] += w["downbeat"] * frame["downbeat"][rows, now][:, None] * change
            after = (st["incomplete"] == AFTER_METER) & self.meter_changed
            logits[:, e0 + 1: e1][after] = -np.inf

    def _rescore_commit(self, choice: np.ndarray, active: np.ndarray) -> None:
        """engine.py:358-369: the rescoring state after the step's tokens."""

        seconds = self.grammar.time_seconds[choice]
        with np.errstate(invalid="ignore"):
            frame = np.clip(np.where(np.isfinite(seconds), seconds * 25, 0).astype(np.int64), 0, self.frames - 1)
        self.frame_now[:] = np.where(active & (seconds > float("-inf")), frame, self.frame_now)
        k0, k1 = self.key_span
        self.key_seen |= active & (choice >= k0) & (choice < k1)
        m0, m1 = self.meter_span
        is_meter = active & (choice >= m0) & (choice < m1)
        meter = np.clip(choice - m0, 0, m1 - m0 - 1)
        changed = (self.active_meter >= 0) & (meter != self.active_meter)
        self.meter_changed[:] = np.where(is_meter, changed, self.meter_changed)
        self.active_meter[:] = np.where(is_meter, meter, self.active_meter)

    def step(self, forced: np.ndarray | None = None):
        """One step (engine.py:294-357). Returns ``(raw logits [B, V], greedy choice [B])``.

        ``forced[slot] >= 0`` commits that token instead of the greedy one
        (teacher forcing); rows that are finished are not evaluated.
        """

        st = self.state
        token, position = st["token"], st["position"]
        active = ~st["finished"]
        logits = np.zeros((self.batch, self.grammar.vocab_size), np.float32)
        for slot in np.nonzero(active)[0]:
            x = self._row_forward(int(slot), int(token[slot]), int(position[slot]))
            logits[slot] = self._logits(x)
        biased = logits.copy() if self.logit_bias is None else logits + self.logit_bias
        if self.rescore:
            self._rescore_logits(biased)
        masked = np.where(self.grammar.allowed(st), biased, -np.inf)
        self.last_masked = masked  # what the argmax saw (tests read it to judge near-ties)
        greedy = masked.argmax(axis=-1)
        choice = greedy.copy()
        if forced is not None:
            choice = np.where(np.asarray(forced) >= 0, forced, choice)
        choice = np.where(active, choice, token)
        new_position = np.where(active, position + 1, position)
        rows = np.arange(self.batch)
        self.out[rows, new_position] = np.where(active, choice, self.out[rows, new_position])
        self.grammar.update(st, choice, active, self.stop, new_position >= self.max_tokens - 1)
        if self.rescore:
            self._rescore_commit(choice, active)
        token[...] = choice
        position[...] = new_position
        return logits, greedy

    def run(self, steps: int) -> None:
        for _ in range(steps):
            self.step()

    def finished(self) -> list[int]:
        return [s for s in range(self.batch) if self.loaded[s] and self.state["finished"][s]]

    def take(self, slot: int) -> tuple[list[int], str]:
        """engine.py:254-262."""

        length = int(self.state["position"][slot]) + 1
        tokens = self.out[slot, :length].tolist()
        if tokens[-1] != EOS:
            tokens.append(EOS)
        self.loaded[slot] = False
        return tokens, ENDED[int(self.state["ended"][slot])]
