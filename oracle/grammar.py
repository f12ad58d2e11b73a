"""Grammar state machines restated in numpy (test infrastructure).

``ClassGrammarOracle`` follows ``sheetsage2_refined/grammar.py``:
``new_state`` 99-112, ``allowed`` 114-138, ``update`` 140-180,
``prefix_state`` 182-197.  ``TableGrammarOracle`` restates the synthetic
table grammar whose rule is documented in ``sheetsage2_refined_b200.grammar``.

States are dicts of numpy arrays with the reference's names and dtypes
(bool for ``in_shift``/``finished``, int64 for the rest).
"""

from __future__ import annotations

import numpy as np

from sheetsage2_refined_b200.grammar import (
    AFTER_BASS,
    AFTER_METER,
    AFTER_PITCH,
    BASS_T,
    EOS_T,
    MAX_SHIFT_RUN,
    METER_T,
    NONE,
    PITCH_T,
    SHIFT_T,
    TIME_T,
)


class ClassGrammarOracle:
    def __init__(self, desc):
        self.token_class = desc.token_class.astype(np.int64)
        self.field_of_class = desc.field_of_class.astype(np.int64)
        self.time_seconds = desc.time_seconds
        self.prompts = desc.prompts
        self.vocab_size = desc.vocab_size

    @staticmethod
    def new_state(batch: int) -> dict:
        """grammar.py:99-112 — the state after ``<out>``."""

        return {
            "in_shift": np.ones(batch, bool),
            "shift_run": np.zeros(batch, np.int64),
            "payload": np.zeros(batch, np.int64),
            "last_field": np.full(batch, -1, np.int64),
            "incomplete": np.full(batch, NONE, np.int64),
            "finished": np.zeros(batch, bool),
            "ended": np.zeros(batch, np.int64),
        }

    def class_mask(self, state: dict) -> np.ndarray:
        """``[B, 13]`` class predicates (grammar.py:117-137)."""

        last, incomplete = state["last_field"], state["incomplete"]
        free = incomplete == NONE
        open_chord = incomplete == AFTER_BASS
        payload, in_shift, run = state["payload"], state["in_shift"], state["shift_run"]
        return np.stack(
            [
                (payload > 0) & ~open_chord,
                ((payload > 0) | in_shift) & (run < MAX_SHIFT_RUN) & ~open_chord,
                free & (last < 0),
                free & (last < 1),
                (incomplete == AFTER_METER) | (free & (last < 1)),
                free & (last < 2),
                free & (last < 3),
                free & (last < 4),
                (incomplete == AFTER_PITCH) | (free & (last <= 5)),
                incomplete == AFTER_PITCH,
                free & (last < 4),
                open_chord,
                np.zeros_like(free),
            ],
            axis=1,
        )

    def allowed(self, state: dict) -> np.ndarray:
        """grammar.py:114-138 — ``[B, vocab]`` bool mask."""

        return self.class_mask(state)[:, self.token_class]

    def update(self, state: dict, tokens, active, stop, at_limit) -> None:
        """grammar.py:140-180 — consume ``tokens`` for the ``active`` rows, in place."""

        tokens = np.asarray(tokens, np.int64)
        kind = self.token_class[tokens]
        is_shift = kind == SHIFT_T
        is_field = (kind != SHIFT_T) & (kind != EOS_T)
        new_event = is_shift & ~state["in_shift"] & (state["payload"] > 0)
        payload = np.where(new_event, 0, state["payload"])
        payload = np.where(is_field, payload + 1, payload)
        last = np.where(new_event, -1, state["last_field"])
        last = np.where(is_field, self.field_of_class[kind], last)
        incomplete = np.where(new_event, NONE, state["incomplete"])
        follows = (kind == METER_T) * AFTER_METER + (kind == PITCH_T) * AFTER_PITCH + (kind == BASS_T) * AFTER_BASS
        incomplete = np.where(is_field, follows, incomplete)
        in_shift = np.where(is_shift, True, np.where(is_field, False, state["in_shift"]))
        shift_run = np.where(is_shift, state["shift_run"] + 1, np.where(is_field, 0, state["shift_run"]))
        eos = kind == EOS_T
        stopped = (kind == TIME_T) & (self.time_seconds[tokens] >= stop)
        ended = np.where(eos, 1, np.where(stopped, 2, np.where(at_limit, 3, 0)))
        finished = eos | stopped | at_limit
        for name, value in (
            ("payload", payload),
            ("last_field", last),
            ("incomplete", incomplete),
            ("in_shift", in_shift),
            ("shift_run", shift_run),
        ):
            state[name][...] = np.where(active, value, state[name])
        state["ended"][...] = np.where(active & finished, ended, state["ended"])
        state["finished"][...] = state["finished"] | (active & finished)

    def prefix_state(self, tokens: list[int], out_index: int) -> dict:
        """grammar.py:182-197 — replay the tokens after ``<out>`` from ``new_state``."""

        state = self.new_state(1)
        never = np.zeros(1, bool)
        for token in tokens[out_index + 1 :]:
            self.update(state, np.array([token]), ~never, np.array([np.inf]), never)
        return state


class TableGrammarOracle:
    def __init__(self, desc):
        self.table = np.asarray(desc.table, bool)
        self.states = desc.states
        self.multiplier = desc.multiplier
        self.time_seconds = desc.time_seconds
        self.prompts = desc.prompts
        self.vocab_size = desc.vocab_size

    @staticmethod
    def new_state(batch: int) -> dict:
        return {
            "g": np.zeros(batch, np.int64),
            "count": np.zeros(batch, np.int64),
            "target": np.full(batch, np.iinfo(np.int64).max, np.int64),
            "finished": np.zeros(batch, bool),
            "ended": np.zeros(batch, np.int64),
        }

    def allowed(self, state: dict) -> np.ndarray:
        return self.table[state["g"]]

    def update(self, state: dict, tokens, active, stop, at_limit) -> None:
        tokens = np.asarray(tokens, np.int64)
        g = (self.multiplier * state["g"] + tokens) % self.states
        count = state["count"] + 1
        done = count >= state["target"]
        ended = np.where(done, 1, np.where(at_limit, 3, 0))
        finished = done | at_limit
        state["g"][...] = np.where(active, g, state["g"])
        state["count"][...] = np.where(active, count, state["count"])
        state["ended"][...] = np.where(active & finished, ended, state["ended"])
        state["finished"][...] = state["finished"] | (active & finished)

    def prefix_state(self, tokens: list[int], out_index: int) -> dict:
        state = self.new_state(1)
        for token in tokens[out_index + 1 :]:
            state["g"][0] = (self.multiplier * state["g"][0] + token) % self.states
        return state


def make_grammar_oracle(desc):
    return TableGrammarOracle(desc) if desc.table is not None else ClassGrammarOracle(desc)
