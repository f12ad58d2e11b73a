"""Grammar descriptors for the device decode step.

Two grammars drive token selection inside the fused logits kernel:

* ``ClassGrammar`` — the event grammar of SheetSage2-Refined
  (``sheetsage2_refined/grammar.py:78-197``): every vocabulary token belongs
  to one of 13 classes (``TYPES`` grammar.py:22-36); the per-slot state
  (``in_shift, shift_run, payload, last_field, incomplete``) decides which
  classes may come next (``allowed`` grammar.py:114-138) and is advanced by the
  chosen token (``update`` grammar.py:140-180).  On the device the mask is
  never materialised: the kernel evaluates the 13 class predicates once per
  row and gathers them through ``token_class``.
* ``TableGrammar`` — a synthetic grammar for vocabularies that are not the
  real one: ``states`` states, a seeded Bernoulli(``density``) table of allowed
  tokens per state (the four special tokens, EOS included, are never allowed),
  the transition ``s' = (multiplier * s + token) mod states``, and a per-slot
  target count of generated tokens after which the slot ends with reason
  ``eos``.  It plugs into the reference engine through the same duck type as
  ``TokenGrammar`` (``allowed/update/prefix_state/time_seconds/prompts``).

Both are plain host descriptors (numpy arrays); the engine copies them to the
device once at construction.
"""

from __future__ import annotations

import numpy as np

from . import vocab_table as vt

# Token classes (grammar.py:22-50).
TYPES = (
    "eos",
    "shift",
    "time",
    "meter",
    "eighth_position",
    "structure",
    "key",
    "chord",
    "pitch",
    "duration",
    "chord_bass",
    "chord_detail",
)
OTHER = len(TYPES)
(
    EOS_T,
    SHIFT_T,
    TIME_T,
    METER_T,
    EIGHTH_T,
    STRUCTURE_T,
    KEY_T,
    CHORD_T,
    PITCH_T,
    DURATION_T,
    BASS_T,
    DETAIL_T,
) = range(len(TYPES))
# Field opened by each class (grammar.py:52).
FIELD_OF_TYPE = (-1, -1, 0, 1, 1, 2, 3, 4, 5, 5, 4, 4, -1)
# "incomplete" states (grammar.py:54).
NONE, AFTER_METER, AFTER_PITCH, AFTER_BASS = range(4)
MAX_SHIFT_RUN = 4  # grammar.py:55

# Token blocks each prompt enables (grammar.py:58-73).
PROMPT_BLOCKS = {
    "timestamp": (("time", None, TIME_T),),
    "downbeat_meter": (("meter", None, METER_T), ("eighth_position", None, EIGHTH_T)),
    "structure": (("structure", None, STRUCTURE_T),),
    "key": (("key", None, KEY_T),),
    "key_mode": (("key_mode", None, KEY_T),),
    "chord_majmin": (("chord_majmin", None, CHORD_T),),
    "chord_full": (("chord_full", None, CHORD_T),),
    "chord_detail": (
        ("chord_bass", None, BASS_T),
        ("chord_detail", (0, vt.NO_CHORD), DETAIL_T),
        ("chord_detail", (vt.NO_CHORD, vt.NO_CHORD + 1), CHORD_T),
    ),
    "melody_vocal": (("pitch", (0, 128), PITCH_T), ("duration", None, DURATION_T)),
    "melody_full": (("pitch", None, PITCH_T), ("duration", None, DURATION_T)),
}

ENDED = ("running", "eos", "stop", "limit")  # grammar.py:75

GRAMMAR_CLASS = 0
GRAMMAR_TABLE = 1


class ClassGrammar:
    """Device descriptor of ``TokenGrammar`` (grammar.py:79-97).

    ``token_class[v]`` is the class of token ``v`` for the requested prompts
    (blocks of prompts not requested stay ``OTHER`` and are never allowed);
    ``time_seconds[v]`` is the time of a time token in float64 seconds and
    ``-inf`` for every other token.  Raises ``ValueError`` for an invalid
    prompt set, like the reference.
    """

    kind = GRAMMAR_CLASS

    def __init__(self, vocab, prompts=vt.FULL_PROMPTS):
        self.prompts = tuple(sorted(set(prompts)))
        vocab.prompt_prefix(prompts)  # validates the prompt set
        token_class = np.full(vocab.size, OTHER, dtype=np.int8)
        token_class[vt.EOS] = EOS_T
        token_class[vocab.start["shift"] : vocab.end["shift"]] = SHIFT_T
        for prompt in self.prompts:
            for block, span, kind in PROMPT_BLOCKS[prompt]:
                first, last = span or (0, vocab.end[block] - vocab.start[block])
                token_class[vocab.start[block] + first : vocab.start[block] + last] = kind
        self.vocab_size = vocab.size
        self.token_class = token_class
        self.field_of_class = np.asarray(FIELD_OF_TYPE, dtype=np.int32)
        seconds = np.full(vocab.size, -np.inf, dtype=np.float64)
        count = vocab.end["time"] - vocab.start["time"]
        seconds[vocab.start["time"] : vocab.end["time"]] = np.arange(count, dtype=np.float64) / vocab.time_hz
        self.time_seconds = seconds
        self.states = 0
        self.table = None
        self.multiplier = 0


class TableGrammar:
    """Synthetic table grammar for vocabularies other than the real one.

    ``table[s, v]`` (bool ``[states, vocab_size]``) is True where token ``v``
    may follow state ``s``; it is drawn as ``numpy.random.default_rng(seed)
    .random((states, vocab_size)) < density``, then the four special tokens
    (PAD, SOS, EOS, OUT) are cleared and a state left with no allowed token
    gets token 4.  The state after token ``t`` is ``(multiplier * s + t) mod
    states``; the state after ``<out>`` is 0.  A slot ends (reason ``eos``)
    once it has generated its target number of tokens, or with ``limit`` when
    the context is full.  No token is a time token.
    """

    kind = GRAMMAR_TABLE

    def __init__(self, vocab_size: int, states: int = 8, density: float = 0.25, seed: int = 0, multiplier: int = 31):
        if states < 1 or vocab_size <= 4:
            raise ValueError("a table grammar needs at least one state and more than 4 tokens")
        rng = np.random.default_rng(seed)
        table = rng.random((states, vocab_size)) < density
        table[:, :4] = False
        empty = ~table.any(axis=1)
        table[empty, 4] = True
        self.vocab_size = vocab_size
        self.states = states
        self.density = density
        self.seed = seed
        self.multiplier = multiplier
        self.table = table
        self.prompts = ("table",)
        self.time_seconds = np.full(vocab_size, -np.inf, dtype=np.float64)
        self.token_class = None
        self.field_of_class = None

    def next_state(self, state: int, token: int) -> int:
        return (self.multiplier * state + token) % self.states
