"""The SheetSage2-Refined token vocabulary as a block table.

Only what the decode step needs on the device is restated here: the block
layout (start/end of each token block), the special token ids and the prompt
prefix rule.  Event (de)serialisation stays with the reference package on the
host.

Reference: ``sheetsage2_refined/vocab.py``

* special ids ``PAD, SOS, EOS, OUT`` — vocab.py:27
* prompt names and their groups — vocab.py:30-41, ``FULL_PROMPTS`` vocab.py:44
* ``FIELDS`` (canonical field order) — vocab.py:47
* block sizes — vocab.py:160-178; the sizes that come from ``theory.py`` are
  written out as numbers: 192 meters (vocab.py:64), 23 structure labels
  (vocab.py:65-89), 25 maj/min chords (vocab.py:90), 361 full chords
  (vocab.py:115-123), 24 durations (vocab.py:125-150), ``NO_CHORD`` = 12 x 62
  qualities = 744 (vocab.py:152), ``NO_KEY`` = 9 modes x 12 = 108 (vocab.py:153)
* ``prompt_prefix`` — vocab.py:204-209
"""

from __future__ import annotations

PAD, SOS, EOS, OUT = 0, 1, 2, 3

PROMPTS = (
    ("timestamp", "timestamp"),
    ("downbeat_meter", "rhythm"),
    ("structure", "structure"),
    ("key", "key"),
    ("chord_majmin", "chord"),
    ("chord_full", "chord"),
    ("melody_vocal", "melody"),
    ("melody_full", "melody"),
    ("chord_detail", "chord"),
    ("key_mode", "key"),
)
PROMPT_NAMES = tuple(name for name, _ in PROMPTS)
_GROUP = dict(PROMPTS)
FULL_PROMPTS = ("timestamp", "downbeat_meter", "structure", "key", "chord_full", "melody_full")
FIELDS = ("timestamp", "rhythm", "structure", "key", "chord", "melody")
PROMPT_CAPACITY = 256
MAX_SHIFT = 256
N_METERS = 192
N_STRUCTURE = 23
N_MAJMIN = 25
N_FULL_CHORDS = 361
N_DURATIONS = 24
NO_CHORD = 744
NO_KEY = 108
SWING_CAPACITY = 32


def meter_tables() -> tuple[list[int], list[int]]:
    """Per meter token: bar-length class ``min(numerator, 16) - 1`` and beat unit.

    The meters are every numerator 1..32 with every denominator of (1, 2, 4,
    8, 16, 32), numerator-major (vocab.py:64); frame-head rescoring reads both
    (engine.py:103-105).
    """

    beats, units = [], []
    for numerator in range(1, 33):
        for denominator in (1, 2, 4, 8, 16, 32):
            beats.append(min(numerator, 16) - 1)
            units.append(denominator)
    return beats, units


class VocabTable:
    """Block layout of the token vocabulary (``vocab.Vocab``, vocab.py:157-187).

    Duck-type compatible with the reference ``Vocab`` for everything the decode
    engine reads: ``start``, ``end``, ``size``, ``time_hz`` and
    ``prompt_prefix``.
    """

    def __init__(self, window_seconds: float = 300.0, time_hz: int = 100):
        self.time_hz = time_hz
        blocks = (
            ("special", 4),
            ("prompt", PROMPT_CAPACITY),
            ("shift", MAX_SHIFT + 1),
            ("time", round(window_seconds * time_hz)),
            ("meter", N_METERS),
            ("eighth_position", 256),
            ("structure", N_STRUCTURE),
            ("key", 24),
            ("chord_majmin", N_MAJMIN),
            ("chord_full", N_FULL_CHORDS),
            ("pitch", 256),
            ("duration", N_DURATIONS),
            ("chord_bass", 12),
            ("chord_detail", NO_CHORD + 1),
            ("key_mode", NO_KEY + 1),
            ("swing", SWING_CAPACITY),
        )
        self.start: dict[str, int] = {}
        self.end: dict[str, int] = {}
        offset = 0
        for name, size in blocks:
            self.start[name], self.end[name] = offset, offset + size
            offset += size
        self.size = offset
        self.names = tuple(name for name, _ in blocks)

    def prompt_prefix(self, prompts) -> list[int]:
        """``<sos> <prompt>... <out>`` for a prompt set (vocab.py:204-209).

        Raises ``ValueError`` for an empty set or two prompts of one group,
        exactly as the reference does.
        """

        names = sorted(set(prompts), key=lambda name: (FIELDS.index(_GROUP[name]), PROMPT_NAMES.index(name)))
        groups = [group for name, group in PROMPTS if name in names]
        if not names or len(groups) != len(set(groups)):
            raise ValueError(f"invalid prompt set {prompts!r}")
        return [SOS, *(self.start["prompt"] + PROMPT_NAMES.index(name) for name in names), OUT]
