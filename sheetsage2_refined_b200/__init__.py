"""B200-native decode engine for SheetSage2-Refined's grammar-constrained greedy token loop.

``BatchDecoder`` is a drop-in for ``sheetsage2_refined.engine.BatchDecoder``;
the step runs in hand-written sm_100a CUDA kernels behind the C ABI of
``include/s2r.h`` (``libs2r.so``).
"""

from .grammar import ENDED, ClassGrammar, TableGrammar
from .vocab_table import FULL_PROMPTS, VocabTable
from .weights import DecoderConfig, DecoderWeights, memory_array, synthetic_state_dict


def __getattr__(name):
    # The engine module needs torch and the CUDA library; import it on first use.
    if name in ("BatchDecoder", "frame_terms", "FRAME_TERMS"):
        from . import engine

        return getattr(engine, name)
    raise AttributeError(name)


__all__ = [
    "BatchDecoder",
    "ClassGrammar",
    "DecoderConfig",
    "DecoderWeights",
    "ENDED",
    "FULL_PROMPTS",
    "TableGrammar",
    "VocabTable",
    "memory_array",
    "synthetic_state_dict",
]
