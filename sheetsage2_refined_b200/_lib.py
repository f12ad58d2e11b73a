"""ctypes binding of ``libs2r.so`` (the C ABI in ``include/s2r.h``).

The library is loaded from this package directory.  There is no fallback:
if it cannot be loaded (not built, no CUDA driver) every engine call fails
with ``RuntimeError``.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libs2r.so"

S2R_OK, S2R_EINVAL, S2R_ECUDA, S2R_ENOMEM, S2R_ESTATE, S2R_ENOTSUP, S2R_EDEVICE = range(7)
S2R_F32, S2R_BF16 = 0, 1
S2R_NO_TARGET = (1 << 63) - 1
S2R_FLAG_NO_PDL, S2R_FLAG_NO_GRAPH = 1, 2
S2R_FLAG_NO_TENSOR_CORE = 32
DTYPE_CODES = {0: "<f4", 1: "<V2", 2: "<i8", 3: "|u1", 4: "<f8", 5: "<i4"}

_fp = C.POINTER(C.c_float)


class Config(C.Structure):
    _fields_ = [(name, C.c_int32) for name in (
        "vocab_size", "width", "layers", "heads", "ffn_width", "max_tokens", "batch", "frames", "kv_pages", "flags")]


LAYER_FIELDS = (
    "self_q_w", "self_q_b", "self_k_w", "self_k_b", "self_v_w", "self_v_b", "self_out_w", "self_out_b",
    "self_norm_w", "self_norm_b",
    "cross_q_w", "cross_q_b", "cross_k_w", "cross_k_b", "cross_v_w", "cross_v_b", "cross_out_w", "cross_out_b",
    "cross_norm_w", "cross_norm_b",
    "fc1_w", "fc1_b", "fc2_w", "fc2_b", "final_norm_w", "final_norm_b",
)


class LayerWeights(C.Structure):
    _fields_ = [(name, C.c_void_p) for name in LAYER_FIELDS]


class Weights(C.Structure):
    _fields_ = [
        ("token_embedding", C.c_void_p),
        ("position_embedding", C.c_void_p),
        ("embedding_norm_w", C.c_void_p),
        ("embedding_norm_b", C.c_void_p),
        ("layers", C.POINTER(LayerWeights)),
    ]


class GrammarDesc(C.Structure):
    _fields_ = [
        ("kind", C.c_int32),
        ("token_class", C.c_void_p),
        ("field_of_class", C.c_void_p),
        ("time_seconds", C.c_void_p),
        ("states", C.c_int32),
        ("multiplier", C.c_int32),
        ("table", C.c_void_p),
    ]


FRAME_TERM_COUNT = 8


class Rescore(C.Structure):
    _fields_ = [
        ("weight", C.c_float * FRAME_TERM_COUNT),
        ("bass_span", C.c_int32 * 2),
        ("detail_span", C.c_int32 * 2),
        ("key_span", C.c_int32 * 2),
        ("eighth_span", C.c_int32 * 2),
        ("meter_span", C.c_int32 * 2),
        ("meter_beats", C.c_void_p),
        ("meter_unit", C.c_void_p),
        ("time_hz", C.c_int32),
    ]


# name -> (restype, argtypes); every symbol include/s2r.h declares.
SIGNATURES = {
    "s2r_abi_version": (C.c_int32, []),
    "s2r_last_error": (C.c_char_p, []),
    "s2r_create": (C.c_int32, [C.POINTER(Config), C.POINTER(Weights), C.POINTER(GrammarDesc), C.c_int32,
                               C.POINTER(C.c_void_p)]),
    "s2r_destroy": (C.c_int32, [C.c_void_p]),
    "s2r_set_logit_bias": (C.c_int32, [C.c_void_p, C.c_void_p]),
    "s2r_set_rescore": (C.c_int32, [C.c_void_p, C.POINTER(Rescore)]),
    "s2r_load_frame_tables": (C.c_int32, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "s2r_load_slot": (C.c_int32, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                                  C.POINTER(C.c_int64), C.c_int32, C.c_double, C.c_int64, C.c_void_p]),
    "s2r_step": (C.c_int32, [C.c_void_p, C.c_int32, C.c_void_p]),
    "s2r_step_debug": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "s2r_poll_finished": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p]),
    "s2r_take": (C.c_int32, [C.c_void_p, C.c_int32, C.POINTER(C.c_int64), C.c_int32, C.POINTER(C.c_int32),
                             C.POINTER(C.c_int32), C.c_void_p]),
    "s2r_get_buffer": (C.c_int32, [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_int64),
                                   C.POINTER(C.c_int32)]),
    "s2r_profile_step": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "s2r_step_launches": (C.c_int32, [C.c_void_p]),
    "s2r_free_pages": (C.c_int32, [C.c_void_p]),
    "s2r_poll_finished_async": (C.c_int32, [C.c_void_p, C.c_void_p]),
    "s2r_poll_finished_ready": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_int32, C.POINTER(C.c_int32)]),
    "s2r_take_async": (C.c_int32, [C.c_void_p, C.c_int32, C.c_void_p]),
    "s2r_take_ready": (C.c_int32, [C.c_void_p, C.c_int32, C.POINTER(C.c_int64), C.c_int32, C.POINTER(C.c_int32),
                                   C.POINTER(C.c_int32), C.c_int32, C.POINTER(C.c_int32)]),
    "s2r_masked_argmax_noalloc": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p,
                                              C.c_void_p]),
}

_lib = None


def load(build_if_missing: bool = True):
    """The loaded library (built first if it is missing or stale and nvcc exists)."""

    global _lib
    if _lib is not None:
        return _lib
    if build_if_missing:
        from . import build as _build

        try:
            if _build.stale():
                _build.build()
        except RuntimeError:
            if not LIB_PATH.exists():
                raise
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m sheetsage2_refined_b200.build`")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class EngineError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{message} (s2r status {code})")
        self.code = code


def check(code: int) -> None:
    if code != S2R_OK:
        msg = _lib.s2r_last_error().decode(errors="replace") if _lib is not None else "library not loaded"
        if code == S2R_EINVAL:
            raise ValueError(msg)
        raise EngineError(code, msg)
