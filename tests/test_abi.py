"""The C ABI library: it loads, exports every symbol ``include/s2r.h`` declares,
and its host-side checks fail with a status code (no GPU needed)."""

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

from sheetsage2_refined_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "s2r.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:int32_t|const char\*)\s+(s2r_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_binding():
    assert declared_symbols() == set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (s2r_\w+)", out))
    missing = declared_symbols() - exported
    assert not missing, missing
    for name in declared_symbols():
        assert getattr(lib, name) is not None


def test_version_and_error_without_gpu():
    lib = _lib.load()
    assert lib.s2r_abi_version() == 1
    assert isinstance(lib.s2r_last_error(), bytes)


def test_create_rejects_bad_shapes_before_touching_the_device():
    lib = _lib.load()
    cfg = _lib.Config(vocab_size=512, width=200, layers=1, heads=4, ffn_width=1024, max_tokens=64, batch=1, frames=8)
    w = _lib.Weights()
    g = _lib.GrammarDesc(kind=1)
    ctx = C.c_void_p()
    rc = lib.s2r_create(C.byref(cfg), C.byref(w), C.byref(g), 0, C.byref(ctx))
    assert rc == _lib.S2R_ENOTSUP
    assert b"heads * 64" in lib.s2r_last_error()
    assert ctx.value is None


def test_null_engine_calls_return_status():
    lib = _lib.load()
    assert lib.s2r_step(None, 1, None) == _lib.S2R_EINVAL
    assert lib.s2r_destroy(None) == _lib.S2R_OK
    assert lib.s2r_step_launches(None) == 0


@pytest.mark.skipif(_lib.C.CDLL is None, reason="ctypes")
def test_check_maps_status_to_exceptions():
    _lib.load()
    with pytest.raises(ValueError):
        _lib.check(_lib.S2R_EINVAL)
    with pytest.raises(_lib.EngineError):
        _lib.check(_lib.S2R_ECUDA)
