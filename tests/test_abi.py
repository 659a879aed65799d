"""The C-ABI library: it loads without a GPU and exports every symbol include/whisper4j_cuda.h declares."""
import ctypes
import os
import re

import pytest

from whisper4j_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "whisper4j_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(w4j_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "w4j_decode" in syms and "w4j_decode_beam" in syms and "w4j_forward" in syms
    assert len(syms) >= 20


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for s in declared_symbols():
        assert hasattr(L, s), f"missing export {s}"
        assert s in _lib.SIGNATURES, f"no ctypes signature for {s}"


def test_version_and_error_text():
    L = _lib.lib()
    assert b"sm_100a" in L.w4j_version()
    assert isinstance(L.w4j_last_error(), bytes)


def test_null_arguments_are_rejected():
    L = _lib.lib()
    assert L.w4j_ctx_create(None, 0, 1, 1, None) == _lib.W4J_ERR_ARG
    assert b"null" in L.w4j_last_error()
    assert L.w4j_decode(None, None, 0, None, 0, 0, 0, None, 0, 0, 0.0, 0, 0, None) == _lib.W4J_ERR_ARG


def test_bad_dims_rejected_before_device_use():
    L = _lib.lib()
    d = _lib.Dims(80, 1500, 384, 6, 4, 51864, 448, 384, 5, 4)  # 384 != 5 * 64
    h = ctypes.c_void_p()
    assert L.w4j_ctx_create(ctypes.byref(d), 0, 1, 1, ctypes.byref(h)) == _lib.W4J_ERR_ARG
    assert b"n_text_head" in L.w4j_last_error()
