"""The C-ABI library loads and exports every symbol include/browservec.h declares.

CPU only: no compute call is made (there may be no GPU).
"""
import ctypes
import os
import re

import pytest

from browservec_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "browservec.h")).read()
    return sorted(set(re.findall(r"BV_API\s+(?:const\s+char\s*\*|int)\s+(bv_\w+)\s*\(", text)))


def test_header_declarations_match_binding():
    decl = declared_symbols()
    assert decl, "no declarations found"
    assert sorted(_lib.EXPORTS) == decl


def test_library_exports_every_declared_symbol():
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("libbvcuda.so not built")
    L = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(L, name), name


def test_last_error_is_callable_without_gpu():
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("libbvcuda.so not built")
    L = _lib.load()
    assert isinstance(L.bv_last_error(), bytes)


def test_create_rejects_bad_config_before_touching_the_gpu():
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("libbvcuda.so not built")
    L = _lib.load()
    h = ctypes.c_void_p()
    cfg = _lib.BvConfig(dim=0, bits=8)
    assert L.bv_create(ctypes.byref(cfg), ctypes.byref(h)) == _lib.BV_ERR_INVALID
    assert b"dimension must be a positive integer" in L.bv_last_error()
    cfg = _lib.BvConfig(dim=16, bits=2)
    assert L.bv_create(ctypes.byref(cfg), ctypes.byref(h)) == _lib.BV_ERR_INVALID
    assert b"quantBits 2 not supported" in L.bv_last_error()
    cfg = _lib.BvConfig(dim=16, bits=8, metric=2)
    assert L.bv_create(ctypes.byref(cfg), ctypes.byref(h)) == _lib.BV_ERR_INVALID
    assert b"cosine/dot only" in L.bv_last_error()
    cfg = _lib.BvConfig(dim=16, bits=8, scoring=2)
    assert L.bv_create(ctypes.byref(cfg), ctypes.byref(h)) == _lib.BV_ERR_INVALID
