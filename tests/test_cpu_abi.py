"""The C-ABI library loads and exports every symbol include/potpori_b200.h declares (no GPU
calls)."""
import ctypes
import os
import re

import pytest

from potpori_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(pp_[a-z_0-9]+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 20
    for name in syms:
        assert hasattr(L, name), name
    assert set(syms) == set(_lib.EXPORTS)


def test_version_and_create_validation():
    L = _lib.load()
    assert b"sm_100a" in L.pp_version()
    # Invalid ranges are rejected before any device work (src/qwen/model.rs:206-217).
    cfg = _lib.Config(2, 8, 12, 4, 2, 1, 16, 1e-6, 1e4)
    for lb, le, cap, chunk in [(1, 1, 8, 2), (0, 3, 8, 2), (0, 2, 0, 0), (0, 2, 4, 8)]:
        d = _lib.ShardDesc(cfg, lb, le, cap, chunk, 0)
        h = ctypes.c_void_p()
        st = L.pp_shard_create(ctypes.byref(d), ctypes.byref(h))
        assert st == _lib.PP_E_INVALID and not h.value
        assert _lib.last_error(None)
