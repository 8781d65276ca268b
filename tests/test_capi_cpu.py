"""C ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and rejects bad arguments on the host before any CUDA call."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from snapjudge_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "snapjudge_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sj_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_header_symbol():
    L = _lib.lib()
    syms = header_symbols()
    assert len(syms) >= 17
    for s in syms:
        assert hasattr(L, s), s
    assert sorted(_lib.EXPORTS) == syms


def test_version():
    assert _lib.lib().sj_b200_version() >= 100


def test_host_side_validation_returns_status():
    L = _lib.lib()
    # negative sizes / null operands are rejected before touching the device
    assert L.sj_gemm(None, None, None, None, -1, 4, 4, 0, 0, None) == _lib.SJ_ERR_INVALID
    assert b"negative" in L.sj_last_error()
    assert L.sj_gemm(None, None, None, None, 4, 4, 4, 0, 7, None) == _lib.SJ_ERR_INVALID
    assert L.sj_gemm_geglu(None, None, None, 4, 4, 4, None) == _lib.SJ_ERR_INVALID
    assert L.sj_add_ln(None, None, None, None, None, 4, 16, 1e-5, 0, 0, None) == _lib.SJ_ERR_INVALID
    bad_cu = np.array([0, 5, 3], np.int32)  # decreasing
    assert L.sj_attn(None, None, C.c_void_p(bad_cu.ctypes.data), None, None, 2, 2, 8, 0,
                     None) == _lib.SJ_ERR_INVALID
    assert b"non-decreasing" in L.sj_last_error()
    nz = np.array([1, 5], np.int32)  # cu[0] != 0
    assert L.sj_rope(None, None, None, None, C.c_void_p(nz.ctypes.data), 1, 2, 8,
                     None) == _lib.SJ_ERR_INVALID


def test_engine_rejects_bad_config():
    L = _lib.lib()
    h = C.c_void_p()
    c = _lib.FastConfig(100, 2, 3, 64, 10, 64, 1e-5, 0, None, 1e4, 1e4, 0, 0, 0)  # 100 % 3 != 0
    assert L.sj_fast_create(C.byref(c), C.byref(h)) == _lib.SJ_ERR_INVALID
    c = _lib.FastConfig(64, 2, 4, 64, 10, 64, 1e-5, 0, None, 1e4, 1e4, 9, 0, 0)  # precision 9
    assert L.sj_fast_create(C.byref(c), C.byref(h)) == _lib.SJ_ERR_UNSUPPORTED


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_LIB", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(ImportError):
        _lib.lib()
