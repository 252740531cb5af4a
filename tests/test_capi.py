"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and rejects bad arguments with a status and a message before
touching the device."""
import ctypes
import os
import re

import pytest

from bfloat16x_b200 import _lib
from oracle import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bf16x_b200.h")


def header_symbols():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(bf16x_\w+)\s*\(", txt)))


@pytest.fixture(scope="module")
def L():
    return _lib.lib()


def test_header_symbols_exported(L):
    syms = header_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(L, s), f"{s} declared in include/bf16x_b200.h but not exported"
    # the Python binding covers the whole header
    assert set(syms) <= set(_lib.exported_symbols()), set(syms) - set(_lib.exported_symbols())


def test_version(L):
    assert L.bf16x_version() >= 1


@pytest.mark.parametrize("n", [0, 1, 5, 15, 31, 32, 33, 100, 1000, 3145728])
@pytest.mark.parametrize("b", [1, 3, 7])
def test_stream_words_matches_reference_rule(L, n, b):
    assert L.bf16x_stream_words(n, b) == oracle.stream_words(n, b)


def test_resident_row_bytes(L):
    assert L.bf16x_resident_row_bytes(256) == 384
    assert L.bf16x_resident_row_bytes(4096) == 16 * 384
    assert L.bf16x_resident_row_bytes(257) == 2 * 384
    assert L.bf16x_resident_row_bytes(14336) == 56 * 384


def _err(L):
    return L.bf16x_last_error().decode()


def test_invalid_arguments_rejected_on_host(L):
    # batch out of range
    rc = L.bf16x_gemv(None, None, None, 16, 256, None, 17, 256, None, None, 0, 16, None, None, 0, None)
    assert rc == -1
    assert "batch" in _err(L)
    # in_f too large for the resident layout
    assert L.bf16x_gemv(None, None, None, 16, 70000, None, 1, 70144, None, None, 0, 16, None, None, 0, None) < 0
    assert "65536" in _err(L)
    # unsupported sub-block size
    assert L.bf16x_decode(None, 1, None, 7, None, 3, None, 2, None, None, 0, 1, 32, 8, None, None) < 0
    assert "sub" in _err(L)
    # streams too short for the shape
    assert L.bf16x_decode(ctypes.c_void_p(16), 1, ctypes.c_void_p(16), 1, ctypes.c_void_p(16), 1,
                          ctypes.c_void_p(16), 1, None, None, 0, 4, 64, 16, ctypes.c_void_p(16), None) < 0
    assert "shorter" in _err(L)
    # an empty weight is a no-op
    assert L.bf16x_decode(None, 0, None, 0, None, 0, None, 0, None, None, 0, 0, 16, 16, None, None) == 0


def test_gemv_missing_counters_and_scratch(L):
    # counters and scratch are checked on the host before any launch
    assert L.bf16x_gemv_scratch_bytes(0, 256) == 0
    v = ctypes.c_void_p(256)
    assert L.bf16x_gemv(v, v, v, 16, 256, v, 1, 256, None, v, 0, 16, None, v, 1 << 30, None) < 0
    assert "tile_counters" in _err(L)


def test_error_raises_python_exception():
    with pytest.raises(_lib.Bf16xError, match="batch"):
        _lib.call("bf16x_gemv", None, None, None, 16, 256, None, 0, 256, None, None, 0, 16, None, None, 0, None)
