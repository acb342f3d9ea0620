"""The C-ABI library: it loads, exports every entry point include/tinker_b200.h
declares, and rejects bad arguments on the host before touching the device.
Runs on the CPU (argument checks return before any CUDA call)."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tinker_b200.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tk_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from tinker_b200 import _lib
    from tinker_b200 import build
    build.build()
    return _lib.lib()


def test_header_declares_the_entry_points():
    names = _declared()
    for n in ("tk_rmsnorm", "tk_add_rmsnorm", "tk_swiglu", "tk_rope_attention", "tk_linear",
              "tk_gate_up_swiglu", "tk_swiglu_ffn", "tk_last_error", "tk_version", "tk_check_device",
              "tk_device_error"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in tinker_b200.h but not exported"


def test_python_signatures_cover_the_header():
    from tinker_b200 import _lib
    assert set(_declared()) - {"tk_last_error"} == set(_lib.SIGNATURES)


def test_version(lib):
    assert lib.tk_version() == 100


def _err(lib):
    return lib.tk_last_error().decode()


def test_host_side_argument_checks(lib):
    from tinker_b200 import _lib
    assert lib.tk_rmsnorm(1, 8, 1, 0, 1, 8, 4, 8, 1e-6, 7, None) == _lib.TK_ERR_INVALID
    assert "dtype" in _err(lib)
    assert lib.tk_rmsnorm(1, 4, 1, 0, 1, 8, 4, 8, 1e-6, 0, None) == _lib.TK_ERR_INVALID
    assert "stride" in _err(lib)
    assert lib.tk_swiglu(None, 8, 1, 8, 1, 8, 4, 8, 0, None) == _lib.TK_ERR_INVALID
    assert lib.tk_linear(16, 12, 16, 32, None, 0, None, 0, 16, 32, None, 4, 12, 0, None) == _lib.TK_ERR_INVALID
    assert "multiples of 8" in _err(lib)
    assert lib.tk_linear(16, 64, 16, 32, None, 0, None, 0, 16, 32, None, 4, 64, 2, None) == _lib.TK_ERR_INVALID
    # head_dim outside {64, 128} is a documented unsupported size
    rc = lib.tk_rope_attention(16, 96, 16, 64, 16, 64, 16, 16, 2, 64, 16, 96, 1, 8, 3, 2, 32, 0, 0, None)
    assert rc == _lib.TK_ERR_UNSUPPORTED and "head_dim" in _err(lib)
    rc = lib.tk_rope_attention(16, 256, 16, 128, 16, 128, 16, 16, 2, 8, 16, 256, 1, 8, 4, 2, 64, 1, 0, None)
    assert rc == _lib.TK_ERR_INVALID and "table" in _err(lib)
    rc = lib.tk_rope_attention(16, 192, 16, 128, 16, 128, 16, 16, 2, 64, 16, 192, 1, 8, 3, 2, 64, 0, 0, None)
    assert rc == _lib.TK_ERR_INVALID and "multiple of num_kv_heads" in _err(lib)
    assert lib.tk_gate_up_swiglu(16, 64, 16, 16, 16, 4, 64, 12, 0, None) == _lib.TK_ERR_INVALID
