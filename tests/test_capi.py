"""The C-ABI library loads on a machine without a GPU and exports every symbol that
include/quack_b200.h declares; argument errors are reported without touching CUDA."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    text = open(os.path.join(ROOT, "include", "quack_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qk_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_are_exported():
    from quack_b200 import _lib

    names = _declared_symbols()
    assert "qk_gemm_blockscaled" in names and "qk_quantize_blockscaled" in names
    for n in names:
        assert hasattr(_lib.lib, n), f"{n} is declared in include/quack_b200.h but not exported"
    assert set(_lib.EXPORTS) <= set(names)


def test_version_and_sizes():
    from quack_b200 import _lib

    assert _lib.lib.qk_version() >= 100
    assert _lib.lib.qk_scale_blocked_bytes(_lib.FMT_MXFP8_E4M3, 2048, 4096) == 16 * 32 * 512
    assert _lib.lib.qk_scale_blocked_bytes(_lib.FMT_NVFP4, 129, 48) == 2 * 1 * 512


def test_argument_errors_without_gpu():
    from quack_b200 import _lib

    rc = _lib.lib.qk_gemm_blockscaled(None)
    assert rc == -1 and b"null argument" in _lib.lib.qk_last_error()
    args = _lib.GemmArgs()
    args.format = 7
    assert _lib.lib.qk_gemm_blockscaled(ctypes.byref(args)) == -2
    rc = _lib.lib.qk_quantize_blockscaled(_lib.FMT_MXFP8_E4M3, None, 0, 4, 48, 48, None, 48, None, None, None)
    assert rc == -1 and b"null pointer" in _lib.lib.qk_last_error()
    rc = _lib.lib.qk_quantize_blockscaled(_lib.FMT_MXFP8_E4M3, ctypes.c_void_p(16), 0, 4, 40, 40,
                                          ctypes.c_void_p(16), 40, ctypes.c_void_p(16), None, None)
    assert rc == -1 and b"divisible" in _lib.lib.qk_last_error()
    with pytest.raises(ValueError):
        _lib.check(rc, "quantize")


def test_struct_layout_matches_header():
    """Field order of the ctypes mirror follows the C struct."""
    from quack_b200 import _lib

    text = open(os.path.join(ROOT, "include", "quack_b200.h")).read()
    body = text[text.index("typedef struct qk_gemm_args {"):text.index("} qk_gemm_args;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    c_fields = re.findall(r"\b([a-z_0-9]+)\s*;", body)
    py_fields = [f[0] for f in _lib.GemmArgs._fields_]
    assert c_fields == py_fields
