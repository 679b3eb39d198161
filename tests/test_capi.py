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


def test_peer_and_scheduler_argument_errors_without_gpu():
    """The transport helpers and the new GEMM knobs validate their arguments before any CUDA call."""
    from quack_b200 import _lib

    L = _lib.lib
    off = ctypes.c_ulonglong(0)
    assert L.qk_ipc_export(None, None, ctypes.byref(off)) == -1 and b"null" in L.qk_last_error()
    assert L.qk_ipc_open(None, None) == -1
    assert L.qk_ipc_close(None) == 0                      # closing nothing is a no-op
    assert L.qk_copy_async(None, None, 0, None) == 0      # empty copy
    assert L.qk_copy_async(None, None, 16, None) == -1 and b"null pointer" in L.qk_last_error()
    assert L.qk_stream_wait_geq32(None, None, 1) == -1
    assert L.qk_stream_wait_geq32(None, ctypes.c_void_p(6), 1) == -1 and b"aligned" in L.qk_last_error()
    assert L.qk_stream_write32(None, ctypes.c_void_p(2), 1) == -1
    # scheduler / split-K fields of the GEMM block
    args = _lib.GemmArgs()
    args.format, args.m, args.n, args.k = _lib.FMT_MXFP8_E4M3, 128, 128, 128
    for f in ("a", "b", "sfa", "sfb", "d", "status"):
        setattr(args, f, 4096)
    args.lda = args.ldb = 128
    args.sfa_stride_rm = args.sfa_stride_rk = args.sfb_stride_rm = args.sfb_stride_rk = 512
    args.ldd = 128
    args.scheduler = 5
    assert L.qk_gemm_blockscaled(ctypes.byref(args)) == -1 and b"scheduler" in L.qk_last_error()
    args.scheduler, args.max_ctas = _lib.SCHED_CLC, 64
    assert L.qk_gemm_blockscaled(ctypes.byref(args)) == -1 and b"max_ctas" in L.qk_last_error()
    args.max_ctas, args.prof = 0, 4096
    assert L.qk_gemm_blockscaled(ctypes.byref(args)) == -2 and b"prof" in L.qk_last_error()
    assert _lib.IPC_HANDLE_BYTES == 64
    # batched stream operations: validated one by one, first failure reported
    assert L.qk_stream_ops(None, 0) == 0
    assert L.qk_stream_ops(None, 3) == -1
    ops = (_lib.StreamOp * 3)(_lib.StreamOp(_lib.OP_COPY, 0, None, None, None, 0),      # empty copy: fine
                              _lib.StreamOp(7, 0, None, None, None, 0),                 # unknown kind
                              _lib.StreamOp(_lib.OP_WRITE32, 1, None, None, None, 0))
    assert L.qk_stream_ops(ops, 3) == -1 and b"op 1 has unknown kind 7" in L.qk_last_error()
    ops[1].kind = _lib.OP_WAIT_GEQ32
    assert L.qk_stream_ops(ops, 3) == -1 and b"null address" in L.qk_last_error()


def test_struct_layout_matches_header():
    """Field order of the ctypes mirror follows the C struct."""
    from quack_b200 import _lib

    text = open(os.path.join(ROOT, "include", "quack_b200.h")).read()
    body = text[text.index("typedef struct qk_gemm_args {"):text.index("} qk_gemm_args;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    c_fields = re.findall(r"\b([a-z_0-9]+)\s*;", body)
    py_fields = [f[0] for f in _lib.GemmArgs._fields_]
    assert c_fields == py_fields
