"""ctypes binding of libquack_b200.so (the C ABI declared in include/quack_b200.h).

There is no fallback: if the shared library has not been built, importing this module
raises, and every operator of the package fails with it.
"""

from __future__ import annotations

import ctypes as C
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("QUACK_B200_LIB") or os.path.join(_HERE, "libquack_b200.so")   # override: variant builds

# enums of csrc/qk_types.h
FMT_NONE, FMT_MXFP8_E4M3, FMT_NVFP4, FMT_MXFP8_E5M2, FMT_MXFP4 = 0, 1, 2, 3, 4
SCALING_DEFAULT, SCALING_FLOOR, SCALING_RCEIL = 0, 1, 2
DT_BF16, DT_F16, DT_F32 = 0, 1, 2
NOALLOC_MAX_CTAS = 256
SCHED_STATIC, SCHED_CLC, SCHED_ARRIVAL = 0, 1, 2
ACT = {None: 0, "relu": 1, "relu_sq": 2, "silu": 3, "gelu_tanh_approx": 4, "tanh": 5,
       "swiglu": 16, "reglu": 17, "geglu": 18, "glu": 19}
STATUS_NAMES = {1: "producer wait", 2: "MMA wait for operands", 3: "MMA wait for accumulator",
                4: "epilogue wait", 5: "all-gather arrival gate", 6: "tile scheduler",
                7: "all-gather in-kernel transport (peer shard not staged, or a copy that did not land)"}

TORCH_TO_DT = {torch.bfloat16: DT_BF16, torch.float16: DT_F16, torch.float32: DT_F32}


AG_MAX_RANKS, AG_MAX_PAYLOADS = 16, 2


class AgPullArgs(C.Structure):
    """qk_ag_pull_args: the in-kernel all-gather transport's table of peer addresses (copied to device memory)."""
    _fields_ = [("num_payloads", C.c_int), ("rank", C.c_int),
                ("shard_bytes", C.c_ulonglong * AG_MAX_PAYLOADS),
                ("local_base", C.c_void_p * AG_MAX_PAYLOADS),
                ("peer_base", (C.c_void_p * AG_MAX_PAYLOADS) * AG_MAX_RANKS),
                ("peer_flags", C.c_void_p * AG_MAX_RANKS),
                ("peer_drained", C.c_void_p * AG_MAX_RANKS),
                ("arrive", C.c_void_p), ("flags_rw", C.c_void_p), ("publish_ns", C.c_void_p),
                ("mode", C.c_int), ("chunks", C.c_int), ("mc_base", C.c_void_p * AG_MAX_PAYLOADS),
                ("mc_flags", C.c_void_p), ("mc_drained", C.c_void_p), ("done", C.c_void_p)]


class AgArgs(C.Structure):
    _fields_ = [("flags", C.c_void_p), ("epoch", C.c_void_p), ("num_shards", C.c_int),
                ("first_shard", C.c_int), ("num_chunks", C.c_int), ("pull", C.c_void_p)]


class StreamOp(C.Structure):
    _fields_ = [("kind", C.c_int), ("value", C.c_uint), ("stream", C.c_void_p), ("dst", C.c_void_p),
                ("src", C.c_void_p), ("bytes", C.c_ulonglong)]


OP_COPY, OP_WAIT_GEQ32, OP_WRITE32 = 0, 1, 2


class GemmArgs(C.Structure):
    _fields_ = [
        ("format", C.c_int), ("format_b", C.c_int), ("m", C.c_int), ("n", C.c_int), ("k", C.c_int),
        ("a", C.c_void_p), ("lda", C.c_longlong), ("b", C.c_void_p), ("ldb", C.c_longlong),
        ("sfa", C.c_void_p), ("sfa_stride_rm", C.c_longlong), ("sfa_stride_rk", C.c_longlong),
        ("sfb", C.c_void_p), ("sfb_stride_rm", C.c_longlong), ("sfb_stride_rk", C.c_longlong),
        ("d", C.c_void_p), ("ldd", C.c_longlong), ("d_dtype", C.c_int),
        ("post", C.c_void_p), ("ldpost", C.c_longlong), ("post_dtype", C.c_int), ("activation", C.c_int),
        ("exact_activation", C.c_int),
        ("bias", C.c_void_p), ("bias_dtype", C.c_int),
        ("alpha", C.c_float), ("alpha_dev", C.c_void_p), ("alpha_dev2", C.c_void_p),
        ("c", C.c_void_p), ("ldc", C.c_longlong), ("c_dtype", C.c_int), ("beta", C.c_float), ("beta_dev", C.c_void_p),
        ("out_format", C.c_int), ("sfd", C.c_void_p), ("sfd_stride_rm", C.c_longlong),
        ("norm_const", C.c_float), ("norm_const_dev", C.c_void_p),
        ("ag", AgArgs),
        ("tile_n", C.c_int), ("cta_group", C.c_int), ("max_ctas", C.c_int), ("scheduler", C.c_int),
        ("split_k", C.c_int), ("workspace", C.c_void_p), ("workspace_bytes", C.c_ulonglong),
        ("status", C.c_void_p), ("timeout_ns", C.c_ulonglong), ("prof", C.c_void_p), ("stream", C.c_void_p),
    ]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python quack_b200/csrc/build.py` "
            "(needs nvcc with sm_100a support). quack_b200 has no CPU or PyTorch fallback.")
    lib = C.CDLL(LIB_PATH)
    lib.qk_version.restype = C.c_int
    lib.qk_last_error.restype = C.c_char_p
    lib.qk_launch_count.restype = C.c_longlong
    lib.qk_scale_blocked_bytes.restype = C.c_size_t
    lib.qk_scale_blocked_bytes.argtypes = [C.c_int, C.c_longlong, C.c_longlong]
    lib.qk_amax.restype = C.c_int
    lib.qk_amax.argtypes = [C.c_void_p, C.c_int, C.c_longlong, C.c_longlong, C.c_longlong, C.c_void_p, C.c_void_p]
    lib.qk_quantize_blockscaled.restype = C.c_int
    lib.qk_quantize_blockscaled.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_longlong, C.c_longlong, C.c_longlong,
                                            C.c_void_p, C.c_longlong, C.c_void_p, C.c_void_p, C.c_void_p]
    lib.qk_quantize_blockscaled_mode.restype = C.c_int
    lib.qk_quantize_blockscaled_mode.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_longlong, C.c_longlong,
                                                 C.c_longlong, C.c_void_p, C.c_longlong, C.c_void_p, C.c_void_p, C.c_void_p]
    lib.qk_quantize_blockscaled_dim0.restype = C.c_int
    lib.qk_quantize_blockscaled_dim0.argtypes = lib.qk_quantize_blockscaled_mode.argtypes
    for name in ("qk_scale_pack_blocked", "qk_scale_unpack_blocked"):
        fn = getattr(lib, name)
        fn.restype = C.c_int
        fn.argtypes = [C.c_void_p, C.c_longlong, C.c_longlong, C.c_void_p, C.c_void_p]
    lib.qk_gemm_blockscaled.restype = C.c_int
    lib.qk_gemm_blockscaled.argtypes = [C.POINTER(GemmArgs)]
    lib.qk_gemm_blockscaled_noalloc.restype = C.c_int
    lib.qk_gemm_blockscaled_noalloc.argtypes = [C.POINTER(GemmArgs), C.c_void_p, C.c_void_p]
    lib.qk_ipc_export.restype = C.c_int
    lib.qk_ipc_export.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(C.c_ulonglong)]
    lib.qk_ipc_open.restype = C.c_int
    lib.qk_ipc_open.argtypes = [C.c_void_p, C.POINTER(C.c_void_p)]
    lib.qk_ipc_close.restype = C.c_int
    lib.qk_ipc_close.argtypes = [C.c_void_p]
    lib.qk_copy_async.restype = C.c_int
    lib.qk_copy_async.argtypes = [C.c_void_p, C.c_void_p, C.c_ulonglong, C.c_void_p]
    lib.qk_stream_wait_geq32.restype = C.c_int
    lib.qk_stream_wait_geq32.argtypes = [C.c_void_p, C.c_void_p, C.c_uint]
    lib.qk_stream_write32.restype = C.c_int
    lib.qk_stream_write32.argtypes = [C.c_void_p, C.c_void_p, C.c_uint]
    lib.qk_tensor_map_cache_stats.restype = None
    lib.qk_tensor_map_cache_stats.argtypes = [C.POINTER(C.c_longlong), C.POINTER(C.c_longlong)]
    lib.qk_stream_ops.restype = C.c_int
    lib.qk_stream_ops.argtypes = [C.c_void_p, C.c_int]
    return lib


lib = _load()

EXPORTS = ("qk_version", "qk_last_error", "qk_launch_count", "qk_scale_blocked_bytes", "qk_amax",
           "qk_quantize_blockscaled", "qk_quantize_blockscaled_mode", "qk_quantize_blockscaled_dim0", "qk_scale_pack_blocked", "qk_scale_unpack_blocked",
           "qk_gemm_blockscaled", "qk_gemm_blockscaled_noalloc", "qk_ipc_export", "qk_ipc_open", "qk_ipc_close",
           "qk_copy_async", "qk_stream_wait_geq32", "qk_stream_write32", "qk_stream_ops", "qk_tensor_map_cache_stats")
IPC_HANDLE_BYTES = 64


def ipc_export(ptr: int):
    """(handle bytes, offset) of the cudaMalloc allocation that contains device address `ptr`."""
    buf = C.create_string_buffer(IPC_HANDLE_BYTES)
    off = C.c_ulonglong(0)
    check(lib.qk_ipc_export(ptr, buf, C.byref(off)), "qk_ipc_export")
    return bytes(buf.raw), int(off.value)


def ipc_open(handle: bytes) -> int:
    base = C.c_void_p(0)
    check(lib.qk_ipc_open(handle, C.byref(base)), "qk_ipc_open")
    return int(base.value)


class QuackB200Error(RuntimeError):
    pass


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib.qk_last_error().decode("utf-8", "replace")
        exc = ValueError if rc == -1 else (NotImplementedError if rc == -2 else QuackB200Error)
        raise exc(f"{what or 'quack_b200'} failed ({rc}): {msg}")


def current_stream(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def tensor_map_cache_stats():
    """(hits, misses) of the library's tensor-map cache."""
    h, m = C.c_longlong(0), C.c_longlong(0)
    lib.qk_tensor_map_cache_stats(C.byref(h), C.byref(m))
    return int(h.value), int(m.value)


def launch_count() -> int:
    return int(lib.qk_launch_count())
