"""Raw operator layer: torch tensors in, C-ABI calls out.  No numerics live here; the
functions only allocate outputs, take pointers / strides and check the device status word.
The public, reference-shaped API (quack_b200.blockscaled, quack_b200.gemm_interface,
quack_b200.gemm, quack_b200.distributed) is built on these.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib
from ._lib import FMT_MXFP4, FMT_MXFP8_E4M3, FMT_MXFP8_E5M2, FMT_NVFP4, FMT_NONE

_FMT_ID = {"mxfp8_e4m3": FMT_MXFP8_E4M3, "mxfp8_e5m2": FMT_MXFP8_E5M2, "mxfp4": FMT_MXFP4, "nvfp4": FMT_NVFP4}
_FMT_VEC = {FMT_MXFP8_E4M3: 32, FMT_MXFP8_E5M2: 32, FMT_MXFP4: 32, FMT_NVFP4: 16}
_FMT_FP4 = (FMT_MXFP4, FMT_NVFP4)


def format_id(name: str) -> int:
    try:
        return _FMT_ID[name]
    except KeyError:
        raise NotImplementedError(
            f"blockscaled format {name!r} has no sm_100a kernel in quack_b200 "
            f"(implemented: {sorted(_FMT_ID)})") from None


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor: quack_b200 has no CPU path")


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else C.c_void_p(t.data_ptr())


def amax(x: torch.Tensor) -> torch.Tensor:
    """max|x| of a 2-D bf16/fp32 CUDA tensor -> (1,) fp32 on device (no host sync)."""
    _require_cuda(x, "x")
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    out = torch.zeros(1, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib.qk_amax(_ptr(x2), _lib.TORCH_TO_DT[x2.dtype], x2.shape[0], x2.shape[1], x2.stride(0),
                                    _ptr(out), C.c_void_p(_lib.current_stream(x.device))), "qk_amax")
    return out


def quantize_rows(x: torch.Tensor, fmt: int, per_tensor_scale: Optional[torch.Tensor] = None,
                  scaling_mode: int = _lib.SCALING_DEFAULT):
    """(rows, K) bf16/fp32 -> (codes uint8, blocked scales uint8 (rm, rk, 32, 4, 4))."""
    _require_cuda(x, "x")
    assert x.ndim == 2
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"quantize expects bf16 or fp32 input, got {x.dtype}")
    if x.stride(-1) != 1 or (x.stride(0) * x.element_size()) % 16 or x.data_ptr() % 16:
        x = x.contiguous()
    rows, k = x.shape
    vec = _FMT_VEC[fmt]
    kb = k // 2 if fmt in _FMT_FP4 else k
    codes = torch.empty(rows, kb, dtype=torch.uint8, device=x.device)
    rm, rk = -(-rows // 128), -(-(k // vec) // 4)
    sf = torch.empty(rm, rk, 32, 4, 4, dtype=torch.uint8, device=x.device)
    if rows == 0 or k == 0:
        return codes, sf
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib.qk_quantize_blockscaled_mode(
            fmt, scaling_mode, _ptr(x), _lib.TORCH_TO_DT[x.dtype], rows, k, x.stride(0), _ptr(codes), codes.stride(0),
            _ptr(sf), _ptr(per_tensor_scale), C.c_void_p(_lib.current_stream(x.device))), "qk_quantize_blockscaled")
    return codes, sf


def quantize_cols(x: torch.Tensor, fmt: int, per_tensor_scale: Optional[torch.Tensor] = None,
                  scaling_mode: int = _lib.SCALING_DEFAULT):
    """(R, C) bf16/fp32 quantised along dim 0 -> (codes uint8 of the TRANSPOSED matrix, (C, R) or (C, R/2) for the
    4-bit formats; blocked scales uint8 (ceil(C/128), ceil(R/vec/4), 32, 4, 4)): the row quantizer's result for
    ``x.T`` without the transposed high-precision copy.  R must be a multiple of 32."""
    _require_cuda(x, "x")
    assert x.ndim == 2
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"quantize expects bf16 or fp32 input, got {x.dtype}")
    if x.stride(-1) != 1 or (x.stride(0) * x.element_size()) % 16 or x.data_ptr() % 16:
        x = x.contiguous()
    r, c = x.shape
    vec = _FMT_VEC[fmt]
    codes = torch.empty(c, r // 2 if fmt in _FMT_FP4 else r, dtype=torch.uint8, device=x.device)
    sf = torch.empty(-(-c // 128), -(-(r // vec) // 4), 32, 4, 4, dtype=torch.uint8, device=x.device)
    if r == 0 or c == 0:
        return codes, sf
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib.qk_quantize_blockscaled_dim0(
            fmt, scaling_mode, _ptr(x), _lib.TORCH_TO_DT[x.dtype], r, c, x.stride(0), _ptr(codes), codes.stride(0),
            _ptr(sf), _ptr(per_tensor_scale), C.c_void_p(_lib.current_stream(x.device))), "qk_quantize_blockscaled_dim0")
    return codes, sf


def scale_pack(scale_2d: torch.Tensor) -> torch.Tensor:
    _require_cuda(scale_2d, "scale")
    s = scale_2d.contiguous().view(torch.uint8)
    mn, sfk = s.shape
    out = torch.empty(-(-mn // 128), -(-sfk // 4), 32, 4, 4, dtype=torch.uint8, device=s.device)
    with torch.cuda.device(s.device):
        _lib.check(_lib.lib.qk_scale_pack_blocked(_ptr(s), mn, sfk, _ptr(out), C.c_void_p(_lib.current_stream(s.device))))
    return out


def scale_unpack(blocked: torch.Tensor, mn: int, sf_k: int) -> torch.Tensor:
    _require_cuda(blocked, "scale")
    b = blocked.contiguous().view(torch.uint8)
    out = torch.empty(mn, sf_k, dtype=torch.uint8, device=b.device)
    with torch.cuda.device(b.device):
        _lib.check(_lib.lib.qk_scale_unpack_blocked(_ptr(b), mn, sf_k, _ptr(out), C.c_void_p(_lib.current_stream(b.device))))
    return out


_status_bufs = {}


def status_buffer(device) -> torch.Tensor:
    """Per-device 4-int status block shared by all GEMM launches of this process."""
    buf = _status_bufs.get(device)
    if buf is not None:
        return buf
    dev = torch.device(device)
    key = (dev.type, dev.index if dev.index is not None else torch.cuda.current_device())
    buf = _status_bufs.get(key)
    if buf is None:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("quack_b200: the first GEMM on a device allocates its status block; run one GEMM (or "
                               "_ops.status_buffer(device)) before capturing a CUDA graph")
        buf = torch.zeros(4, dtype=torch.int32, device=dev)
        _status_bufs[key] = buf
    _status_bufs[device] = buf
    return buf


def check_status(device, sync: bool = True) -> None:
    """Raise if a kernel on `device` abandoned a bounded wait.  Reads the status word (a
    4-int device->host copy), so it synchronises with the launches before it.  A kernel that gave up may
    have left split-K arrival counters half counted: the scratch buffers of the device are zeroed again
    before the error is raised, so the next launch starts clean."""
    buf = status_buffer(device)
    st = buf.tolist()
    if st[0] != 0:
        buf.zero_()
        index = buf.device.index
        for (idx, _stream), ws in _workspaces.items():
            if idx == index:
                ws[2].zero_()
        torch.cuda.synchronize(buf.device)
        raise _lib.QuackB200Error(
            f"block-scaled GEMM gave up a bounded wait: {_lib.STATUS_NAMES.get(st[0], st[0])} "
            f"(detail={st[1]}, block/flag={st[2]}, aux={st[3]})")


def build_gemm_args(
    fmt: int, a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, m: int, n: int, k: int, *,
    d: Optional[torch.Tensor] = None, post: Optional[torch.Tensor] = None, activation=None,
    bias: Optional[torch.Tensor] = None, alpha: float = 1.0, alpha_dev: Optional[torch.Tensor] = None,
    alpha_dev2: Optional[torch.Tensor] = None,
    out_format: int = FMT_NONE, sfd: Optional[torch.Tensor] = None, norm_const: float = 1.0,
    norm_const_dev: Optional[torch.Tensor] = None, ag=None, tile_n: int = 0, cta_group: int = 0, max_ctas: int = 0,
    timeout_ns: int = 0, prof: Optional[torch.Tensor] = None, scheduler: int = 0, split_k: int = 0,
    workspace: Optional[torch.Tensor] = None,
    c: Optional[torch.Tensor] = None, beta: float = 1.0, beta_dev: Optional[torch.Tensor] = None,
    exact_activation: bool = False, fmt_b: int = 0,
) -> "_lib.GemmArgs":
    """Fill a `qk_gemm_args` block (everything except the status buffer and the stream).  `a` is
    (m, k_storage) K-major codes, `b` is (n, k_storage) K-major codes (any 1-byte dtype),
    `sfa`/`sfb` blocked scales (rm, rk, 32, 4, 4) whose atom strides may be any multiple of 512 B."""
    _require_cuda(a, "A")
    args = _lib.GemmArgs()
    args.format, args.format_b, args.m, args.n, args.k = fmt, fmt_b, m, n, k
    args.a, args.lda = a.data_ptr(), a.stride(0) * a.element_size()
    args.b, args.ldb = b.data_ptr(), b.stride(0) * b.element_size()
    args.sfa, args.sfa_stride_rm, args.sfa_stride_rk = sfa.data_ptr(), sfa.stride(-5), sfa.stride(-4)
    args.sfb, args.sfb_stride_rm, args.sfb_stride_rk = sfb.data_ptr(), sfb.stride(-5), sfb.stride(-4)
    quant_d = out_format != FMT_NONE and post is None
    if d is not None:
        args.d, args.ldd = d.data_ptr(), d.stride(0)
        args.d_dtype = 0 if quant_d else _lib.TORCH_TO_DT[d.dtype]
    if post is not None:
        args.post, args.ldpost = post.data_ptr(), post.stride(0)
        args.post_dtype = 0 if out_format != FMT_NONE else _lib.TORCH_TO_DT[post.dtype]
    args.activation = _lib.ACT[activation]
    args.exact_activation = 1 if exact_activation else 0
    if bias is not None:
        if bias.stride(-1) != 1:
            bias = bias.contiguous()
        args.bias, args.bias_dtype = bias.data_ptr(), _lib.TORCH_TO_DT[bias.dtype]
    args.alpha = float(alpha)
    if alpha_dev is not None:
        args.alpha_dev = alpha_dev.data_ptr()
        if alpha_dev2 is not None:
            args.alpha_dev2 = alpha_dev2.data_ptr()
    if c is not None:
        assert c.stride(-1) == 1, "the residual operand must be row-major"
        args.c, args.ldc, args.c_dtype, args.beta = c.data_ptr(), c.stride(0), _lib.TORCH_TO_DT[c.dtype], float(beta)
        if beta_dev is not None:
            args.beta_dev = beta_dev.data_ptr()
    args.out_format = out_format
    if sfd is not None:
        args.sfd, args.sfd_stride_rm = sfd.data_ptr(), sfd.stride(-5)
    args.norm_const = float(norm_const)
    if norm_const_dev is not None:
        args.norm_const_dev = norm_const_dev.data_ptr()
    if ag is not None:
        args.ag.flags = ag.flags.data_ptr()
        args.ag.epoch = ag.epoch.data_ptr()
        args.ag.num_shards, args.ag.first_shard, args.ag.num_chunks = ag.num_shards, ag.first_shard, ag.num_chunks
        pull = getattr(ag, "pull", None)
        args.ag.pull = pull.data_ptr() if pull is not None else None
    args.tile_n, args.cta_group, args.max_ctas = tile_n, cta_group, max_ctas
    args.scheduler = scheduler
    args.split_k = split_k     # 0 = the library decides (needs the workspace launch_gemm_args attaches), 1 = off
    if workspace is not None:  # an explicit scratch tensor (zeroed by the caller) instead of the per-stream one
        args.workspace, args.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    args.timeout_ns = timeout_ns
    if prof is not None:
        args.prof = prof.data_ptr()
    return args


_gemm_fn = _lib.lib.qk_gemm_blockscaled
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None) or (lambda i: torch.cuda.current_stream(i).cuda_stream)


WORKSPACE_BYTES = 32 << 20
_workspaces: dict = {}


def workspace(index: int, stream: int):
    """(pointer, bytes) of the split-K scratch of one (device, stream): zeroed once, and launches
    on one stream run in order, so they can share it; other streams get their own.  None while a CUDA
    graph is being captured on a stream that has no scratch yet (an allocation made during capture would
    belong to the graph's pool): such launches run unsplit."""
    ws = _workspaces.get((index, stream))
    if ws is None:
        if torch.cuda.is_current_stream_capturing():
            return None
        t = torch.zeros(WORKSPACE_BYTES, dtype=torch.uint8, device=torch.device("cuda", index))
        ws = _workspaces[(index, stream)] = (t.data_ptr(), WORKSPACE_BYTES, t)
    return ws


def launch_gemm_args(args, dev: torch.device, status: Optional[torch.Tensor] = None, stream: Optional[int] = None) -> None:
    """Launch a filled argument block on `dev` (current stream unless given)."""
    st = status if status is not None else status_buffer(dev)
    args.status = st.data_ptr()
    idx = dev.index
    if idx is None or idx == torch.cuda.current_device():
        if idx is None:
            idx = torch.cuda.current_device()
        args.stream = stream if stream is not None else _raw_stream(idx)
        if args.split_k != 1 and not args.workspace:
            ws = workspace(idx, args.stream or 0)
            if ws is not None:
                args.workspace, args.workspace_bytes = ws[0], ws[1]
        rc = _gemm_fn(C.byref(args))
    else:
        with torch.cuda.device(dev):
            args.stream = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
            if args.split_k != 1 and not args.workspace:
                ws = workspace(idx, args.stream or 0)
                if ws is not None:
                    args.workspace, args.workspace_bytes = ws[0], ws[1]
            rc = _gemm_fn(C.byref(args))
    if rc:
        _lib.check(rc, "qk_gemm_blockscaled")


def gemm_blockscaled(fmt, a, sfa, b, sfb, m, n, k, *, status=None, stream=None, **kw):
    """One launch of the block-scaled GEMM (see build_gemm_args for the operands)."""
    args = build_gemm_args(fmt, a, sfa, b, sfb, m, n, k, **kw)
    launch_gemm_args(args, a.device, status, stream)
    return args
