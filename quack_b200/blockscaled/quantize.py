"""Block-scale quantizers and scale-factor layout helpers (host side).

Same names, arguments and results as ``quack/blockscaled/quantize.py`` in the reference,
with the arithmetic done by the sm_100a kernels of libquack_b200 (``qk_quantize_blockscaled``,
``qk_scale_pack_blocked`` ...).  The quantizers need CUDA tensors: there is no CPU path.

Implemented on the GPU: ``to_mx`` (MXFP8 E4M3 / E5M2, rceil or floor scales; reference :47-114),
``to_mxfp4`` (:285-316), ``to_nvfp4`` (:403-442), ``nvfp4_per_tensor_scale`` (:398-400), the blocked
scale layout (:637-674).  The dequantisation helpers (:593-618) are plain torch: they are the
reference-side tools of the parity tests, not a kernel path.
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _ops
from .._lib import FMT_MXFP4, FMT_MXFP8_E4M3, FMT_MXFP8_E5M2, FMT_NVFP4, SCALING_FLOOR, SCALING_RCEIL

F8E4M3_MAX = 448.0
F8E5M2_MAX = 57344.0
F4_E2M1_MAX = 6.0
E4M3_EPS = 2.0 ** -6

# code -> value table of E2M1 (bit 3 = sign); reference :541-558
FP4_E2M1FN_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def _check_input(x: torch.Tensor, block: int) -> None:
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise AssertionError(f"expected bf16 or fp32 input, got {x.dtype}")
    if x.shape[-1] % block != 0:
        raise AssertionError(f"last dim ({x.shape[-1]}) must be divisible by {block}")
    if not x.is_contiguous():
        raise AssertionError("input must be contiguous")


def to_mx(data_hp: torch.Tensor, block_size: int = 32, scaling_mode: str = "rceil",
          elem_dtype: torch.dtype = torch.float8_e4m3fn):
    """MXFP8 quantisation along the last dim -> (qdata ``elem_dtype``, scale float8_e8m0fnu
    (..., K/32)).  ``elem_dtype`` float8_e4m3fn or float8_e5m2; ``scaling_mode`` "rceil" (the
    scale is the smallest power of two that keeps the block maximum in range) or "floor"
    (exponent of the maximum minus the exponent of the format maximum; maxima may saturate)."""
    _check_input(data_hp, block_size)
    assert scaling_mode in ("rceil", "floor")
    assert elem_dtype in (torch.float8_e4m3fn, torch.float8_e5m2)
    if block_size != 32:
        raise NotImplementedError("quack_b200 implements to_mx for block_size=32 (the MX block size)")
    shape = data_hp.shape
    x2 = data_hp.reshape(-1, shape[-1])
    fmt = FMT_MXFP8_E4M3 if elem_dtype == torch.float8_e4m3fn else FMT_MXFP8_E5M2
    codes, sf_blocked = _ops.quantize_rows(x2, fmt, None, SCALING_RCEIL if scaling_mode == "rceil" else SCALING_FLOOR)
    sf2d = _ops.scale_unpack(sf_blocked, x2.shape[0], shape[-1] // 32)
    return (codes.view(elem_dtype).reshape(shape),
            sf2d.view(torch.float8_e8m0fnu).reshape(*shape[:-1], shape[-1] // 32))


def to_mx_dim0(data_hp: torch.Tensor, block_size: int = 32, scaling_mode: str = "rceil"):
    """MXFP8-E4M3 quantisation of a 2-D tensor along dim 0 ("column-wise"): the numerics of ``to_mx`` on the
    transposed input; qdata keeps the input's (M, K) row-major layout, the scale blocks run along M ->
    (qdata float8_e4m3fn (M, K), scale float8_e8m0fnu (M / 32, K)); reference :117-162.  The kernel produces the
    transposed codes and the blocked scales of the (K, M) operand in one pass over the input; the two results
    are brought into this function's layouts by transposes of the 1-byte data."""
    assert data_hp.ndim == 2 and data_hp.dtype in (torch.bfloat16, torch.float32)
    assert data_hp.shape[0] % block_size == 0 and data_hp.is_contiguous()
    assert scaling_mode in ("rceil", "floor")
    if block_size != 32:
        raise NotImplementedError("quack_b200 implements to_mx_dim0 for block_size=32 (the MX block size)")
    m, k = data_hp.shape
    codes_t, sf_blocked = _ops.quantize_cols(data_hp, FMT_MXFP8_E4M3, None,
                                             SCALING_RCEIL if scaling_mode == "rceil" else SCALING_FLOOR)
    sf2d_t = _ops.scale_unpack(sf_blocked, k, m // 32)       # (K, M / 32)
    return (codes_t.t().contiguous().view(torch.float8_e4m3fn), sf2d_t.t().contiguous().view(torch.float8_e8m0fnu))


def to_mx_e5m2(data_hp: torch.Tensor, block_size: int = 32, scaling_mode: str = "rceil"):
    """``to_mx`` with the E5M2 target (format maximum 57344); reference :111-114."""
    return to_mx(data_hp, block_size, scaling_mode, elem_dtype=torch.float8_e5m2)


def to_mxfp4(x: torch.Tensor, block_size: int = 32):
    """MXFP4 quantisation: E2M1 codes packed two per byte (first value in the low nibble) + per-32
    E8M0 scales, floor rule -> (packed uint8 (..., K/2), scale float8_e8m0fnu (..., K/32));
    reference :285-316."""
    _check_input(x, block_size)
    if block_size != 32:
        raise NotImplementedError("quack_b200 implements to_mxfp4 for block_size=32 (the MX block size)")
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    codes, sf_blocked = _ops.quantize_rows(x2, FMT_MXFP4)
    sf2d = _ops.scale_unpack(sf_blocked, x2.shape[0], shape[-1] // 32)
    return (codes.reshape(*shape[:-1], shape[-1] // 2),
            sf2d.view(torch.float8_e8m0fnu).reshape(*shape[:-1], shape[-1] // 32))


def nvfp4_per_tensor_scale(amax: torch.Tensor) -> torch.Tensor:
    """amax / (448 * 6), fp32 (reference :398-400)."""
    return amax.to(torch.float32) / (F8E4M3_MAX * F4_E2M1_MAX)


def to_nvfp4(x: torch.Tensor, block_size: int = 16, per_tensor_scale: Optional[torch.Tensor] = None):
    """NVFP4 quantisation -> (packed uint8 (..., K/2), scale float8_e4m3fn (..., K/16),
    per-tensor scale (1.0 when none was given))."""
    _check_input(x, 16)
    assert block_size == 16, "NVFP4 requires block_size=16"
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    pts = None
    if per_tensor_scale is not None:
        pts = per_tensor_scale.to(device=x.device, dtype=torch.float32).reshape(1)
    codes, sf_blocked = _ops.quantize_rows(x2, FMT_NVFP4, pts)
    sf2d = _ops.scale_unpack(sf_blocked, x2.shape[0], shape[-1] // 16)
    ret_pts = (torch.tensor(1.0, dtype=torch.float32, device=x.device) if per_tensor_scale is None
               else per_tensor_scale.to(torch.float32))
    return (codes.reshape(*shape[:-1], shape[-1] // 2),
            sf2d.view(torch.float8_e4m3fn).reshape(*shape[:-1], shape[-1] // 16), ret_pts)


# name -> (eager fn, "compiled" fn).  Both slots hold the CUDA kernel: there is no tracing
# compiler in this package.  Formats without a kernel are absent (from_parts only).
QUANTIZERS = {
    "mxfp8_e4m3": (to_mx, to_mx),
    "mxfp8_e5m2": (to_mx_e5m2, to_mx_e5m2),
    "mxfp4": (to_mxfp4, to_mxfp4),
    "nvfp4": (to_nvfp4, to_nvfp4),
}
to_mx_compiled = to_mx
to_mx_dim0_compiled = to_mx_dim0
to_mx_e5m2_compiled = to_mx_e5m2
to_mxfp4_compiled = to_mxfp4
to_nvfp4_compiled = to_nvfp4


def quantize_to_blocked(x2: torch.Tensor, format_name: str, per_tensor_scale: Optional[torch.Tensor] = None):
    """(rows, K) -> (codes uint8, blocked scales uint8 (rm, rk, 32, 4, 4)) in ONE kernel: the
    scale bytes never exist in the 2-D layout (the reference quantises, then swizzles in a
    second kernel; quack/blockscaled/operand.py:766-780)."""
    return _ops.quantize_rows(x2, _ops.format_id(format_name), per_tensor_scale)


def check_blocked_scale_atom(SF: torch.Tensor, name: str = "scale") -> None:
    """Rank 5/6 with a trailing contiguous (32, 4, 4) atom (strides (16, 4, 1)); reference
    :621-634."""
    if SF.ndim not in (5, 6) or tuple(SF.shape[-3:]) != (32, 4, 4):
        raise ValueError(
            f"{name}: expected (rm, rk, 32, 4, 4) or (L, rm, rk, 32, 4, 4) blocked scale factors, "
            f"got shape {tuple(SF.shape)}")
    if tuple(SF.stride()[-3:]) != (16, 4, 1):
        raise ValueError(
            f"{name}: inner (32, 4, 4) atom must be contiguous with strides (16, 4, 1), got {SF.stride()[-3:]}")


def _pack_torch(u8: torch.Tensor) -> torch.Tensor:
    l, mn, sfk = u8.shape
    rm, rk = -(-mn // 128), -(-sfk // 4)
    pad = torch.zeros(l, rm * 128, rk * 4, dtype=torch.uint8, device=u8.device)
    pad[:, :mn, :sfk] = u8
    return pad.view(l, rm, 4, 32, rk, 4).permute(0, 1, 4, 3, 2, 5).contiguous()


def pack_scale_2d_to_blocked_contig(scale_2d: torch.Tensor) -> torch.Tensor:
    """(l, mn, sf_k) or (mn, sf_k) scales -> contiguous (l, rm, rk, 32, 4, 4), zero padded
    (reference :637-662).  CUDA tensors go through ``qk_scale_pack_blocked``; CPU tensors
    (host-side bookkeeping only) are permuted with torch."""
    if scale_2d.dim() == 2:
        scale_2d = scale_2d.unsqueeze(0)
    assert scale_2d.dim() == 3, f"expected (l, mn, sf_k), got shape {tuple(scale_2d.shape)}"
    dt = scale_2d.dtype
    u8 = scale_2d.contiguous().view(torch.uint8)
    if u8.is_cuda:
        out = torch.stack([_ops.scale_pack(u8[i]) for i in range(u8.shape[0])])
    else:
        out = _pack_torch(u8)
    return out.view(dt)


def unpack_scale_blocked_to_2d(blocked: torch.Tensor, mn: int, sf_k: int) -> torch.Tensor:
    """(l, rm, rk, 32, 4, 4) -> (l, mn, sf_k) (reference :665-674)."""
    assert tuple(blocked.shape[3:]) == (32, 4, 4)
    dt = blocked.dtype
    u8 = blocked.view(torch.uint8)
    l, rm, rk = u8.shape[:3]
    if u8.is_cuda and u8.is_contiguous():
        out = torch.stack([_ops.scale_unpack(u8[i], mn, sf_k) for i in range(l)])
    else:
        out = u8.permute(0, 1, 4, 3, 2, 5).reshape(l, rm * 128, rk * 4)[:, :mn, :sf_k].contiguous()
    return out.view(dt)


def to_blocked(input_matrix: torch.Tensor) -> torch.Tensor:
    """(H, W) scales -> flat blocked buffer, the layout cuBLAS block scaling consumes
    (reference :511-532)."""
    return pack_scale_2d_to_blocked_contig(input_matrix).reshape(-1)


def dequant_operand(x: torch.Tensor, fmt=None) -> torch.Tensor:
    """Codes -> fp32 values without the scale factors (reference :593-618).  fp4x2 bytes
    unpack to two values (low nibble first)."""
    if x.dtype == torch.float4_e2m1fn_x2:
        u8 = x.view(torch.uint8)
        table = torch.tensor(FP4_E2M1FN_VALUES, dtype=torch.float32, device=x.device)
        lo, hi = table[(u8 & 0xF).long()], table[(u8 >> 4).long()]
        return torch.stack([lo, hi], dim=-1).reshape(*x.shape[:-1], x.shape[-1] * 2)
    if x.dtype == torch.uint8:
        raise ValueError("uint8 operand bytes are ambiguous; quack_b200 decodes float8 and float4_e2m1fn_x2 storage")
    return x.float()
