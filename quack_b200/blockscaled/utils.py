"""Thin wrappers around the container API, mirroring the parts of
``quack/blockscaled/utils.py`` (reference) that belong to the quantised-linear path:
``blockscaled_quantize`` (:262-278), ``scale_view_for_kernel`` (:306-323),
``scale_blocked_for_cublas`` (:326-332), ``blockscaled_gemm_reference`` (:957-967) and the
``BLOCKSCALED_FORMATS`` table (:248-252)."""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from .operand import BLOCKSCALED_FORMAT_REGISTRY, BlockScaledOperand, legacy_format_name
from .quantize import (QUANTIZERS, dequant_operand, pack_scale_2d_to_blocked_contig,  # noqa: F401
                       unpack_scale_blocked_to_2d)

# legacy short name -> (storage dtype, scale dtype, scale vector size) of the formats that
# have a quantizer kernel here
BLOCKSCALED_FORMATS = {
    legacy_format_name(f): (f.qdata_dtype, f.scale_dtype, f.sf_vec_size)
    for f in BLOCKSCALED_FORMAT_REGISTRY.values() if f.name in QUANTIZERS
}


def blockscaled_quantize(x: torch.Tensor, format: str = "mxfp8",
                         per_tensor_scale: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Raw ``(qdata, blocked scales)`` of ``BlockScaledOperand.quantize``.  GEMMs take the
    container, so wrap the parts with ``BlockScaledOperand.from_parts`` (passing the NVFP4
    per-tensor scale there)."""
    op = BlockScaledOperand.quantize(x, format, per_tensor_scale=per_tensor_scale)
    return op.qdata, op.scale


def blockscaled_quantize_dim0(x: torch.Tensor, format: str = "mxfp8") -> Tuple[torch.Tensor, torch.Tensor]:
    """Quantise an (M, K) tensor along M (dim 0) -> ``(q, sf)``: q (M, K) fp8 in the layout of ``x``, sf the
    blocked scale factors of the logical operand (mn = K, sf_k = M / 32); reference :281-303.  Wrap with
    ``BlockScaledOperand.from_parts(q, sf, "mxfp8", quant_dim=-2)``.  (The GEMM of this package takes K-major
    operands: use ``BlockScaledOperand.quantize(x, format, dim=-2)``, which keeps the kernel's transposed
    codes, to feed it.)"""
    from .. import _ops
    assert format in ("mxfp8", "mxfp8_e4m3"), "dim0 quantization currently supports mxfp8 only"
    assert x.ndim == 2, f"expected (M, K), got shape {tuple(x.shape)}"
    assert x.shape[0] % 32 == 0, f"M ({x.shape[0]}) must be divisible by 32"
    codes_t, sf = _ops.quantize_cols(x, _ops.format_id("mxfp8_e4m3"))
    return codes_t.t().contiguous().view(torch.float8_e4m3fn), sf.view(torch.float8_e8m0fnu)


def scale_view_for_kernel(scale_contig: torch.Tensor, mn: int, sf_k: int, l: int) -> torch.Tensor:
    """Check a (l, rm, rk, 32, 4, 4) scale tensor (only the 512-byte atom must be contiguous;
    outer strides are free) and return it unchanged."""
    rm, rk = -(-mn // 128), -(-sf_k // 4)
    assert tuple(scale_contig.shape) == (l, rm, rk, 32, 4, 4), (
        f"expected (l, rm, rk, 32, 4, 4) = ({l}, {rm}, {rk}, 32, 4, 4), got {tuple(scale_contig.shape)}")
    assert tuple(scale_contig.stride()[-3:]) == (16, 4, 1), (
        f"inner (32, 4, 4) atom must be contiguous with strides (16, 4, 1), got {scale_contig.stride()[-3:]}")
    return scale_contig


def scale_blocked_for_cublas(scale_contig: torch.Tensor, mn: int, sf_k: int, l_idx: int = 0) -> torch.Tensor:
    """One batch entry of a contiguous blocked scale tensor as the flat buffer
    ``torch._scaled_mm`` expects."""
    assert scale_contig.is_contiguous() and scale_contig.dim() == 6
    return scale_contig[l_idx].reshape(-1)


def blockscaled_gemm_reference(a_ref, b_ref, sfa_ref, sfb_ref) -> torch.Tensor:
    """einsum reference on (m,k,l)/(n,k,l) value and scale tensors."""
    return torch.einsum("mkl,nkl->mnl", a_ref * sfa_ref, b_ref * sfb_ref)
