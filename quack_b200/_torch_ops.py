"""``torch.library`` custom ops of the block-scaled GEMMs, so that the package can sit inside a
``torch.compile``d model and its launches can be captured in CUDA graphs.

The reference registers ``quack::gemm_out``, ``quack::gemm_quant_out``, ``quack::gemm_add_out``,
``quack::gemm_add_inplace``, ``quack::gemm_act_out`` and ``quack::gemm_gated_out`` as mutating ops
with no-op fakes (quack/gemm_interface.py:1311-1449, :1686-1842, :2062-2122, :2242-2456,
:3052-3068): ``out`` is allocated by the caller in the traced graph, the op only fills it.  The
same names and the same flattening rules are used here:

* containers are unpacked before the boundary (a schema has no ``BlockScaledOperand`` type):
  codes, blocked scale factors and the two format names travel as separate arguments;
* ``float | Tensor`` arguments are split into a float and an optional tensor (``alpha`` +
  ``alpha_tensor``); the two NVFP4 per-tensor scales travel as ``alpha_tensor`` /
  ``alpha_tensor2`` and are multiplied in by the kernel (no torch multiply in the graph);
* E8M0 scale factors and 4-bit codes cross as ``uint8`` views while compiling and are viewed back
  from the format name inside the op (the reference's work-around for functionalisation of
  ``float8_e8m0fnu`` inputs, quack/gemm_interface.py:332-355).

The namespace is ``quack`` (drop-in for the reference's graphs); when the reference package has
already registered it in this process, ``quack_b200`` is used instead.  The op bodies call the
kernel-level ``quack_b200.gemm.gemm``; nothing here runs on the CPU.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import gemm as _kernel
from .blockscaled.operand import BlockScaledFormat

__all__ = ["NAMESPACE", "ops", "encode", "compiling"]


def _pick_namespace() -> str:
    try:
        torch.ops.quack.gemm_out   # noqa: B018  (attribute lookup raises when the op does not exist)
        return "quack_b200"
    except (AttributeError, RuntimeError):
        return "quack"


NAMESPACE = _pick_namespace()


def compiling() -> bool:
    return torch.compiler.is_compiling()


def encode(t: Optional[Tensor]) -> Optional[Tensor]:
    """Scale factors / codes whose dtype the compile stack handles badly cross the boundary as uint8."""
    if t is not None and t.dtype in (torch.float8_e8m0fnu, torch.float4_e2m1fn_x2):
        return t.view(torch.uint8)
    return t


def _codes(t: Tensor, fmt_name: str) -> Tensor:
    want = BlockScaledFormat.from_name(fmt_name).qdata_dtype
    return t if t.dtype == want else t.view(want)


def _scales(t: Optional[Tensor], fmt_name: Optional[str]) -> Optional[Tensor]:
    if t is None or t.dtype != torch.uint8:
        return t
    return t.view(BlockScaledFormat.from_name(fmt_name).scale_dtype)


def _merge(value, tensor_value):
    return tensor_value if tensor_value is not None else value


def _nk(B: Tensor) -> Tensor:
    """(K, N) logical view of a K-major (N, K) weight -> the (N, K) storage."""
    Bt = B.mT
    if Bt.stride(-1) != 1:
        raise NotImplementedError("B must be the .mT view of a K-major (N, K) weight")
    return Bt


def _define(name: str, mutates):
    return torch.library.custom_op(f"{NAMESPACE}::{name}", mutates_args=mutates, device_types="cuda")


def _noop_fake(op):
    @op.register_fake
    def _fake(*args, **kwargs):
        return None
    return op


@_define("gemm_out", ("out",))
def gemm_out(A: Tensor, B: Tensor, out: Tensor, bias: Optional[Tensor] = None, alpha: float = 1.0,
             alpha_tensor: Optional[Tensor] = None, alpha_tensor2: Optional[Tensor] = None, dynamic_scheduler: bool = False,
             tuned: bool = True, SFA: Optional[Tensor] = None, SFB: Optional[Tensor] = None, bs_format_a: Optional[str] = None,
             bs_format_b: Optional[str] = None, split_k: Optional[int] = 1, split_k_mode: int = 0, tile_m: int = 0,
             tile_n: int = 0, cluster_m: int = 0) -> None:
    """``out = alpha * A @ B + bias`` (block-scaled A (M, K) and B (K, N))."""
    has_dev = alpha_tensor is not None
    _kernel.gemm(_codes(A, bs_format_a), _codes(_nk(B), bs_format_b), out, None, None, tile_m, tile_n, cluster_m, 1,
                 is_dynamic_persistent=dynamic_scheduler, rowvec_bias=bias, alpha=_merge(alpha, alpha_tensor),
                 alpha_dev2=alpha_tensor2, alpha_host=alpha if has_dev else 1.0, SFA=_scales(SFA, bs_format_a),
                 SFB=_scales(SFB, bs_format_b), bs_format_a=bs_format_a, bs_format_b=bs_format_b, split_k=split_k or 1,
                 split_k_mode=split_k_mode)


@_define("gemm_quant_out", ("out", "SFD"))
def gemm_quant_out(A: Tensor, B: Tensor, out: Tensor, SFD: Tensor, bs_format_d: str, sfd_dim: str = "n",
                   bias: Optional[Tensor] = None, alpha: float = 1.0, alpha_tensor: Optional[Tensor] = None,
                   alpha_tensor2: Optional[Tensor] = None, dynamic_scheduler: bool = False, tuned: bool = True,
                   sfd_norm_const: float = 1.0, sfd_norm_const_tensor: Optional[Tensor] = None, SFA: Optional[Tensor] = None,
                   SFB: Optional[Tensor] = None, bs_format_a: Optional[str] = None, bs_format_b: Optional[str] = None,
                   tile_m: int = 0, tile_n: int = 0, cluster_m: int = 0) -> None:
    """GEMM with re-quantised output: codes in ``out``, blocked scale factors in ``SFD`` (vectors along N)."""
    if sfd_dim != "n":
        raise NotImplementedError("column-direction output scale factors have no kernel in quack_b200")
    has_dev = alpha_tensor is not None
    _kernel.gemm(_codes(A, bs_format_a), _codes(_nk(B), bs_format_b), _codes(out, bs_format_d), None, None, tile_m, tile_n,
                 cluster_m, 1, is_dynamic_persistent=dynamic_scheduler, rowvec_bias=bias, alpha=_merge(alpha, alpha_tensor),
                 alpha_dev2=alpha_tensor2, alpha_host=alpha if has_dev else 1.0, SFA=_scales(SFA, bs_format_a),
                 SFB=_scales(SFB, bs_format_b), bs_format_a=bs_format_a, bs_format_b=bs_format_b,
                 SFD=_scales(SFD, bs_format_d), sfd_norm_const=_merge(sfd_norm_const, sfd_norm_const_tensor),
                 bs_format_d=bs_format_d)


@_define("gemm_add_out", ("out",))
def gemm_add_out(A: Tensor, B: Tensor, C: Tensor, out: Tensor, bias: Optional[Tensor] = None, alpha: float = 1.0,
                 beta: float = 1.0, alpha_tensor: Optional[Tensor] = None, beta_tensor: Optional[Tensor] = None,
                 alpha_tensor2: Optional[Tensor] = None, dynamic_scheduler: bool = False, tuned: bool = True,
                 SFA: Optional[Tensor] = None, SFB: Optional[Tensor] = None, bs_format_a: Optional[str] = None,
                 bs_format_b: Optional[str] = None, split_k: Optional[int] = 1, split_k_mode: int = 0, tile_m: int = 0,
                 tile_n: int = 0, cluster_m: int = 0) -> None:
    """``out = alpha * A @ B + beta * C + bias``; ``C`` may be ``out`` itself."""
    has_dev = alpha_tensor is not None
    _kernel.gemm(_codes(A, bs_format_a), _codes(_nk(B), bs_format_b), out, C, None, tile_m, tile_n, cluster_m, 1,
                 is_dynamic_persistent=dynamic_scheduler, rowvec_bias=bias, alpha=_merge(alpha, alpha_tensor),
                 beta=_merge(beta, beta_tensor), alpha_dev2=alpha_tensor2, alpha_host=alpha if has_dev else 1.0,
                 SFA=_scales(SFA, bs_format_a), SFB=_scales(SFB, bs_format_b), bs_format_a=bs_format_a,
                 bs_format_b=bs_format_b, split_k=split_k or 1, split_k_mode=split_k_mode)


@_define("gemm_add_inplace", ("out",))
def gemm_add_inplace(A: Tensor, B: Tensor, out: Tensor, bias: Optional[Tensor] = None, alpha: float = 1.0,
                     beta: float = 1.0, alpha_tensor: Optional[Tensor] = None, beta_tensor: Optional[Tensor] = None,
                     alpha_tensor2: Optional[Tensor] = None, dynamic_scheduler: bool = False, tuned: bool = True,
                     SFA: Optional[Tensor] = None, SFB: Optional[Tensor] = None, bs_format_a: Optional[str] = None,
                     bs_format_b: Optional[str] = None, split_k: Optional[int] = 1, split_k_mode: int = 0, tile_m: int = 0,
                     tile_n: int = 0, cluster_m: int = 0) -> None:
    """``out = alpha * A @ B + beta * out + bias``: every element is read by the thread that writes it."""
    has_dev = alpha_tensor is not None
    _kernel.gemm(_codes(A, bs_format_a), _codes(_nk(B), bs_format_b), out, out, None, tile_m, tile_n, cluster_m, 1,
                 is_dynamic_persistent=dynamic_scheduler, rowvec_bias=bias, alpha=_merge(alpha, alpha_tensor),
                 beta=_merge(beta, beta_tensor), alpha_dev2=alpha_tensor2, alpha_host=alpha if has_dev else 1.0,
                 SFA=_scales(SFA, bs_format_a), SFB=_scales(SFB, bs_format_b), bs_format_a=bs_format_a,
                 bs_format_b=bs_format_b, split_k=split_k or 1, split_k_mode=split_k_mode)


def _act_body(A, B, preact_out, postact_out, C, bias, activation, alpha, alpha_tensor, alpha_tensor2, dynamic_scheduler, SFA,
              SFB, bs_format_a, bs_format_b, tile_m, tile_n, cluster_m, exact_activation, SFD=None, bs_format_d=None,
              sfd_norm_const=None):
    has_dev = alpha_tensor is not None
    post = postact_out if bs_format_d is None else _codes(postact_out, bs_format_d)
    _kernel.gemm(_codes(A, bs_format_a), _codes(_nk(B), bs_format_b), preact_out, C, None, tile_m, tile_n, cluster_m, 1,
                 is_dynamic_persistent=dynamic_scheduler, rowvec_bias=bias, alpha=_merge(alpha, alpha_tensor),
                 alpha_dev2=alpha_tensor2, alpha_host=alpha if has_dev else 1.0, SFA=_scales(SFA, bs_format_a),
                 SFB=_scales(SFB, bs_format_b), bs_format_a=bs_format_a, bs_format_b=bs_format_b, activation=activation,
                 postact_out=post, exact_activation=exact_activation, SFD=_scales(SFD, bs_format_d),
                 sfd_norm_const=sfd_norm_const, bs_format_d=bs_format_d)


# one op per set of mutated tensors (an optional tensor cannot be named in mutates_args)
@_define("gemm_act_out", ("preact_out", "postact_out"))
def gemm_act_out(A: Tensor, B: Tensor, preact_out: Tensor, postact_out: Tensor, C: Optional[Tensor] = None,
                 bias: Optional[Tensor] = None, activation: Optional[str] = None, alpha: float = 1.0,
                 alpha_tensor: Optional[Tensor] = None, alpha_tensor2: Optional[Tensor] = None,
                 dynamic_scheduler: bool = False, tuned: bool = True, SFA: Optional[Tensor] = None,
                 SFB: Optional[Tensor] = None, bs_format_a: Optional[str] = None, bs_format_b: Optional[str] = None,
                 tile_m: int = 0, tile_n: int = 0, cluster_m: int = 0, exact_activation: bool = False) -> None:
    """``preact_out = alpha * A @ B + C + bias``; ``postact_out = act(preact)`` (plain or gated)."""
    _act_body(A, B, preact_out, postact_out, C, bias, activation, alpha, alpha_tensor, alpha_tensor2, dynamic_scheduler, SFA, SFB,
              bs_format_a, bs_format_b, tile_m, tile_n, cluster_m, exact_activation)


@_define("gemm_act_out_nopreact", ("postact_out",))
def gemm_act_out_nopreact(A: Tensor, B: Tensor, postact_out: Tensor, C: Optional[Tensor] = None,
                          bias: Optional[Tensor] = None, activation: Optional[str] = None, alpha: float = 1.0,
                          alpha_tensor: Optional[Tensor] = None, alpha_tensor2: Optional[Tensor] = None,
                          dynamic_scheduler: bool = False, tuned: bool = True, SFA: Optional[Tensor] = None,
                          SFB: Optional[Tensor] = None, bs_format_a: Optional[str] = None, bs_format_b: Optional[str] = None,
                          tile_m: int = 0, tile_n: int = 0, cluster_m: int = 0, exact_activation: bool = False) -> None:
    """``postact_out = act(alpha * A @ B + C + bias)``; the pre-activation is not stored."""
    _act_body(A, B, None, postact_out, C, bias, activation, alpha, alpha_tensor, alpha_tensor2, dynamic_scheduler, SFA, SFB,
              bs_format_a, bs_format_b, tile_m, tile_n, cluster_m, exact_activation)


@_define("gemm_act_quant_out", ("postact_out", "SFD"))
def gemm_act_quant_out(A: Tensor, B: Tensor, postact_out: Tensor, SFD: Tensor, bs_format_d: str,
                       bias: Optional[Tensor] = None, activation: Optional[str] = None, alpha: float = 1.0,
                       alpha_tensor: Optional[Tensor] = None, alpha_tensor2: Optional[Tensor] = None,
                       dynamic_scheduler: bool = False, sfd_norm_const: float = 1.0,
                       sfd_norm_const_tensor: Optional[Tensor] = None, SFA: Optional[Tensor] = None,
                       SFB: Optional[Tensor] = None, bs_format_a: Optional[str] = None, bs_format_b: Optional[str] = None,
                       tile_m: int = 0, tile_n: int = 0, cluster_m: int = 0, exact_activation: bool = True) -> None:
    """Fused up-projection: ``act(alpha * A @ B + bias)`` re-quantised into ``postact_out`` / ``SFD``."""
    _act_body(A, B, None, postact_out, None, bias, activation, alpha, alpha_tensor, alpha_tensor2, dynamic_scheduler, SFA, SFB,
              bs_format_a, bs_format_b, tile_m, tile_n, cluster_m, exact_activation, SFD=SFD, bs_format_d=bs_format_d,
              sfd_norm_const=_merge(sfd_norm_const, sfd_norm_const_tensor))


for _op in (gemm_out, gemm_quant_out, gemm_add_out, gemm_add_inplace, gemm_act_out, gemm_act_out_nopreact, gemm_act_quant_out):
    _noop_fake(_op)

# the gated variant shares the body of gemm_act_out in this package (one kernel serves both)
gemm_gated_out = gemm_act_out

ops = getattr(torch.ops, NAMESPACE)
