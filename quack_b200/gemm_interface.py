"""Public GEMM API for block-scaled operands, drop-in for the block-scaled surface of
``quack.gemm_interface`` (reference): ``gemm`` (:974-1308), ``gemm_act`` / ``gemm_gated``
(:2123-2239), the torch references ``gemm_blockscaled_ref`` (:1521-1559), ``gemm_ref``
(:1452-1518), ``gemm_act_ref`` (:2288-2334) and the activation tables (:81-102).

Operands are ``BlockScaledOperand`` containers; A is quantised along its last dim, B is the
``.mT`` view of an (N, K) weight quantised along K.  NVFP4 per-tensor scales are folded into
alpha on the device (no host sync).  Arguments of the reference that select features outside
the quantised-linear path are accepted and rejected with ``NotImplementedError``.
"""

from __future__ import annotations

import os
from functools import partial
from typing import Literal, NamedTuple, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _torch_ops as _tops
from . import gemm as _kernel
from .blockscaled.operand import BlockScaledFormat, BlockScaledOperand, mma_kind_for_pair
from .gemm_config import GemmConfig, SplitKMode, blockscaled_default_config, config_to_kernel  # noqa: F401


def _silu_tanh(x: Tensor) -> Tensor:
    h = 0.5 * x
    return h * torch.tanh(h) + h


act_to_pytorch_fn_map = {
    None: lambda x: x,
    "silu": F.silu,
    "silu-tanh": _silu_tanh,
    "relu": F.relu,
    "relu_sq": lambda x: F.relu(x).square(),
    "gelu_tanh_approx": partial(F.gelu, approximate="tanh"),
    "tanh": torch.tanh,
}

gated_to_pytorch_fn_map = {
    "swiglu": lambda gate, up: F.silu(gate) * up,
    "swiglu-tanh": lambda gate, up: _silu_tanh(gate) * up,
    "swiglu_oai": lambda gate, up: gate * torch.sigmoid(1.702 * gate) * (up + 1),
    "swiglu_oai-tanh": lambda gate, up: (0.5 * gate * torch.tanh(1.702 * 0.5 * gate) + 0.5 * gate) * (up + 1),
    "reglu": lambda gate, up: F.relu(gate) * up,
    "geglu": lambda gate, up: F.gelu(gate, approximate="tanh") * up,
    "glu": lambda gate, up: torch.sigmoid(gate) * up,
}

_EXACT_ACT_DEFAULT = os.environ.get("QK_EXACT_ACT", "0") not in ("", "0")

# block-scaled formats the epilogue can re-quantise into (the reference's set, tests/test_gemm_quant_out.py:104)
_OUT_FORMATS = ("mxfp8_e4m3", "mxfp4", "nvfp4")

# activations with a fused epilogue in the B200 kernel
_KERNEL_ACTS = (None, "relu", "relu_sq", "silu", "gelu_tanh_approx", "tanh", "swiglu", "reglu", "geglu", "glu")

Activation = Literal[None, "silu", "silu-tanh", "relu", "relu_sq", "gelu_tanh_approx", "tanh", "swiglu", "swiglu-tanh",
                     "swiglu_oai", "swiglu_oai-tanh", "reglu", "geglu", "glu"]


class _Operand(NamedTuple):
    data: Tensor
    sf: Optional[Tensor] = None
    fmt: Optional[BlockScaledFormat] = None
    per_tensor_scale: Optional[Tensor] = None
    quant_dim: Optional[int] = None


def _unpack_operand(X) -> _Operand:
    if isinstance(X, BlockScaledOperand):
        return _Operand(X.qdata, X.scale, X.format, X.per_tensor_scale, X.quant_dim)
    if isinstance(X, (tuple, list)):
        raise TypeError("blockscaled operands must be BlockScaledOperand containers; (data, scale_factor) tuples are "
                        "no longer accepted - wrap the parts with quack.BlockScaledOperand.from_parts(data, "
                        "scale_factor, format)")
    return _Operand(X)


def _prep_blockscaled(opA: _Operand, opB: _Operand):
    """Pair legality and operand orientation (reference :203-235)."""
    assert (opA.sf is None) == (opB.sf is None), "A and B must both (or neither) carry scale factors"
    if opA.sf is None:
        raise NotImplementedError("quack_b200.gemm_interface implements block-scaled GEMMs only: pass "
                                  "BlockScaledOperand operands (dense bf16/fp16 GEMM is outside this package)")
    mma_kind_for_pair(opA.fmt, opB.fmt)
    if opA.quant_dim != -1:
        raise ValueError("A must be quantized along its last dim (the contraction dim K of (M, K)); got scales "
                         "along dim -2 - remove a stray transpose or quantize with dim=-1")
    if opB.quant_dim != -2:
        raise ValueError("B must be quantized along dim -2 (the contraction dim K of (K, N)); pass W.mT of an "
                         "(N, K) weight, or quantize the (K, N) data with dim=-2")
    return opA.sf, opB.sf, opA.fmt.name, opB.fmt.name


def _fold_per_tensor_scales(alpha, opA: _Operand, opB: _Operand):
    """alpha <- alpha * ptsA * ptsB without a host sync (reference :238-247).  Returns
    ``(alpha, alpha_dev2, alpha_host)`` for the kernel-level call: the kernel multiplies a host
    float by up to two device scalars, so two tensor scales (or one tensor scale and a device
    alpha) cost no torch kernel; only a device alpha on top of two tensor scales is
    pre-multiplied."""
    devs = [t.reshape(1) for t in (opA.per_tensor_scale, opB.per_tensor_scale) if t is not None]
    if not devs:
        return alpha, None, 1.0
    if isinstance(alpha, Tensor):
        first = devs[0] * devs[1] if len(devs) == 2 else devs[0]
        return first, alpha.to(torch.float32).reshape(1), 1.0
    return devs[0], (devs[1] if len(devs) == 2 else None), float(alpha)


def _meta(t):
    return None if t is None else (t.dtype, t.shape, t.stride())


def _op_alpha(alpha, alpha_dev2, alpha_host) -> dict:
    """(alpha, second device factor, host factor) as the schema-typed keyword arguments of the custom ops."""
    if isinstance(alpha, Tensor):
        return dict(alpha=float(alpha_host), alpha_tensor=alpha, alpha_tensor2=alpha_dev2)
    return dict(alpha=float(alpha) * float(alpha_host))


def _op_norm(norm) -> dict:
    if norm is None:
        return {}
    return dict(sfd_norm_const_tensor=norm) if isinstance(norm, Tensor) else dict(sfd_norm_const=float(norm))


class _GemmPlan:
    """A validated launch: the filled C argument block of one (shapes, strides, dtypes, formats,
    config) combination with a host-float alpha.  Replaying copies the block (so concurrent threads
    never share one) and refreshes the pointers."""
    __slots__ = ("blob", "out_shape", "out_dtype")

    def __init__(self, args, out_shape, out_dtype):
        self.blob = bytes(args)
        self.out_shape, self.out_dtype = out_shape, out_dtype

    def replay(self, qa, qb, sfa, sfb, out, bias, alpha, pts_a, pts_b):
        from . import _lib, _ops

        args = _lib.GemmArgs.from_buffer_copy(self.blob)
        args.a, args.b, args.sfa, args.sfb, args.d = qa.data_ptr(), qb.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), out.data_ptr()
        if bias is not None:
            args.bias = bias.data_ptr()
        args.alpha = alpha
        if pts_a is not None:
            args.alpha_dev = pts_a.data_ptr()
            if pts_b is not None:
                args.alpha_dev2 = pts_b.data_ptr()
        elif pts_b is not None:
            args.alpha_dev = pts_b.data_ptr()
        _ops.launch_gemm_args(args, qa.device)


_PLANS: dict = {}


def _resolve_blockscaled_out(out_dtype) -> Optional[BlockScaledFormat]:
    if isinstance(out_dtype, BlockScaledFormat):
        return out_dtype
    if isinstance(out_dtype, str):
        return BlockScaledFormat.from_name(out_dtype)
    return None


def _reserve_blockscaled_out(out_dtype) -> None:
    if _resolve_blockscaled_out(out_dtype) is not None:
        raise NotImplementedError(f"blockscaled output (out_dtype={out_dtype}) is only supported by quack.gemm "
                                  "for now (and by gemm_act_quant in quack_b200)")


def _alloc_blockscaled_out(out_shape, fmt: BlockScaledFormat, device):
    """(codes, blocked scales) of a quantised (..., M, N) output, scale vectors along N
    (reference :272-300)."""
    vec = fmt.sf_vec_size
    *batch, m, n = out_shape
    if fmt.qdata_dtype == torch.float4_e2m1fn_x2:
        assert n % 32 == 0, f"fp4 output requires N % 32 == 0 (16 B rows), got N={n}"
        out = torch.empty(*batch, m, n // 2, dtype=torch.uint8, device=device).view(fmt.qdata_dtype)
    else:
        assert n % 16 == 0, f"fp8 output requires N % 16 == 0 (16 B rows), got N={n}"
        out = torch.empty(*batch, m, n, dtype=fmt.qdata_dtype, device=device)
    rm, rk = -(-m // 128), -(-n // (4 * vec))
    out_sf = torch.empty(*batch, rm, rk, 32, 4, 4, dtype=torch.uint8, device=device).view(fmt.scale_dtype)
    return out, out_sf


def _kernel_config(config: Optional[GemmConfig], tuned, m, n):
    """(tile_M, tile_N, cluster_M, dynamic scheduler) to request; zeros leave the choice to the
    library.  An explicit config with ``is_dynamic_persistent`` selects the cluster-launch-control
    scheduler (the reference's meaning of the flag on SM100, quack/gemm_config.py:215-225)."""
    if config is None:
        return 0, 0, 0, False
    tile_n, cg = config_to_kernel(config)
    return (256 if cg == 2 else 128), tile_n, (2 if cg == 2 else 1), bool(config.is_dynamic_persistent)


def _check_unsupported(**kw):
    for name, (value, default) in kw.items():
        bad = (value is not default) if default is None or isinstance(default, bool) else (value != default)
        if bad:
            raise NotImplementedError(f"quack_b200: {name} is not supported on the block-scaled B200 path")


def _bkn_to_nk(B: Tensor) -> Tensor:
    """B arrives as the logical (K, N) `.mT` view of a K-major (N, K) weight."""
    Bt = B.mT
    if Bt.stride(-1) != 1:
        raise NotImplementedError("B must be the .mT view of a K-major (N, K) weight (MN-major operands have no "
                                  "kernel in quack_b200)")
    return Bt


def gemm(
    A: Tensor | BlockScaledOperand,
    B: Tensor | BlockScaledOperand,
    out: Optional[Tensor | BlockScaledOperand] = None,
    bias: Optional[Tensor] = None,
    alpha: float | Tensor = 1.0,
    out_dtype: Optional[torch.dtype | BlockScaledFormat | str] = None,
    out_quant_dim: int = -1,
    out_transposed: bool = False,
    out_per_tensor_scale: Optional[float | Tensor] = None,
    cu_seqlens_m: Optional[Tensor] = None,
    cu_seqlens_k: Optional[Tensor] = None,
    A_idx: Optional[Tensor] = None,
    batch_idx_permute: Optional[Tensor] = None,
    dynamic_scheduler: bool = False,
    tuned: bool = True,
    rounding_mode: int = 0,
    sr_seed: int | Tensor = 0,
    concat_layout: tuple | None = None,
    split_k: Optional[int] = 1,
    split_k_mode: int = SplitKMode.SERIAL,
    config: Optional[GemmConfig] = None,
) -> Tensor | BlockScaledOperand:
    """``alpha * (A @ B) + bias`` with block-scaled A (M, K) and B (K, N).  ``out_dtype`` may
    name a block-scaled format: the epilogue then re-quantises and a ``BlockScaledOperand`` is
    returned."""
    # Replay of a validated call: the key holds everything the checks below read, so a hit
    # skips them (the per-call path of the reference's plan cache, quack/gemm_interface.py:1090-1153).
    if (type(A) is BlockScaledOperand and type(B) is BlockScaledOperand and out_dtype.__class__ is not str
            and cu_seqlens_m is None and cu_seqlens_k is None and A_idx is None and batch_idx_permute is None
            and not out_transposed and out_per_tensor_scale is None and rounding_mode == 0 and not concat_layout
            and split_k in (1, None) and (out is None or out.__class__ is Tensor) and not torch.compiler.is_compiling()):
        qa, qb, pa, pb = A.qdata, B.qdata, A.per_tensor_scale, B.per_tensor_scale
        fast_key = (qa.dtype, qa.shape, qa.stride(), qb.shape, qb.stride(), A.scale.shape, A.scale.stride(),
                    B.scale.shape, B.scale.stride(), A.format.name, B.format.name, A.quant_dim, B.quant_dim,
                    _meta(out), out_dtype, _meta(bias), alpha.__class__ is float, pa is None, pb is None, config, qa.device)
        plan = _PLANS.get(fast_key)
        if plan is not None:
            if out is None:
                out = torch.empty(plan.out_shape, dtype=plan.out_dtype, device=qa.device)
            plan.replay(qa, qb, A.scale, B.scale, out, bias, alpha, pa, pb)
            return out
    else:
        fast_key = None
    fmt_d = _resolve_blockscaled_out(out_dtype)
    if fmt_d is not None and out_transposed:
        assert out_quant_dim == -2, "out_transposed requires out_quant_dim=-2"
        assert bias is None, "out_transposed quantized output does not support bias yet"
        return gemm(B.mT, A.mT, out=out, alpha=alpha, out_dtype=out_dtype, out_quant_dim=-1,
                    out_per_tensor_scale=out_per_tensor_scale, dynamic_scheduler=dynamic_scheduler, tuned=tuned,
                    rounding_mode=rounding_mode, sr_seed=sr_seed, split_k=split_k, split_k_mode=split_k_mode)
    assert not out_transposed, "out_transposed requires a blockscaled out_dtype"
    opA, opB = _unpack_operand(A), _unpack_operand(B)
    SFA, SFB, fa, fb = _prep_blockscaled(opA, opB)
    _check_unsupported(cu_seqlens_m=(cu_seqlens_m, None), cu_seqlens_k=(cu_seqlens_k, None), A_idx=(A_idx, None),
                       batch_idx_permute=(batch_idx_permute, None), rounding_mode=(rounding_mode, 0),
                       concat_layout=(concat_layout or None, None))
    Ad, Bd = opA.data, opB.data
    user_alpha = alpha
    alpha, alpha_dev2, alpha_host = _fold_per_tensor_scales(alpha, opA, opB)
    plan_key = fast_key if (fmt_d is None and Ad.ndim == 2 and isinstance(user_alpha, float)) else None
    out_sf = None
    if fmt_d is not None:
        assert out_quant_dim in (-1, -2), f"out_quant_dim must be -1 or -2, got {out_quant_dim}"
        if out_quant_dim == -2:
            raise NotImplementedError("column-direction quantized output has no kernel in quack_b200; use "
                                      "out_transposed=True")
        if fmt_d.name not in _OUT_FORMATS:
            raise NotImplementedError(f"quantized output format {fmt_d.name} has no kernel in quack_b200")
        if isinstance(out, BlockScaledOperand):
            assert out.format == fmt_d, f"out container format {out.format.name} != out_dtype {fmt_d.name}"
            assert out.quant_dim == out_quant_dim, f"out container quant_dim {out.quant_dim} != out_quant_dim {out_quant_dim}"
            out_sf, out = out.scale, out.qdata
    else:
        assert out_per_tensor_scale is None, "out_per_tensor_scale requires a blockscaled out_dtype"
        assert not isinstance(out, BlockScaledOperand), "a BlockScaledOperand out requires a blockscaled out_dtype"
    out_shape = (Ad.shape[0], Bd.shape[-1]) if Ad.ndim == 2 else (Ad.shape[0], Ad.shape[-2], Bd.shape[-1])
    if out is None:
        if fmt_d is not None:
            out, out_sf = _alloc_blockscaled_out(out_shape, fmt_d, Ad.device)
        else:
            out = torch.empty(out_shape, dtype=torch.bfloat16 if out_dtype is None else out_dtype, device=Ad.device)
    pts = norm = None
    if fmt_d is not None:
        assert out_sf is not None, "quantized output requires out as a BlockScaledOperand (or out=None to allocate)"
        if out_per_tensor_scale is not None:
            assert fmt_d.has_per_tensor_scale, f"{fmt_d.name} does not take out_per_tensor_scale"
            if isinstance(out_per_tensor_scale, Tensor):
                pts = out_per_tensor_scale.float().reshape(1)
                norm = pts.reciprocal()
            else:
                pts = torch.full((1,), float(out_per_tensor_scale), dtype=torch.float32, device=out.device)
                norm = 1.0 / out_per_tensor_scale
        out_op = BlockScaledOperand(qdata=out, scale=out_sf, format=fmt_d, per_tensor_scale=pts, quant_dim=out_quant_dim)
    if out.numel() == 0:
        return out_op if fmt_d is not None else out
    if Ad.numel() == 0:
        assert fmt_d is None, "quantized output does not support K == 0"
        out.zero_()
        if bias is not None:
            out += bias
        return out
    assert tuple(out.shape[:-1]) == tuple(out_shape[:-1]), f"out shape {tuple(out.shape)} does not match {out_shape}"
    tm, tn, cm, dyn = _kernel_config(config, tuned, out_shape[-2], out_shape[-1])
    if _tops.compiling():
        # the torch.library boundary: schema-typed, flattened arguments (see quack_b200/_torch_ops.py)
        common = dict(bias=bias, dynamic_scheduler=dyn, tuned=tuned, SFA=_tops.encode(SFA), SFB=_tops.encode(SFB), bs_format_a=fa,
                      bs_format_b=fb, tile_m=tm, tile_n=tn, cluster_m=cm, **_op_alpha(alpha, alpha_dev2, alpha_host))
        if fmt_d is not None:
            _tops.ops.gemm_quant_out(_tops.encode(Ad), _tops.encode(Bd), _tops.encode(out), _tops.encode(out_sf), fmt_d.name, "n",
                                     **common, **_op_norm(norm))
            return out_op
        _tops.ops.gemm_out(_tops.encode(Ad), _tops.encode(Bd), out, split_k=split_k or 1, split_k_mode=int(split_k_mode), **common)
        return out
    args = _kernel.gemm(Ad, _bkn_to_nk(Bd), out, None, None, tm, tn, cm, 1, is_dynamic_persistent=dyn, rowvec_bias=bias, alpha=alpha, SFA=SFA,
                        SFB=SFB, split_k=split_k or 1, bs_format_a=fa, bs_format_b=fb, SFD=out_sf, sfd_norm_const=norm,
                        bs_format_d=None if fmt_d is None else fmt_d.name, alpha_dev2=alpha_dev2, alpha_host=alpha_host)
    if plan_key is not None and args is not None and (bias is None or bias.stride(-1) == 1):
        if len(_PLANS) > 4096:
            _PLANS.clear()
        _PLANS[plan_key] = _GemmPlan(args, tuple(out.shape), out.dtype)
    return out_op if fmt_d is not None else out


def gemm_add(
    A: Tensor | BlockScaledOperand,
    B: Tensor | BlockScaledOperand,
    C: Tensor,
    out: Optional[Tensor] = None,
    bias: Optional[Tensor] = None,
    alpha: float | Tensor = 1.0,
    beta: float | Tensor = 1.0,
    out_dtype: Optional[torch.dtype | BlockScaledFormat | str] = None,
    cu_seqlens_m: Optional[Tensor] = None,
    cu_seqlens_k: Optional[Tensor] = None,
    A_idx: Optional[Tensor] = None,
    batch_idx_permute: Optional[Tensor] = None,
    dynamic_scheduler: bool = False,
    tuned: bool = True,
    concat_layout: tuple | None = None,
    split_k: Optional[int] = 1,
    split_k_mode: int = SplitKMode.SERIAL,
    config: Optional[GemmConfig] = None,
) -> Tensor:
    """``D = alpha * A @ B + beta * C [+ bias]`` with block-scaled A and B: the residual and the bias are
    independent epilogue terms of one launch (reference quack/gemm_interface.py:1562-1683).  ``C`` is
    (M, N) or (L, M, N), bf16 / fp16 / fp32, row-major."""
    _reserve_blockscaled_out(out_dtype)
    opA, opB = _unpack_operand(A), _unpack_operand(B)
    SFA, SFB, fa, fb = _prep_blockscaled(opA, opB)
    _check_unsupported(cu_seqlens_m=(cu_seqlens_m, None), cu_seqlens_k=(cu_seqlens_k, None), A_idx=(A_idx, None),
                       batch_idx_permute=(batch_idx_permute, None), concat_layout=(concat_layout or None, None))
    Ad, Bd = opA.data, opB.data
    alpha, alpha_dev2, alpha_host = _fold_per_tensor_scales(alpha, opA, opB)
    out_shape = (*Ad.shape[:-1], Bd.shape[-1])
    assert tuple(C.shape) == tuple(out_shape), f"C shape {tuple(C.shape)} does not match the output {out_shape}"
    assert C.is_cuda and C.stride(-1) == 1, "C must be a row-major CUDA tensor"
    if out is None:
        out = torch.empty(out_shape, dtype=out_dtype if out_dtype is not None else torch.bfloat16, device=Ad.device)
    else:
        assert tuple(out.shape) == tuple(out_shape), f"out shape {tuple(out.shape)} does not match {out_shape}"
    tm, tn, cm, dyn = _kernel_config(config, tuned, out_shape[-2], out_shape[-1])
    if _tops.compiling():
        kw = dict(bias=bias, dynamic_scheduler=dyn, tuned=tuned, SFA=_tops.encode(SFA), SFB=_tops.encode(SFB), bs_format_a=fa,
                  bs_format_b=fb, split_k=split_k or 1, split_k_mode=int(split_k_mode), tile_m=tm, tile_n=tn, cluster_m=cm,
                  **_op_alpha(alpha, alpha_dev2, alpha_host))
        kw.update(dict(beta_tensor=beta) if isinstance(beta, Tensor) else dict(beta=float(beta)))
        if C is out:
            _tops.ops.gemm_add_inplace(_tops.encode(Ad), _tops.encode(Bd), out, **kw)
        else:
            _tops.ops.gemm_add_out(_tops.encode(Ad), _tops.encode(Bd), C, out, **kw)
        return out
    _kernel.gemm(Ad, _bkn_to_nk(Bd), out, C, None, tm, tn, cm, 1, is_dynamic_persistent=dyn, rowvec_bias=bias, alpha=alpha,
                 beta=beta, SFA=SFA, SFB=SFB, split_k=split_k or 1, bs_format_a=fa, bs_format_b=fb, alpha_dev2=alpha_dev2,
                 alpha_host=alpha_host)
    return out


def gemm_add_inplace(
    A: Tensor | BlockScaledOperand,
    B: Tensor | BlockScaledOperand,
    out: Tensor,
    bias: Optional[Tensor] = None,
    alpha: float | Tensor = 1.0,
    beta: float | Tensor = 1.0,
    **kwargs,
) -> None:
    """``out = alpha * A @ B + beta * out [+ bias]`` (reference :1934-1960): every element of ``out`` is read by
    the thread that later writes it, so the residual may alias the output."""
    gemm_add(A, B, out, out=out, bias=bias, alpha=alpha, beta=beta, **kwargs)


def gemm_act(
    A: Tensor | BlockScaledOperand,
    B: Tensor | BlockScaledOperand,
    C: Optional[Tensor] = None,
    bias: Optional[Tensor] = None,
    activation: Activation = None,
    alpha: float | Tensor = 1.0,
    preact_out: Optional[Tensor] = None,
    postact_out: Optional[Tensor] = None,
    out_dtype: Optional[torch.dtype] = None,
    postact_dtype: Optional[torch.dtype] = None,
    cu_seqlens_m: Optional[Tensor] = None,
    A_idx: Optional[Tensor] = None,
    store_preact: bool = True,
    dynamic_scheduler: bool = False,
    tuned: bool = True,
    config: Optional[GemmConfig] = None,
    concat_layout: tuple | None = None,
    split_k: Optional[int] = 1,
    split_k_mode: int = SplitKMode.SERIAL,
    exact_activation: Optional[bool] = None,
) -> Tuple[Optional[Tensor], Tensor]:
    """``postact = act(alpha * A @ B + bias)``; gated activations read (gate, up) from even /
    odd output columns and halve N.  Returns ``(preact | None, postact)``.

    ``exact_activation`` (not in the reference): sigmoid / SiLU by ``expf`` and IEEE division, bit-equal to
    torch's CUDA ``F.silu`` / ``torch.sigmoid``, instead of the fast ``ex2.approx`` form the reference's device
    code uses (quack/activation.py:54-69).  Default: fast (``QK_EXACT_ACT=1`` in the environment flips it)."""
    _reserve_blockscaled_out(out_dtype)
    _reserve_blockscaled_out(postact_dtype)
    if split_k not in (None, 1):
        raise NotImplementedError("gemm_act does not support split_k > 1; split_k is currently supported by gemm, "
                                  "gemm_add, and gemm_add_inplace.")
    opA, opB = _unpack_operand(A), _unpack_operand(B)
    SFA, SFB, fa, fb = _prep_blockscaled(opA, opB)
    _check_unsupported(cu_seqlens_m=(cu_seqlens_m, None), A_idx=(A_idx, None),
                       concat_layout=(concat_layout or None, None))
    if activation not in _KERNEL_ACTS:
        if activation in act_to_pytorch_fn_map or activation in gated_to_pytorch_fn_map:
            raise NotImplementedError(f"activation {activation!r} has no fused epilogue in quack_b200")
        raise ValueError(f"unknown activation {activation!r}")
    Ad, Bd = opA.data, opB.data
    alpha, alpha_dev2, alpha_host = _fold_per_tensor_scales(alpha, opA, opB)
    is_gated = activation in gated_to_pytorch_fn_map
    out_dtype = torch.bfloat16 if out_dtype is None else out_dtype
    postact_dtype = torch.bfloat16 if postact_dtype is None else postact_dtype
    out_shape = (Ad.shape[0], Bd.shape[-1]) if Ad.ndim == 2 else (Ad.shape[0], Ad.shape[-2], Bd.shape[-1])
    post_shape = (*out_shape[:-1], out_shape[-1] // 2) if is_gated else out_shape
    if preact_out is None and store_preact:
        preact_out = torch.empty(out_shape, dtype=out_dtype, device=Ad.device)
    if postact_out is None:
        postact_out = torch.empty(post_shape, dtype=postact_dtype, device=Ad.device)
    if postact_out.numel() == 0 or Ad.numel() == 0:
        if preact_out is not None:
            preact_out.zero_()
        postact_out.zero_()
        return preact_out, postact_out
    tm, tn, cm, dyn = _kernel_config(config, tuned, out_shape[-2], out_shape[-1])
    exact = _EXACT_ACT_DEFAULT if exact_activation is None else bool(exact_activation)
    if _tops.compiling() and activation is not None:
        kw = dict(C=C, bias=bias, activation=activation, dynamic_scheduler=dyn, tuned=tuned, SFA=_tops.encode(SFA),
                  SFB=_tops.encode(SFB), bs_format_a=fa, bs_format_b=fb, tile_m=tm, tile_n=tn, cluster_m=cm, exact_activation=exact,
                  **_op_alpha(alpha, alpha_dev2, alpha_host))
        if preact_out is None:
            _tops.ops.gemm_act_out_nopreact(_tops.encode(Ad), _tops.encode(Bd), postact_out, **kw)
        else:
            _tops.ops.gemm_act_out(_tops.encode(Ad), _tops.encode(Bd), preact_out, postact_out, **kw)
        return preact_out, postact_out
    if activation is None:
        # identity "activation": postact is a second copy of the pre-activation
        _kernel.gemm(Ad, _bkn_to_nk(Bd), postact_out, C, None, tm, tn, cm, 1, is_dynamic_persistent=dyn, rowvec_bias=bias, alpha=alpha, SFA=SFA,
                     SFB=SFB, bs_format_a=fa, bs_format_b=fb, alpha_dev2=alpha_dev2, alpha_host=alpha_host)
        if preact_out is not None:
            preact_out.copy_(postact_out)
        return preact_out, postact_out
    _kernel.gemm(Ad, _bkn_to_nk(Bd), preact_out, C, None, tm, tn, cm, 1, is_dynamic_persistent=dyn, rowvec_bias=bias, alpha=alpha, SFA=SFA,
                 SFB=SFB, bs_format_a=fa, bs_format_b=fb, activation=activation, postact_out=postact_out,
                 alpha_dev2=alpha_dev2, alpha_host=alpha_host, exact_activation=exact)
    return preact_out, postact_out


gemm_gated = gemm_act


def gemm_act_quant(
    A: BlockScaledOperand,
    B: BlockScaledOperand,
    bias: Optional[Tensor] = None,
    activation: Activation = "swiglu",
    alpha: float | Tensor = 1.0,
    postact_format: BlockScaledFormat | str = "nvfp4",
    postact_per_tensor_scale: Optional[float | Tensor] = None,
    postact_out: Optional[BlockScaledOperand] = None,
    config: Optional[GemmConfig] = None,
    exact_activation: bool = True,
    preact_out: Optional[Tensor] = None,
) -> BlockScaledOperand:
    """Fused up-projection of a quantised MLP: ``act(alpha * A @ B + bias)`` re-quantised in the
    epilogue (codes + blocked scales + optional NVFP4 tensor scale), ready to feed the down
    projection.  The reference expresses this with its epilogue-mod object
    (``swiglu_quant_mod.gemm``, quack/epilogue/library.py:204-234, which has no alpha / bias
    operands); here the whole chain alpha -> bias -> activation -> quantise is one call.

    ``exact_activation`` (default on): SiLU / sigmoid by ``expf`` and IEEE division, so that codes and scale
    bytes equal torch's ``F.silu(gate) * up`` followed by the reference's output-quantiser model
    (tests/test_gemm_quant_out.py:57-101) bit for bit; ``False`` selects the fast ``ex2.approx`` form of the
    reference's device code.  ``preact_out``: optional (M, N) bf16 / fp16 / fp32 tensor that receives the
    pre-activation ``alpha * A @ B + bias``."""
    opA, opB = _unpack_operand(A), _unpack_operand(B)
    SFA, SFB, fa, fb = _prep_blockscaled(opA, opB)
    fmt_d = _resolve_blockscaled_out(postact_format)
    if fmt_d is None or fmt_d.name not in _OUT_FORMATS:
        raise NotImplementedError(f"quantized postact format {postact_format!r} has no kernel in quack_b200")
    if activation not in _KERNEL_ACTS or activation is None:
        raise NotImplementedError(f"activation {activation!r} has no fused quantising epilogue in quack_b200")
    Ad, Bd = opA.data, opB.data
    assert Ad.ndim == 2, "gemm_act_quant takes 2-D operands"
    alpha, alpha_dev2, alpha_host = _fold_per_tensor_scales(alpha, opA, opB)
    is_gated = activation in gated_to_pytorch_fn_map
    m, n = Ad.shape[0], Bd.shape[-1]
    n_out = n // 2 if is_gated else n
    pts = norm = None
    if postact_per_tensor_scale is not None:
        assert fmt_d.has_per_tensor_scale, f"{fmt_d.name} does not take a per-tensor scale"
        if isinstance(postact_per_tensor_scale, Tensor):
            pts = postact_per_tensor_scale.float().reshape(1)
            norm = pts.reciprocal()
        else:
            pts = torch.full((1,), float(postact_per_tensor_scale), dtype=torch.float32, device=Ad.device)
            norm = 1.0 / postact_per_tensor_scale
    if postact_out is None:
        q, sf = _alloc_blockscaled_out((m, n_out), fmt_d, Ad.device)
    else:
        assert postact_out.format == fmt_d
        q, sf = postact_out.qdata, postact_out.scale
    tm, tn, cm, dyn = _kernel_config(config, True, m, n)
    if _tops.compiling() and preact_out is None:
        _tops.ops.gemm_act_quant_out(_tops.encode(Ad), _tops.encode(Bd), _tops.encode(q), _tops.encode(sf), fmt_d.name, bias=bias,
                                     activation=activation, dynamic_scheduler=dyn, SFA=_tops.encode(SFA), SFB=_tops.encode(SFB),
                                     bs_format_a=fa, bs_format_b=fb, tile_m=tm, tile_n=tn, cluster_m=cm,
                                     exact_activation=bool(exact_activation), **_op_alpha(alpha, alpha_dev2, alpha_host),
                                     **_op_norm(norm))
        return BlockScaledOperand(qdata=q, scale=sf, format=fmt_d, per_tensor_scale=pts, quant_dim=-1)
    _kernel.gemm(Ad, _bkn_to_nk(Bd), preact_out, None, None, tm, tn, cm, 1, is_dynamic_persistent=dyn, rowvec_bias=bias, alpha=alpha, SFA=SFA, SFB=SFB,
                 bs_format_a=fa, bs_format_b=fb, activation=activation, postact_out=q, SFD=sf, sfd_norm_const=norm,
                 bs_format_d=fmt_d.name, alpha_dev2=alpha_dev2, alpha_host=alpha_host, exact_activation=exact_activation)
    return BlockScaledOperand(qdata=q, scale=sf, format=fmt_d, per_tensor_scale=pts, quant_dim=-1)


# ---------------------------------------------------------------------------------------------
# torch references (any device): the parity yardsticks of the tests, not a kernel path
# ---------------------------------------------------------------------------------------------

def gemm_ref(A: Tensor, B: Tensor, out: Optional[Tensor] = None, bias: Optional[Tensor] = None,
             alpha: float | Tensor = 1.0, out_dtype: Optional[torch.dtype] = None, **unused) -> Tensor:
    out_dtype = A.dtype if out_dtype is None else out_dtype
    res = (torch.bmm if A.ndim == 3 else torch.mm)(A.float(), B.float())
    if not isinstance(alpha, float) or alpha != 1.0:
        res = res * alpha
    if bias is not None:
        res = res + (bias if A.ndim == 2 else bias.unsqueeze(1)).float()
    res = res.to(out_dtype)
    if out is not None:
        out.copy_(res)
        return out
    return res


def gemm_blockscaled_ref(A: BlockScaledOperand, B: BlockScaledOperand, alpha: float | Tensor = 1.0,
                         out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
    """Dequantise, fp32 matmul, x per-tensor scales, x alpha, cast (reference :1521-1559)."""
    from .blockscaled.quantize import dequant_operand, unpack_scale_blocked_to_2d

    opA, opB = _unpack_operand(A), _unpack_operand(B)
    assert opA.fmt is not None and opB.fmt is not None, "gemm_blockscaled_ref requires blockscaled A and B"
    mma_kind_for_pair(opA.fmt, opB.fmt)
    assert opA.fmt.sf_vec_size == opB.fmt.sf_vec_size
    vec = opA.fmt.sf_vec_size
    Ad, Bd = opA.data, opB.data
    batched = Ad.ndim == 3
    a3 = Ad if batched else Ad.unsqueeze(0)
    b3 = (Bd if batched else Bd.unsqueeze(0)).mT
    a_val, b_val = dequant_operand(a3, opA.fmt), dequant_operand(b3, opB.fmt)
    l, m, k = a_val.shape
    n = b_val.shape[1]
    SFA = opA.sf.unsqueeze(0) if opA.sf.ndim == 5 else opA.sf
    SFB = opB.sf.unsqueeze(0) if opB.sf.ndim == 5 else opB.sf
    sfa = unpack_scale_blocked_to_2d(SFA.contiguous(), m, k // vec).float()
    sfb = unpack_scale_blocked_to_2d(SFB.contiguous(), n, k // vec).float()
    out = torch.einsum("lmk,lnk->lmn", a_val * sfa.repeat_interleave(vec, dim=-1),
                       b_val * sfb.repeat_interleave(vec, dim=-1))
    for s in (opA.per_tensor_scale, opB.per_tensor_scale):
        if s is not None:
            out = out * s
    if not (isinstance(alpha, float) and alpha == 1.0):
        out = out * alpha
    out = out.to(out_dtype)
    return out if batched else out.squeeze(0)


def gemm_act_ref(A: Tensor, B: Tensor, C: Optional[Tensor] = None, bias: Optional[Tensor] = None,
                 activation: Activation = None, alpha: float | Tensor = 1.0, out_dtype: Optional[torch.dtype] = None,
                 postact_dtype: Optional[torch.dtype] = None, store_preact: bool = True, **unused):
    out_dtype = A.dtype if out_dtype is None else out_dtype
    postact_dtype = A.dtype if postact_dtype is None else postact_dtype
    pre = gemm_ref(A, B, bias=bias, alpha=alpha, out_dtype=torch.float32)
    if C is not None:
        pre = pre + C.float()
    if activation in gated_to_pytorch_fn_map:
        post = gated_to_pytorch_fn_map[activation](pre[..., ::2], pre[..., 1::2]).to(postact_dtype)
    else:
        post = act_to_pytorch_fn_map[activation](pre).to(postact_dtype)
    return (pre.to(out_dtype) if store_preact else None), post


gemm_gated_ref = gemm_act_ref


def gemm_add_ref(A: Tensor, B: Tensor, C: Tensor, bias: Optional[Tensor] = None, out: Optional[Tensor] = None,
                 alpha: float | Tensor = 1.0, beta: float | Tensor = 1.0, out_dtype: Optional[torch.dtype] = None,
                 **unused) -> Tensor:
    """fp32 yardstick of gemm_add on dequantised operands (reference :1748-1790)."""
    out_dtype = A.dtype if out_dtype is None else out_dtype
    res = gemm_ref(A, B, bias=bias, alpha=alpha, out_dtype=torch.float32) + beta * C.float()
    res = res.to(out_dtype)
    if out is not None:
        out.copy_(res)
        return out
    return res
