"""Kernel-level block-scaled GEMM call: validation + one launch through the C ABI.

Mirrors ``quack.gemm.gemm`` of the reference (quack/gemm.py:378-443) for the block-scaled
dense path and its ``AllGatherArguments`` (:360-375).  The reference builds a plan, JIT-compiles
a CuTe-DSL kernel and launches it through TVM-FFI; here the kernels are compiled ahead of time
and ``qk_gemm_blockscaled`` is called directly.  Features of the reference kernel that are not
on the quantised-linear path (dense bf16 GEMM, varlen, gather_A, column bias, stochastic
rounding, column-direction output scales, split-K modes other than SERIAL) raise
``NotImplementedError``.
"""

from __future__ import annotations

from typing import NamedTuple, Optional

import torch
from torch import Tensor

from . import _ops
from . import _lib
from ._lib import FMT_NONE
from .blockscaled.operand import BlockScaledFormat, mma_kind_for_pair
from .gemm_config import COMPILED_TILES, SplitKMode


class AllGatherArguments(NamedTuple):
    """Scheduler arguments of the all-gather GEMM: ``flags[shard * num_chunks + c] >= *epoch``
    (modular) releases the tiles of that chunk; tiles are visited shard by shard starting at
    ``first_shard`` (the rank's own, already resident shard)."""

    flags: Tensor       # (num_shards * num_chunks,) int32, device
    epoch: Tensor       # (1,) int32, device-resident epoch slot
    num_shards: int
    first_shard: int
    num_chunks: int = 1
    # in-kernel transport: a device tensor holding the table of peer addresses (qk_ag_pull_args); the GEMM then
    # fetches the remote shards itself and sets the flags
    pull: Optional[Tensor] = None


def validate_blockscaled_sf(A, B, SFA, SFB, *, fmt_a: BlockScaledFormat, fmt_b: BlockScaledFormat):
    """Layout / consistency checks of the scale factors against (l, m, k_storage) /
    (l, n, k_storage) operands (reference quack/gemm_tvm_ffi_utils.py:70-223, dense case).
    Returns the scale vector size."""
    assert SFB is not None and SFA is not None, "SFA and SFB must be provided together"
    assert fmt_a.scale_dtype == fmt_b.scale_dtype and fmt_a.sf_vec_size == fmt_b.sf_vec_size
    assert SFA.dtype == fmt_a.scale_dtype and SFB.dtype == fmt_b.scale_dtype, (
        f"SF dtype mismatch: {SFA.dtype} / {SFB.dtype} vs {fmt_a.name}/{fmt_b.name} scales "
        f"{fmt_a.scale_dtype}/{fmt_b.scale_dtype}")
    assert A.dtype == fmt_a.qdata_dtype, f"A dtype mismatch: {A.dtype} vs {fmt_a.name} qdata {fmt_a.qdata_dtype}"
    assert B.dtype == fmt_b.qdata_dtype, f"B dtype mismatch: {B.dtype} vs {fmt_b.name} qdata {fmt_b.qdata_dtype}"
    vec = fmt_a.sf_vec_size
    k_a, k_b = fmt_a.logical_k(A.shape[-1]), fmt_b.logical_k(B.shape[-1])
    assert k_a == k_b, (f"logical K mismatch: A storage K {A.shape[-1]} ({fmt_a.name}) => {k_a} vs B storage K "
                        f"{B.shape[-1]} ({fmt_b.name}) => {k_b}")
    rk = -(-k_a // (4 * vec))
    l = A.shape[0] if A.ndim == 3 else 1
    for name, SF, mn in (("SFA", SFA, A.shape[-2]), ("SFB", SFB, B.shape[-2])):
        core = (-(-mn // 128), rk, 32, 4, 4)
        if SF.ndim == 5:
            assert A.ndim == 2, f"{name}: unbatched 5-D scale factors require 2D operands, A is {A.ndim}D"
            expected = core
        else:
            expected = (l, *core)
        assert tuple(SF.shape) == expected, f"{name} shape {tuple(SF.shape)} != {expected}"
        assert tuple(SF.stride()[-3:]) == (16, 4, 1), (
            f"{name}: inner (32, 4, 4) block must be contiguous with strides (16, 4, 1), got {SF.stride()[-3:]}")
    return vec


def validate_ag_geometry(A, ag_args: AllGatherArguments, tile_M: int, cluster_M: int) -> None:
    """Shard and arrival-chunk boundaries must fall on whole scheduler clusters along M
    (reference quack/gemm_tvm_ffi_utils.py:452-468)."""
    m_rows = A.shape[-2]
    assert m_rows % ag_args.num_shards == 0, f"AG+GEMM: M ({m_rows}) must divide into num_shards ({ag_args.num_shards})"
    shard_rows = m_rows // ag_args.num_shards
    assert shard_rows % (tile_M * cluster_M * ag_args.num_chunks) == 0, (
        f"AG+GEMM: shard rows ({shard_rows}) must be a multiple of tile_M * cluster_M * arrival_chunks "
        f"({tile_M} * {cluster_M} * {ag_args.num_chunks}) so shard/chunk boundaries land on whole scheduler clusters")


def _unsupported(name: str):
    raise NotImplementedError(f"quack_b200.gemm: {name} is not part of the block-scaled B200 path")


def gemm(
    A: Tensor,                      # (l, m, k_storage) or (m, k_storage), K-major codes
    B: Tensor,                      # (l, n, k_storage) or (n, k_storage), K-major codes
    D: Optional[Tensor],            # (l, m, n) or (m, n); quantised codes when SFD is given
    C: Optional[Tensor] = None,
    tile_count_semaphore: Optional[Tensor] = None,
    tile_M: int = 0,
    tile_N: int = 0,
    cluster_M: int = 0,
    cluster_N: int = 1,
    cluster_K: int = 1,
    tile_K: Optional[int] = None,
    pingpong: bool = False,
    persistent: bool = True,
    is_dynamic_persistent: bool = False,
    max_swizzle_size: int = 8,
    rowvec_bias: Optional[Tensor] = None,   # (n,) or (l, n)
    colvec_bias: Optional[Tensor] = None,
    alpha: float | Tensor = 1.0,
    beta: float | Tensor = 1.0,
    cu_seqlens_m: Optional[Tensor] = None,
    cu_seqlens_k: Optional[Tensor] = None,
    A_idx: Optional[Tensor] = None,
    batch_idx_permute: Optional[Tensor] = None,
    add_to_output: bool = False,
    rounding_mode: int = 0,
    sr_seed: int | Tensor = 0,
    use_tma_gather: bool = False,
    concat_layout=None,
    num_warps: Optional[int] = None,
    SFA: Optional[Tensor] = None,
    SFB: Optional[Tensor] = None,
    bs_format_a: Optional[str] = None,
    bs_format_b: Optional[str] = None,
    split_k: int = 1,
    split_k_mode: int = SplitKMode.SERIAL,
    b_kn: bool = False,
    SFD: Optional[Tensor] = None,
    sfd_norm_const: Optional[float | Tensor] = None,
    SFDCol: Optional[Tensor] = None,
    ag_args: Optional[AllGatherArguments] = None,
    *,
    # epilogue operands of the activation variants (reference: quack/epilogue/library.py:527-576)
    activation: Optional[str] = None,
    postact_out: Optional[Tensor] = None,
    bs_format_d: Optional[str] = None,
    alpha_dev2: Optional[Tensor] = None,    # second device factor of alpha (two NVFP4 tensor scales need no torch multiply)
    alpha_host: float = 1.0,                # host factor applied on top of a tensor alpha
    timeout_ns: int = 0,
    max_ctas: int = 0,
    ag_arrival_order: bool = False,         # all-gather: take the shards in the order they land (QK_SCHED_ARRIVAL)
    exact_activation: bool = False,         # sigmoid / SiLU by expf + IEEE division (bit-equal to torch's CUDA kernels)
):
    """Block-scaled ``D = epilogue(alpha * A @ B^T + bias)`` on the current CUDA stream."""
    if SFA is None or SFB is None:
        assert SFA is None and SFB is None, "A and B must both (or neither) carry scale factors"
        _unsupported("a GEMM without scale factors (dense bf16/fp16)")
    assert bs_format_a is not None and bs_format_b is not None, "bs_format_a / bs_format_b are required with SFA / SFB"
    for cond, name in ((colvec_bias is not None, "a column bias"),
                       (cu_seqlens_m is not None or cu_seqlens_k is not None, "varlen"),
                       (A_idx is not None, "gather_A"), (batch_idx_permute is not None, "batch_idx_permute"),
                       (add_to_output, "add_to_output"), (rounding_mode != 0, "stochastic rounding"),
                       (bool(concat_layout), "concat_layout"),
                       (split_k not in (1, None) and split_k_mode != SplitKMode.SERIAL, "split_k modes other than SERIAL"),
                       (b_kn, "b_kn"), (SFDCol is not None, "column-direction output scales"),
                       (cluster_N not in (0, 1) or cluster_K != 1, "cluster_N / cluster_K > 1 (operand multicast)")):
        if cond:
            _unsupported(name)
    fmt_a, fmt_b = BlockScaledFormat.from_name(bs_format_a), BlockScaledFormat.from_name(bs_format_b)
    kind = mma_kind_for_pair(fmt_a, fmt_b)
    if fmt_a.name not in _ops._FMT_ID or fmt_b.name not in _ops._FMT_ID:
        raise NotImplementedError(
            f"quack_b200 has kernels for {sorted(_ops._FMT_ID)}; got {fmt_a.name} x {fmt_b.name} (MMA kind {kind})")
    if SFA.dtype == torch.uint8:
        SFA = SFA.view(fmt_a.scale_dtype)
    if SFB.dtype == torch.uint8:
        SFB = SFB.view(fmt_b.scale_dtype)
    assert A.ndim == B.ndim and A.ndim in (2, 3), "A and B must both be 2-D or both 3-D"
    assert A.stride(-1) == 1 and B.stride(-1) == 1, "A and B must be K-major (unit stride along K)"
    validate_blockscaled_sf(A, B, SFA, SFB, fmt_a=fmt_a, fmt_b=fmt_b)
    fmt = _ops.format_id(fmt_a.name)
    k = fmt_a.logical_k(A.shape[-1])
    m, n = A.shape[-2], B.shape[-2]

    # configuration: explicit (tile_M, tile_N, cluster_M) or the library's choice
    tile_n = tile_N or 0
    cg = 0
    if tile_M:
        assert tile_M in (128, 256), f"tile_M must be 128 or 256, got {tile_M}"
        cg = 2 if (tile_M == 256 and (cluster_M or 2) % 2 == 0) else 1
        if tile_M == 256 and cg == 1:
            raise ValueError("tile_M=256 needs an even cluster_M (the MMA tile spans a CTA pair)")
        if tile_n and (tile_n, cg) not in COMPILED_TILES:
            raise ValueError(f"no compiled kernel for tile_N={tile_n} with {cg} CTA(s) per MMA tile; "
                             f"available: {sorted(COMPILED_TILES)}")
    if ag_args is not None:
        assert A.ndim == 2, "AG+GEMM takes 2-D operands"
        # rows of one scheduler cluster in this kernel: a 256-row MMA tile spans the CTA pair (the reference counts
        # tile_M x cluster_M with per-CTA tiles); the library picks 256-row tiles for shards of at least 512 rows
        rows_per_cluster = tile_M or (256 if m // ag_args.num_shards >= 512 else 128)
        validate_ag_geometry(A, ag_args, rows_per_cluster, 1)

    out_format = FMT_NONE
    if SFD is not None:
        fmt_d = BlockScaledFormat.from_name(bs_format_d) if bs_format_d is not None else (
            BlockScaledFormat.from_name("mxfp8_e4m3") if SFD.dtype == torch.float8_e8m0fnu
            else BlockScaledFormat.from_name("nvfp4"))
        out_format = _ops.format_id(fmt_d.name)
        if SFD.dtype == torch.uint8:
            SFD = SFD.view(fmt_d.scale_dtype)
    norm_host, norm_dev = 1.0, None
    if sfd_norm_const is not None:
        if isinstance(sfd_norm_const, Tensor):
            norm_dev = sfd_norm_const.to(torch.float32).reshape(1)
        else:
            norm_host = float(sfd_norm_const)
    alpha_dev = None
    if isinstance(alpha, Tensor):
        alpha_dev = alpha if (alpha.dtype == torch.float32 and alpha.numel() == 1) else alpha.to(torch.float32).reshape(1)
        alpha_host = float(alpha_host)
    else:
        alpha_host = float(alpha) * float(alpha_host)
    beta_host, beta_dev = 1.0, None
    if C is not None:
        assert tuple(C.shape[-2:]) == (m, n), f"C must be (..., {m}, {n}), got {tuple(C.shape)}"
        if isinstance(beta, Tensor):
            beta_dev = beta if (beta.dtype == torch.float32 and beta.numel() == 1) else beta.to(torch.float32).reshape(1)
        else:
            beta_host = float(beta)

    batched = A.ndim == 3
    L = A.shape[0] if batched else 1
    last_args = None
    for li in range(L):
        a_i, b_i = (A[li], B[li]) if batched else (A, B)
        sfa_i = SFA[li] if SFA.ndim == 6 else SFA
        sfb_i = SFB[li] if SFB.ndim == 6 else SFB
        d_i = None if D is None else (D[li] if batched else D)
        p_i = None if postact_out is None else (postact_out[li] if batched else postact_out)
        bias_i = None
        if rowvec_bias is not None:
            bias_i = rowvec_bias[li] if rowvec_bias.ndim == 2 else rowvec_bias
        c_i = None if C is None else (C[li] if batched else C)
        sfd_i = None
        if SFD is not None:
            sfd_i = SFD[li] if SFD.ndim == 6 else SFD
            # pad slots of the blocked scale buffer are not covered by any tile: keep them defined
            n_out = n // 2 if (activation in _GATED and p_i is not None) else n
            if m % 128 or (n_out // _ops._FMT_VEC[out_format]) % 4:
                sfd_i.view(torch.uint8).zero_()
        # all code / scale tensors are 1-byte element types: pointers and strides are used as they are
        last_args = _ops.gemm_blockscaled(
            fmt, a_i, sfa_i, b_i, sfb_i, m, n, k, d=d_i, post=p_i, activation=activation, bias=bias_i, alpha=alpha_host,
            alpha_dev=alpha_dev, alpha_dev2=alpha_dev2 if alpha_dev is not None else None, out_format=out_format,
            sfd=sfd_i, norm_const=norm_host, norm_const_dev=norm_dev, ag=ag_args, tile_n=tile_n, cta_group=cg,
            max_ctas=max_ctas, timeout_ns=timeout_ns,
            # the reference's dynamic persistent scheduler is cluster launch control on SM100
            scheduler=(_lib.SCHED_ARRIVAL if (ag_args is not None and ag_arrival_order and ag_args.num_chunks == 1
                                              and ag_args.num_shards <= 32)
                       else _lib.SCHED_CLC if (is_dynamic_persistent and max_ctas == 0 and ag_args is None)
                       else _lib.SCHED_STATIC),
            # 1 (the reference's default) leaves the choice to the library: a split changes neither the
            # result's determinism nor the call; an explicit value > 1 is honoured or fails
            split_k=0 if split_k in (1, None) else int(split_k),
            c=c_i, beta=beta_host, beta_dev=beta_dev, exact_activation=exact_activation,
            fmt_b=_ops.format_id(fmt_b.name))
    return last_args


_GATED = ("swiglu", "reglu", "geglu", "glu")
