"""Parity of the block-scaled GEMM at the sizes of the benchmark configurations, the exact-arithmetic SwiGLU
epilogue, and the operand formats beyond MXFP8-E4M3 / NVFP4.

Operands of the full-size cases are quantised on the GPU (the quantizer is pinned bit for bit against the
oracle in tests/test_quantize_gpu.py) and their bytes are copied back, so the CPU oracle dequantises exactly
what the kernel read; the oracle then checks row slabs of the result, and size-independent properties
(bit equality between schedules, between the fused epilogue and torch applied to the stored pre-activation)
cover the rest."""

import numpy as np
import pytest
import torch

from oracle import blockscaled_oracle as orc
from tests.helpers import (dev, identity_weight, make_operand_pair, oracle_quantize, rel_err, torch_quant_out_nvfp4)

pytestmark = pytest.mark.gpu

TOL_BF16 = 5e-3


def _gpu_operand(x_cpu, fmt, with_pts=True):
    """Quantise on the GPU -> (BlockScaledOperand, dequantised fp32 rows callable, per-tensor scale or None)."""
    from quack_b200.blockscaled import BlockScaledOperand, nvfp4_per_tensor_scale
    x = x_cpu.cuda()
    kw = {}
    if fmt == "nvfp4" and with_pts:
        kw["per_tensor_scale"] = nvfp4_per_tensor_scale(x.abs().amax())
    op = BlockScaledOperand.quantize(x, fmt, **kw)
    del x
    return op


def _dequant_rows(op, rows):
    """Oracle dequantisation (without the tensor scale) of the given row range of a GPU operand."""
    from quack_b200 import _ops
    fmt = op.format.name
    vec = op.format.sf_vec_size
    mn, kb = op.qdata.shape
    k = op.format.logical_k(kb)
    codes = op.qdata.view(torch.uint8)[rows].cpu().numpy()
    sf2d = _ops.scale_unpack(op.scale.view(torch.uint8), mn, k // vec)[rows].cpu().numpy()
    if fmt == "mxfp8_e4m3":
        return orc.dequant_mxfp8(codes, sf2d)
    if fmt == "nvfp4":
        return orc.dequant_nvfp4(codes, sf2d)
    raise ValueError(fmt)


@pytest.mark.parametrize("n,k", [(28672, 4096), (4096, 14336), (6144, 4096), (4096, 4096)])
def test_config2_llama_shapes_few_rows(n, k):
    """Llama-3-8B linear shapes in MXFP8 at M = 1, 16, 128 (few-rows variants, 256-wide single-CTA tiles,
    automatic split-K for K = 14336) and M = 1024 against the oracle's dequantise -> fp32 matmul."""
    from quack_b200.gemm_interface import gemm
    W = _gpu_operand(orc.make_weight(n, k, 1), "mxfp8_e4m3")
    wdq = _dequant_rows(W, slice(None))
    for m in (1, 16, 128, 1024):
        A = _gpu_operand(orc.make_activation(m, k, 10 + m), "mxfp8_e4m3")
        out = gemm(A, W.mT)
        torch.cuda.synchronize()
        ref = orc.gemm_blockscaled_ref(_dequant_rows(A, slice(None)), wdq)
        assert rel_err(out.float().cpu().numpy(), ref) < TOL_BF16, (m, n, k)
        out32 = gemm(A, W.mT, out_dtype=torch.float32)
        assert rel_err(out32.cpu().numpy(), ref) < 1e-5, (m, n, k)
    from quack_b200 import _ops
    _ops.check_status(torch.device("cuda", 0))


def test_swiglu_nvfp4_postact_exact_matches_torch():
    """SwiGLU -> NVFP4 with the exact-arithmetic epilogue: codes and scale bytes equal, bit for bit, torch's
    fp32 ``F.silu(gate) * up`` of the kernel's own stored fp32 pre-activation followed by the reference's
    output-quantiser model (tests/test_gemm_quant_out.py:57-101), computed on the GPU.  Every tile shape,
    ragged M, with the tensor scales, the bias and the output's tensor scale in play.  The pre-activation itself
    is checked against the CPU oracle."""
    from quack_b200 import _ops
    fmt = "nvfp4"
    for (m, n, k), (tile_n, cg) in (((256, 1024, 512), (256, 2)), ((200, 768, 512), (128, 1)), ((384, 1024, 256), (192, 2)),
                                    ((1024, 4096, 1024), (0, 0)), ((130, 512, 256), (64, 1)), ((512, 512, 512), (256, 1))):
        ops = make_operand_pair(fmt, m, n, k, seed=21)
        bias = orc.make_bias(n)
        alpha = ops["pa"] * ops["pb"]
        pre_ref = orc.gemm_blockscaled_ref(ops["adq"], ops["bdq"], alpha=alpha, bias=bias)
        pts_out = float(np.abs(orc.gemm_act_ref(pre_ref, "swiglu")).max() / (6.0 * 448.0))
        no = n // 2
        pre = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        P = torch.zeros(m, no // 2, dtype=torch.uint8, device="cuda")
        SFD = torch.zeros(-(-m // 128), -(-(no // 16) // 4), 32, 4, 4, dtype=torch.uint8, device="cuda")
        st = torch.zeros(4, dtype=torch.int32, device="cuda")
        _ops.gemm_blockscaled(_ops.format_id(fmt), dev(ops["ac"]), dev(ops["asf_b"]), dev(ops["bc"]), dev(ops["bsf_b"]), m, n, k,
                              d=pre, post=P, activation="swiglu", bias=bias.cuda(), alpha=alpha, out_format=_ops.format_id("nvfp4"),
                              sfd=SFD, norm_const=1.0 / pts_out, exact_activation=True, tile_n=tile_n, cta_group=cg, status=st)
        torch.cuda.synchronize()
        assert st.tolist()[0] == 0
        assert rel_err(pre.cpu().numpy(), pre_ref) < 1e-5
        post = torch.nn.functional.silu(pre[:, 0::2]) * pre[:, 1::2]
        rc, rsf = torch_quant_out_nvfp4(post, 1.0 / pts_out)
        sf2d = _ops.scale_unpack(SFD, m, no // 16)
        assert torch.equal(sf2d, rsf), ("scale bytes", m, n, k, tile_n, cg)
        assert torch.equal(P, rc), ("codes", m, n, k, tile_n, cg)
        # without the stored pre-activation the quantised output is the same
        P2, SFD2 = torch.zeros_like(P), torch.zeros_like(SFD)
        _ops.gemm_blockscaled(_ops.format_id(fmt), dev(ops["ac"]), dev(ops["asf_b"]), dev(ops["bc"]), dev(ops["bsf_b"]), m, n, k,
                              post=P2, activation="swiglu", bias=bias.cuda(), alpha=alpha, out_format=_ops.format_id("nvfp4"),
                              sfd=SFD2, norm_const=1.0 / pts_out, exact_activation=True, tile_n=tile_n, cta_group=cg, status=st)
        assert torch.equal(P2, P) and torch.equal(SFD2, SFD)


@pytest.mark.parametrize("act", ["silu", "swiglu", "glu"])
def test_exact_activation_matches_torch_bitwise(act):
    """fp32 outputs of the exact mode: silu / swiglu / glu of the stored pre-activation, as torch computes
    them on the GPU, bit for bit; the fast mode stays within 2e-6 of it (relative to the largest value)."""
    from quack_b200 import _ops
    fmt, m, n, k = "mxfp8_e4m3", 300, 512, 256
    ops = make_operand_pair(fmt, m, n, k, seed=5)
    bias = orc.make_bias(n)
    gated = act != "silu"
    outs = {}
    for exact in (True, False):
        pre = torch.empty(m, n, dtype=torch.float32, device="cuda")
        post = torch.empty(m, n // 2 if gated else n, dtype=torch.float32, device="cuda")
        st = torch.zeros(4, dtype=torch.int32, device="cuda")
        _ops.gemm_blockscaled(_ops.format_id(fmt), dev(ops["ac"]), dev(ops["asf_b"]), dev(ops["bc"]), dev(ops["bsf_b"]), m, n, k,
                              d=pre, post=post, activation=act, bias=bias.cuda(), alpha=2.5, exact_activation=exact, status=st)
        torch.cuda.synchronize()
        assert st.tolist()[0] == 0
        outs[exact] = (pre, post)
    pre, post = outs[True]
    if act == "silu":
        ref = torch.nn.functional.silu(pre)
    elif act == "swiglu":
        ref = torch.nn.functional.silu(pre[:, 0::2]) * pre[:, 1::2]
    else:
        ref = torch.sigmoid(pre[:, 0::2]) * pre[:, 1::2]
    assert torch.equal(post, ref)
    assert torch.equal(outs[False][0], pre)
    assert (outs[False][1] - ref).abs().max() <= 2e-6 * ref.abs().max()


def test_config3_full_size_fused_up_projection():
    """Configuration 3 at full size: NVFP4 A (16384, 4096) x W (28672, 4096, gate / up interleaved) -> bias ->
    SwiGLU -> NVFP4 (16384, 14336) codes + scale bytes with an output tensor scale.
    (a) codes and scale bytes are bit-equal to torch's silu * up of the stored fp32 pre-activation followed by
    the reference's quantiser model, over the whole output; (b) row slabs of the pre-activation match the CPU
    oracle; (c) the call without the stored pre-activation gives the same bytes."""
    from quack_b200 import _ops
    from quack_b200.gemm_interface import gemm_act_quant
    m, k, n = 16384, 4096, 28672
    A = _gpu_operand(orc.make_activation(m, k, 0), "nvfp4")
    W = _gpu_operand(orc.make_weight(n, k, 1), "nvfp4")
    bias = orc.make_bias(n).cuda()
    pts_out = torch.tensor([2.0e-3], device="cuda")          # about amax(post) / (6 * 448) for these inputs
    pre = torch.empty(m, n, dtype=torch.float32, device="cuda")
    h = gemm_act_quant(A, W.mT, bias=bias, activation="swiglu", postact_format="nvfp4", postact_per_tensor_scale=pts_out,
                       preact_out=pre)
    torch.cuda.synchronize()
    _ops.check_status(torch.device("cuda", 0))
    norm = float((1.0 / pts_out).item())
    no = n // 2
    sf2d = _ops.scale_unpack(h.scale.view(torch.uint8), m, no // 16)
    codes = h.qdata.view(torch.uint8)
    step = 2048
    for r0 in range(0, m, step):                               # in slabs: the torch model makes fp32 temporaries
        p = pre[r0:r0 + step]
        post = torch.nn.functional.silu(p[:, 0::2]) * p[:, 1::2]
        rc, rsf = torch_quant_out_nvfp4(post, norm)
        assert torch.equal(sf2d[r0:r0 + step], rsf), ("scale bytes", r0)
        assert torch.equal(codes[r0:r0 + step], rc), ("codes", r0)
    assert int((codes != 0).sum()) > 0.5 * codes.numel()       # the output tensor scale did not flush the result
    # (b) oracle on row slabs
    wdq = _dequant_rows(W, slice(None))
    alpha = float(A.per_tensor_scale.item()) * float(W.per_tensor_scale.item())
    for rows in (slice(0, 128), slice(8192 - 64, 8192 + 64), slice(m - 128, m)):
        ref = orc.gemm_blockscaled_ref(_dequant_rows(A, rows), wdq, alpha=alpha, bias=bias.cpu())
        assert rel_err(pre[rows].cpu().numpy(), ref) < 1e-5, rows
    del pre, wdq
    # (c)
    h2 = gemm_act_quant(A, W.mT, bias=bias, activation="swiglu", postact_format="nvfp4", postact_per_tensor_scale=pts_out)
    assert torch.equal(h2.qdata.view(torch.uint8), codes) and torch.equal(h2.scale.view(torch.uint8), h.scale.view(torch.uint8))


def test_config1_full_size_matches_oracle_slabs():
    """Configuration 1 (NVFP4 8192^3 + fp32 bias -> bf16): row slabs against the CPU oracle."""
    from quack_b200 import _ops
    from quack_b200.gemm_interface import gemm
    m = n = k = 8192
    A = _gpu_operand(orc.make_activation(m, k, 0), "nvfp4")
    W = _gpu_operand(orc.make_weight(n, k, 1), "nvfp4")
    bias = orc.make_bias(n).cuda()
    out = gemm(A, W.mT, bias=bias)
    out32 = gemm(A, W.mT, bias=bias, out_dtype=torch.float32)
    torch.cuda.synchronize()
    _ops.check_status(torch.device("cuda", 0))
    wdq = _dequant_rows(W, slice(None))
    alpha = float(A.per_tensor_scale.item()) * float(W.per_tensor_scale.item())
    for rows in (slice(0, 256), slice(4000, 4256), slice(m - 256, m)):
        ref = orc.gemm_blockscaled_ref(_dequant_rows(A, rows), wdq, alpha=alpha, bias=bias.cpu())
        assert rel_err(out[rows].float().cpu().numpy(), ref) < TOL_BF16
        assert rel_err(out32[rows].cpu().numpy(), ref) < 1e-5


def test_config4_rank_block_at_8_way_geometry():
    """The per-rank problem of the all-gather GEMM at 8 GPUs on one GPU: A (32768, 8192) MXFP8 in 8 shards of
    4096 rows, the rank's weight block (3584, 8192), every shard's flag already published.  The gated kernel
    (static and arrival-order schedules, two different first shards) is bit-equal to the dense kernel, and row
    slabs from three shards match the CPU oracle."""
    from quack_b200 import _lib, _ops
    from quack_b200.gemm import AllGatherArguments
    from quack_b200.gemm import gemm as kernel_gemm
    m, n, k, shards = 32768, 3584, 8192, 8
    A = _gpu_operand(orc.make_activation(m, k, 1000), "mxfp8_e4m3")
    W = _gpu_operand(orc.make_weight(n, k, 1234), "mxfp8_e4m3")
    dense = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    kernel_gemm(A.qdata, W.qdata, dense, SFA=A.scale, SFB=W.scale, bs_format_a="mxfp8_e4m3", bs_format_b="mxfp8_e4m3")
    flags = torch.full((shards,), 5, dtype=torch.int32, device="cuda")
    epoch = torch.full((1,), 5, dtype=torch.int32, device="cuda")
    for first in (0, 5):
        for arrival in (False, True):
            D = torch.zeros_like(dense)
            kernel_gemm(A.qdata, W.qdata, D, SFA=A.scale, SFB=W.scale, bs_format_a="mxfp8_e4m3", bs_format_b="mxfp8_e4m3",
                        ag_args=AllGatherArguments(flags, epoch, shards, first, 1), ag_arrival_order=arrival)
            assert torch.equal(D, dense), (first, arrival)
    torch.cuda.synchronize()
    _ops.check_status(torch.device("cuda", 0))
    wdq = _dequant_rows(W, slice(None))
    for rows in (slice(0, 128), slice(4096 * 3 - 64, 4096 * 3 + 64), slice(m - 128, m)):
        ref = orc.gemm_blockscaled_ref(_dequant_rows(A, rows), wdq)
        assert rel_err(dense[rows].float().cpu().numpy(), ref) < TOL_BF16


# ---- operand formats beyond MXFP8-E4M3 and NVFP4 -----------------------------------------------------------

PAIRS = [("mxfp8_e5m2", "mxfp8_e5m2"), ("mxfp8_e4m3", "mxfp8_e5m2"), ("mxfp8_e5m2", "mxfp8_e4m3"), ("mxfp4", "mxfp4")]


@pytest.mark.parametrize("fa,fb", PAIRS)
@pytest.mark.parametrize("tile_n,cg", [(64, 1), (128, 1), (256, 1), (128, 2), (192, 2), (256, 2)])
def test_other_format_pairs_match_oracle(fa, fb, tile_n, cg):
    """E5M2 and mixed E4M3 / E5M2 pairs (kind::mxf8f6f4) and MXFP4 x MXFP4 (kind::mxf4nvf4, one E8M0 scale per
    32): the pairs of quack/blockscaled/operand.py:418-483, against the oracle at the bf16 and fp32 bars."""
    from quack_b200 import _ops
    for (m, n, k) in [(128, 128, 256), (384, 640, 1280), (200, 448, 384), (1, 128, 64), (129, 448, 96)]:
        if fa == "mxfp4" and k % 64:
            continue
        ops = make_operand_pair(fa, m, n, k, seed=3, fmt_b=fb)
        bias = orc.make_bias(n)
        ref = orc.gemm_blockscaled_ref(ops["adq"], ops["bdq"], alpha=1.5, bias=bias)
        for odt, tol in ((torch.bfloat16, TOL_BF16), (torch.float32, 1e-5)):
            D = torch.full((m, n), float("nan"), dtype=odt, device="cuda")
            st = torch.zeros(4, dtype=torch.int32, device="cuda")
            _ops.gemm_blockscaled(_ops.format_id(fa), dev(ops["ac"]), dev(ops["asf_b"]), dev(ops["bc"]), dev(ops["bsf_b"]), m, n, k,
                                  d=D, bias=bias.cuda(), alpha=1.5, tile_n=tile_n, cta_group=cg, fmt_b=_ops.format_id(fb), status=st,
                                  timeout_ns=500_000_000)
            torch.cuda.synchronize()
            assert st.tolist()[0] == 0
            assert rel_err(D.float().cpu().numpy(), ref) < tol, (fa, fb, m, n, k, odt)


def test_other_format_pairs_through_the_public_api():
    """Containers of every supported format through quack_b200.gemm_interface.gemm; illegal pairs are refused
    with the reference's wording."""
    from quack_b200.blockscaled import BlockScaledOperand
    from quack_b200.gemm_interface import gemm, gemm_blockscaled_ref
    m, n, k = 256, 384, 512
    a, w = orc.make_activation(m, k, 2).cuda(), orc.make_weight(n, k, 3).cuda()
    for fa, fb in PAIRS:
        A, W = BlockScaledOperand.quantize(a, fa), BlockScaledOperand.quantize(w, fb)
        out = gemm(A, W.mT)
        ref = gemm_blockscaled_ref(A, W.mT, out_dtype=torch.float32)
        assert rel_err(out.float().cpu().numpy(), ref.cpu().numpy()) < TOL_BF16, (fa, fb)
    A4, W8 = BlockScaledOperand.quantize(a, "mxfp4"), BlockScaledOperand.quantize(w, "mxfp8_e4m3")
    A16 = BlockScaledOperand.quantize(a, "nvfp4")
    with pytest.raises(ValueError, match="cannot pair"):       # no MMA kind mixes E4M3 and E8M0 scales
        gemm(A16, W8.mT)
    with pytest.raises(NotImplementedError, match="MMA kind"):  # legal on the hardware (kind::mxf8f6f4), no kernel here
        gemm(A4, W8.mT)


@pytest.mark.parametrize("fmt", ["mxfp8_e4m3", "nvfp4", "mxfp4"])
def test_mxfp4_quantised_output_bit_exact(fmt):
    """B = identity: D == dequant(A) exactly, so the MXFP4 output quantiser (E2M1 codes + E8M0 scale per 32,
    exponent rounded up) must reproduce the oracle's bytes (tests/test_gemm_quant_out.py:104-126 with
    fmt = mxfp4), for every operand kind and tile shape; plus reglu -> MXFP4."""
    from quack_b200 import _ops
    for tile_n, cg in ((256, 2), (192, 2), (128, 1), (64, 1)):
        for (m, n) in [(256, 256), (200, 384), (128, 448)]:
            k = n
            a = orc.make_activation(m, k, 3)
            ac, asf, adq = oracle_quantize(a, fmt)
            bc, bsf = identity_weight(fmt, n, k)
            ref = adq + np.float32(0)
            rc, rsf, _ = orc.quant_out_ref(ref, "mxfp4", 1.0)
            D = torch.zeros(m, n // 2, dtype=torch.uint8, device="cuda")
            SFD = torch.zeros(-(-m // 128), -(-(n // 32) // 4), 32, 4, 4, dtype=torch.uint8, device="cuda")
            st = torch.zeros(4, dtype=torch.int32, device="cuda")
            _ops.gemm_blockscaled(_ops.format_id(fmt), dev(ac), dev(orc.pack_scale_blocked(asf)), dev(bc),
                                  dev(orc.pack_scale_blocked(bsf)), m, n, k, d=D, out_format=_ops.format_id("mxfp4"), sfd=SFD,
                                  tile_n=tile_n, cta_group=cg, status=st)
            torch.cuda.synchronize()
            assert st.tolist()[0] == 0
            assert np.array_equal(SFD.cpu().numpy(), orc.pack_scale_blocked(rsf)), ("scale bytes", fmt, tile_n, cg, m, n)
            assert np.array_equal(D.cpu().numpy(), rc), ("codes", fmt, tile_n, cg, m, n)
    m, n = 256, 512
    a = orc.make_activation(m, n, 5)
    ac, asf, adq = oracle_quantize(a, fmt)
    bc, bsf = identity_weight(fmt, n, n)
    rc, rsf, _ = orc.quant_out_ref(orc.gemm_act_ref(adq + np.float32(0), "reglu"), "mxfp4", 1.0)
    P = torch.zeros(m, n // 4, dtype=torch.uint8, device="cuda")
    SFD = torch.zeros(m // 128, n // 2 // 32 // 4, 32, 4, 4, dtype=torch.uint8, device="cuda")
    st = torch.zeros(4, dtype=torch.int32, device="cuda")
    _ops.gemm_blockscaled(_ops.format_id(fmt), dev(ac), dev(orc.pack_scale_blocked(asf)), dev(bc), dev(orc.pack_scale_blocked(bsf)),
                          m, n, n, post=P, activation="reglu", out_format=_ops.format_id("mxfp4"), sfd=SFD, status=st)
    torch.cuda.synchronize()
    assert np.array_equal(SFD.cpu().numpy(), orc.pack_scale_blocked(rsf)) and np.array_equal(P.cpu().numpy(), rc)


def test_quantised_output_nan_and_inf_blocks():
    """An inf in the accumulator saturates its block (E4M3 scale 448 / E8M0 scale 2^127), a NaN makes the
    block's scale byte the format's NaN (0x7F / 0xFF) as torch's clamp-and-convert does for E4M3; finite
    elements of such a block are multiplied by FLT_MAX, the model's factor for a scale that is not positive."""
    from quack_b200 import _ops
    fmt, m, n = "mxfp8_e4m3", 128, 128
    a = orc.make_activation(m, n, 3)
    ac, asf, adq = oracle_quantize(a, fmt)
    bc, bsf = identity_weight(fmt, n, n)
    # a bias that injects the special values: columns 5 (NaN) and 40 (+inf)
    bias = torch.zeros(n)
    bias[5] = float("nan")
    bias[40] = float("inf")
    ref = adq + bias.numpy()[None, :]
    for ofmt, vec in (("nvfp4", 16), ("mxfp8_e4m3", 32), ("mxfp4", 32)):
        fp4 = ofmt != "mxfp8_e4m3"
        D = torch.zeros(m, n // 2 if fp4 else n, dtype=torch.uint8, device="cuda")
        SFD = torch.zeros(1, -(-(n // vec) // 4), 32, 4, 4, dtype=torch.uint8, device="cuda")
        st = torch.zeros(4, dtype=torch.int32, device="cuda")
        _ops.gemm_blockscaled(_ops.format_id(fmt), dev(ac), dev(orc.pack_scale_blocked(asf)), dev(bc), dev(orc.pack_scale_blocked(bsf)),
                              m, n, n, d=D, bias=bias.cuda(), out_format=_ops.format_id(ofmt), sfd=SFD, status=st)
        torch.cuda.synchronize()
        sf2 = orc.unpack_scale_blocked(SFD.cpu().numpy(), m, n // vec)
        rc, rsf, _ = orc.quant_out_ref(ref, ofmt, 1.0)
        nan_blk, inf_blk = 5 // vec, 40 // vec
        assert (sf2[:, nan_blk] == (0x7F if ofmt == "nvfp4" else 0xFF)).all()
        assert (sf2[:, inf_blk] == (0x7E if ofmt == "nvfp4" else 254)).all()
        ok_blocks = [b for b in range(n // vec) if b != nan_blk]
        assert np.array_equal(sf2[:, ok_blocks], rsf[:, ok_blocks])
        got = orc.unpack_fp4(D.cpu().numpy()) if fp4 else orc.e4m3_to_f32(D.cpu().numpy())
        want = orc.unpack_fp4(rc) if fp4 else orc.e4m3_to_f32(rc)
        cols = np.array([c for c in range(n) if c // vec != nan_blk])
        assert np.array_equal(got[:, cols], want[:, cols])
        if ofmt == "nvfp4":     # the NaN block of the E4M3-scaled format follows the model too (finite elements)
            cols = np.array([c for c in range(nan_blk * vec, nan_blk * vec + vec) if c != 5])
            assert np.array_equal(got[:, cols], want[:, cols])
