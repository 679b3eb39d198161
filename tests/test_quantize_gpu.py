"""CUDA quantizer (through the C ABI) against the CPU oracle and the reference's golden
vectors: codes and scale bytes must be bit exact."""

import numpy as np
import pytest
import torch

from oracle import blockscaled_oracle as orc

pytestmark = pytest.mark.gpu


def _q(x, fmt, pts=None, mode=0):
    from quack_b200 import _ops
    codes, sf = _ops.quantize_rows(x.cuda(), _ops.format_id(fmt), None if pts is None else pts.cuda(), mode)
    torch.cuda.synchronize()
    return codes.cpu().numpy(), sf.cpu().numpy()


def _bf16(a):
    return torch.from_numpy(a.copy()).view(torch.bfloat16)


def test_golden_mxfp8(golden):
    codes, sf = _q(_bf16(golden["mx_x_bf16"]), "mxfp8_e4m3")
    assert np.array_equal(codes, golden["mx_codes"])
    assert np.array_equal(sf, golden["mx_scale_blocked"][0])
    codes, sf = _q(torch.from_numpy(golden["mx32_x"].copy()), "mxfp8_e4m3")
    assert np.array_equal(codes, golden["mx32_codes"])
    assert np.array_equal(sf, orc.pack_scale_blocked(golden["mx32_scale"]))


def test_golden_nvfp4(golden):
    x = _bf16(golden["nv_x_bf16"])
    codes, sf = _q(x, "nvfp4", torch.from_numpy(golden["nv_pts"].copy()))
    assert np.array_equal(codes, golden["nv_codes"])
    assert np.array_equal(sf, golden["nv_sf_blocked"][0])
    codes, sf = _q(x, "nvfp4")
    assert np.array_equal(codes, golden["nv_codes_nopts"])
    assert np.array_equal(sf, orc.pack_scale_blocked(golden["nv_sf_nopts"]))


def test_edge_blocks(golden):
    """zero / denormal / inf / NaN / block max 500 (reference tests/test_blockscaled_quantize.py:28-53)."""
    codes, sf = _q(torch.from_numpy(golden["mxedge_x"].copy()), "mxfp8_e4m3")
    s2 = orc.unpack_scale_blocked(sf, 8, 1)
    assert np.array_equal(s2, golden["mxedge_scale"])
    g = golden["mxedge_codes"]
    assert np.array_equal(codes & 0x7F, g & 0x7F)           # NaN codes: sign is not defined
    finite = [0, 1, 4, 5, 6, 7]
    assert np.array_equal(codes[finite], g[finite])
    assert s2[4, 0] == 128 and orc.e4m3_to_f32(codes[4]).max() == 256.0   # 500 -> scale 2, code 256


def test_golden_nvfp4_inf_nan_blocks(golden):
    """inf blocks saturate; a NaN anywhere in a block gives the E4M3 NaN scale byte and code 4 for every
    element, as the reference's torch arithmetic does (quack/blockscaled/quantize.py:415-442, :165-207)."""
    x = torch.from_numpy(golden["nvedge_x"].copy())
    for pts, ck, sk in ((torch.from_numpy(golden["nvedge_pts"].copy()), "nvedge_codes", "nvedge_sf"),
                        (None, "nvedge_codes_nopts", "nvedge_sf_nopts")):
        codes, sf = _q(x, "nvfp4", pts)
        assert np.array_equal(orc.unpack_scale_blocked(sf, 6, 2), golden[sk])
        assert np.array_equal(codes, golden[ck])


def test_golden_mxfp8_e5m2_mxfp4_and_floor(golden):
    """The other MX element types and the floor scale rule against the reference's own outputs
    (to_mx(elem_dtype=float8_e5m2), to_mxfp4, scaling_mode="floor")."""
    from quack_b200 import _lib
    xb = _bf16(golden["mx_x_bf16"])
    x32 = torch.from_numpy(golden["mx32_x"].copy())
    e = torch.from_numpy(golden["mxedge_x"].copy())
    def chk(x, fmt, mode, ck, sk, mask=0xFF, rows=None):
        codes, sf = _q(x, fmt, None, mode)
        s2 = orc.unpack_scale_blocked(sf, x.shape[0], x.shape[1] // 32)
        assert np.array_equal(s2, golden[sk]), (fmt, mode, sk)
        sel = slice(None) if rows is None else rows
        assert np.array_equal(codes[sel] & mask, golden[ck][sel] & mask), (fmt, mode, ck)
    chk(xb, "mxfp8_e4m3", _lib.SCALING_FLOOR, "mx_codes_floor", "mx_scale_floor")
    chk(xb, "mxfp8_e4m3", _lib.SCALING_RCEIL, "mx_codes", "mx_scale")
    chk(xb, "mxfp8_e5m2", _lib.SCALING_DEFAULT, "mx5_codes", "mx5_scale")
    chk(xb, "mxfp8_e5m2", _lib.SCALING_FLOOR, "mx5_codes_floor", "mx5_scale_floor")
    chk(xb, "mxfp4", _lib.SCALING_DEFAULT, "mx4_codes", "mx4_scale")
    chk(x32, "mxfp8_e5m2", 0, "mx32_5_codes", "mx32_5_scale")
    chk(x32, "mxfp4", 0, "mx32_4_codes", "mx32_4_scale")
    # edge blocks: NaN codes compared without the sign; NaN elements of MXFP4 (row 3) have no defined code
    chk(e, "mxfp8_e5m2", 0, "mxedge_5_codes", "mxedge_5_scale", mask=0x7F)
    chk(e, "mxfp8_e4m3", _lib.SCALING_FLOOR, "mxedge_codes_floor", "mxedge_scale_floor", mask=0x7F)
    chk(e, "mxfp4", 0, "mxedge_4_codes", "mxedge_4_scale", rows=[0, 1, 2, 4, 5, 6, 7])
    with pytest.raises(NotImplementedError):
        _q(xb, "mxfp4", None, _lib.SCALING_RCEIL)
    with pytest.raises(ValueError):
        _q(xb, "nvfp4", None, _lib.SCALING_FLOOR)


@pytest.mark.parametrize("fmt", ["mxfp8_e5m2", "mxfp4"])
def test_other_mx_formats_ragged_and_container(fmt):
    from quack_b200.blockscaled import BlockScaledOperand, to_mx, to_mx_e5m2, to_mxfp4
    ref = orc.to_mx_e5m2 if fmt == "mxfp8_e5m2" else orc.to_mxfp4
    for rows, k in ((1, 32), (127, 128), (129, 4096), (300, 14336)):
        x = orc.make_activation(rows, k, seed=rows + k)
        codes, sf = _q(x, fmt)
        rc, rs = ref(x)
        assert np.array_equal(codes, rc) and np.array_equal(sf, orc.pack_scale_blocked(rs)), (rows, k)
    x = orc.make_activation(256, 512, 1).cuda()
    op = BlockScaledOperand.quantize(x, fmt)
    assert op.qdata.dtype == (torch.float8_e5m2 if fmt == "mxfp8_e5m2" else torch.float4_e2m1fn_x2)
    assert op.scale.dtype == torch.float8_e8m0fnu and op.shape == x.shape
    bound = 0.2 if fmt == "mxfp8_e5m2" else 0.6
    assert (op.dequantize(torch.float32) - x.float()).abs().max() / x.float().abs().max() < bound
    q, s = (to_mx_e5m2(x) if fmt == "mxfp8_e5m2" else to_mxfp4(x))
    rc, rs = ref(x.cpu())
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), rc) and np.array_equal(s.view(torch.uint8).cpu().numpy(), rs)
    if fmt == "mxfp8_e5m2":
        qf, sf = to_mx(x, 32, "floor", torch.float8_e5m2)
        rcf, rsf = orc.to_mx_e5m2(x.cpu(), scaling_mode="floor")
        assert np.array_equal(qf.view(torch.uint8).cpu().numpy(), rcf) and np.array_equal(sf.view(torch.uint8).cpu().numpy(), rsf)


@pytest.mark.parametrize("fmt", ["mxfp8_e4m3", "nvfp4"])
@pytest.mark.parametrize("rows", [1, 127, 128, 129])
@pytest.mark.parametrize("k", [32, 128, 4096, 14336])
def test_ragged_shapes(fmt, rows, k):
    x = orc.make_activation(rows, k, seed=rows + k)
    if k > 64:
        x[0, :64] = 0      # zero blocks (not the whole tensor: the NVFP4 tensor scale would be 0)
    pts = None
    if fmt == "nvfp4":
        pts = torch.tensor([float(orc.nvfp4_per_tensor_scale(x.float().abs().max().item()))])
    codes, sf = _q(x, fmt, pts)
    if fmt == "mxfp8_e4m3":
        rc, rs = orc.to_mx_e4m3(x)
    else:
        rc, rs = orc.to_nvfp4(x, pts.item())
    assert np.array_equal(codes, rc)
    assert np.array_equal(sf, orc.pack_scale_blocked(rs))   # includes the zero-filled pad slots


@pytest.mark.parametrize("fmt", ["mxfp8_e4m3", "nvfp4"])
def test_config0_operands(fmt):
    """A (2048, 4096) with outlier channels and W (4096, 4096) ~ N(0, 0.02) of configuration 0."""
    for x in (orc.make_activation(2048, 4096, 0), orc.make_weight(4096, 4096, 1)):
        pts = None
        if fmt == "nvfp4":
            pts = torch.tensor([float(orc.nvfp4_per_tensor_scale(x.float().abs().max().item()))])
        codes, sf = _q(x, fmt, pts)
        rc, rs = orc.to_mx_e4m3(x) if fmt == "mxfp8_e4m3" else orc.to_nvfp4(x, pts.item())
        assert np.array_equal(codes, rc) and np.array_equal(sf, orc.pack_scale_blocked(rs))


def test_fp32_input_and_special_values():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(96, 512, generator=g) * torch.logspace(-8, 8, 96).unsqueeze(1)
    x[3, 5] = -0.0
    x[4, :32] = torch.tensor([448.0 * 2.0 ** i for i in range(-16, 16)])
    codes, sf = _q(x, "mxfp8_e4m3")
    rc, rs = orc.to_mx_e4m3(x)
    assert np.array_equal(codes, rc) and np.array_equal(sf, orc.pack_scale_blocked(rs))
    y = torch.randn(64, 256, generator=g)
    y[2, :16] = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0])
    codes, sf = _q(y, "nvfp4")
    rc, rs = orc.to_nvfp4(y, None)
    assert np.array_equal(codes, rc) and np.array_equal(sf, orc.pack_scale_blocked(rs))


def test_amax_and_scale_layout():
    from quack_b200 import _ops
    x = orc.make_activation(300, 1024, 5)
    assert _ops.amax(x.cuda()).item() == x.float().abs().max().item()
    for mn, sfk in [(1, 4), (128, 4), (384, 12), (512, 16), (300, 10)]:
        s = torch.randint(0, 255, (mn, sfk), dtype=torch.uint8)
        b = _ops.scale_pack(s.cuda())
        assert np.array_equal(b.cpu().numpy(), orc.pack_scale_blocked(s.numpy()))
        flat = b.cpu().numpy().reshape(-1)
        rk = b.shape[1]
        for m in sorted({0, 1, 17, 31, 33, 127, min(128, mn - 1), mn - 1} & set(range(mn))):
            for kk in sorted({0, 1, 3, 4, 7, sfk - 1} & set(range(sfk))):
                assert flat[orc.sf_byte_offset(m, kk, rk)] == s[m, kk]
        assert torch.equal(_ops.scale_unpack(b, mn, sfk).cpu(), s)


def test_container_quantize_api():
    """BlockScaledOperand.quantize: metadata, batched input, dim=-2, round trip bounds
    (reference tests/test_blockscaled_operand.py:129-140, :663-682)."""
    from quack_b200.blockscaled import BlockScaledOperand, nvfp4_per_tensor_scale, to_mx, to_nvfp4
    x = orc.make_activation(256, 512, 1).cuda()
    op = BlockScaledOperand.quantize(x, "mxfp8_e4m3")
    assert op.shape == x.shape and op.dtype == x.dtype and op.device == x.device and op.quant_dim == -1
    assert op.qdata.dtype == torch.float8_e4m3fn and op.scale.dtype == torch.float8_e8m0fnu
    assert (op.dequantize(torch.float32) - x.float()).abs().max() / x.float().abs().max() < 0.1
    xb = torch.stack([x, x * 2.0, x * 0.5])
    ob = BlockScaledOperand.quantize(xb, "mxfp8")
    assert ob.qdata.shape == (3, 256, 512) and ob.scale.shape == (3, 2, 4, 32, 4, 4)
    assert torch.equal(ob.qdata[0].view(torch.uint8), op.qdata.view(torch.uint8))
    assert torch.equal(ob.scale[0].view(torch.uint8), op.scale.view(torch.uint8))
    xr = torch.stack([x[:100], x[100:200]])                  # rows not a multiple of 128: per-batch launches
    orr = BlockScaledOperand.quantize(xr, "mxfp8_e4m3")
    assert torch.equal(orr.qdata[1].view(torch.uint8), BlockScaledOperand.quantize(x[100:200].contiguous(), "mxfp8").qdata.view(torch.uint8))
    t = BlockScaledOperand.quantize(x, "mxfp8_e4m3", dim=-2)
    ref = BlockScaledOperand.quantize(x.mT.contiguous(), "mxfp8_e4m3")
    assert t.quant_dim == -2 and t.shape == x.shape
    assert torch.equal(t.qdata.mT.contiguous().view(torch.uint8), ref.qdata.view(torch.uint8))
    pts = nvfp4_per_tensor_scale(x.abs().amax())
    o4 = BlockScaledOperand.quantize(x, "nvfp4", per_tensor_scale=pts)
    assert o4.per_tensor_scale.shape == (1,) and o4.qdata.dtype == torch.float4_e2m1fn_x2
    assert (o4.dequantize(torch.float32) - x.float()).abs().max() / x.float().abs().max() < 0.6
    # functional forms return 2-D scales like the reference's to_mx / to_nvfp4
    q, s = to_mx(x)
    rc, rs = orc.to_mx_e4m3(x.cpu())
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), rc) and np.array_equal(s.view(torch.uint8).cpu().numpy(), rs)
    q4, s4, p4 = to_nvfp4(x, 16, pts)
    rc4, rs4 = orc.to_nvfp4(x.cpu(), pts.item())
    assert np.array_equal(q4.cpu().numpy(), rc4) and np.array_equal(s4.view(torch.uint8).cpu().numpy(), rs4)


@pytest.mark.parametrize("fmt", ["mxfp8_e4m3", "mxfp8_e5m2", "mxfp4", "nvfp4"])
def test_dim0_quantizer_equals_row_quantizer_of_the_transpose(fmt):
    """qk_quantize_blockscaled_dim0: codes of the transposed matrix and its blocked scales in one pass, bit-equal
    to the oracle applied to the transposed input; ragged column counts, bf16 and fp32 inputs, NVFP4 with its
    tensor scale; and through the container (quantize(dim=-2)) and the functional forms."""
    from quack_b200 import _lib, _ops
    from quack_b200.blockscaled import BlockScaledOperand, blockscaled_quantize_dim0, to_mx_dim0
    ref = {"mxfp8_e4m3": orc.to_mx_e4m3, "mxfp8_e5m2": orc.to_mx_e5m2, "mxfp4": orc.to_mxfp4}.get(fmt)
    for (r, c), dt in (((128, 128), torch.bfloat16), ((256, 200), torch.bfloat16), ((96, 1000), torch.float32),
                       ((4096, 264), torch.bfloat16), ((32, 8), torch.float32)):
        x = orc.make_activation(r, c, seed=r + c).to(dt)
        if r >= 64:
            x[:32, 0] = 0
        pts = None
        if fmt == "nvfp4":
            pts = torch.tensor([float(orc.nvfp4_per_tensor_scale(x.float().abs().max().item()))])
            rc, rs = orc.to_nvfp4(x.T.contiguous(), pts.item())
        else:
            rc, rs = ref(x.T.contiguous())
        codes, sf = _ops.quantize_cols(x.cuda(), _ops.format_id(fmt), None if pts is None else pts.cuda())
        torch.cuda.synchronize()
        assert np.array_equal(codes.cpu().numpy(), rc), (fmt, r, c)
        assert np.array_equal(sf.cpu().numpy(), orc.pack_scale_blocked(rs)), (fmt, r, c)
    x = orc.make_activation(256, 384, 3).cuda()
    kw = dict(per_tensor_scale=torch.tensor([0.01], device="cuda")) if fmt == "nvfp4" else {}
    t = BlockScaledOperand.quantize(x, fmt, dim=-2, **kw)
    via_copy = BlockScaledOperand.quantize(x.mT.contiguous(), fmt, **kw)
    assert t.quant_dim == -2 and t.shape == x.shape
    assert torch.equal(t.qdata.mT.contiguous().view(torch.uint8), via_copy.qdata.view(torch.uint8))
    assert torch.equal(t.scale.view(torch.uint8), via_copy.scale.view(torch.uint8))
    if fmt == "mxfp8_e4m3":
        q, s = to_mx_dim0(x)
        rc, rs = orc.to_mx_dim0(x.cpu())
        assert np.array_equal(q.view(torch.uint8).cpu().numpy(), rc) and np.array_equal(s.view(torch.uint8).cpu().numpy(), rs)
        qf, sf_ = to_mx_dim0(x, 32, "floor")
        rcf, rsf = orc.to_mx_dim0(x.cpu(), scaling_mode="floor")
        assert np.array_equal(qf.view(torch.uint8).cpu().numpy(), rcf) and np.array_equal(sf_.view(torch.uint8).cpu().numpy(), rsf)
        q2, sfb = blockscaled_quantize_dim0(x)
        assert torch.equal(q2.view(torch.uint8), q.view(torch.uint8))
        assert np.array_equal(sfb.view(torch.uint8).cpu().numpy(), orc.pack_scale_blocked(np.ascontiguousarray(rs.T)))
        # the quantised (K, N) weight feeds the GEMM as B directly
        from quack_b200.gemm_interface import gemm, gemm_blockscaled_ref
        A = BlockScaledOperand.quantize(orc.make_activation(128, 256, 9).cuda(), fmt)
        B = BlockScaledOperand.quantize(x, fmt, dim=-2)            # x is (K = 256, N = 384)
        out = gemm(A, B)
        refo = gemm_blockscaled_ref(A, B, out_dtype=torch.float32)
        assert float((out.float() - refo).abs().max() / refo.abs().max()) < 5e-3
