"""The CPU oracle against golden vectors produced by the reference's own torch code
(tests/golden/make_golden.py) and against the reference's known-answer tests."""

import numpy as np
import torch

from oracle import blockscaled_oracle as orc


def _bf16(a_int16):
    return torch.from_numpy(a_int16.copy()).view(torch.bfloat16)


def test_to_mx_matches_reference(golden):
    x = _bf16(golden["mx_x_bf16"])
    codes, sc = orc.to_mx_e4m3(x)
    assert np.array_equal(sc, golden["mx_scale"])
    assert np.array_equal(codes, golden["mx_codes"])
    codes_f, sc_f = orc.to_mx_e4m3(x, scaling_mode="floor")
    assert np.array_equal(sc_f, golden["mx_scale_floor"])
    assert np.array_equal(codes_f, golden["mx_codes_floor"])


def test_to_mx_fp32_input_decades(golden):
    codes, sc = orc.to_mx_e4m3(golden["mx32_x"])
    assert np.array_equal(sc, golden["mx32_scale"])
    assert np.array_equal(codes, golden["mx32_codes"])
    # rceil never saturates (reference tests/test_blockscaled_quantize.py:15-26)
    deq = orc.e4m3_to_f32(codes)
    assert np.abs(deq).max() <= 448.0


def test_to_mx_edge_blocks(golden):
    codes, sc = orc.to_mx_e4m3(golden["mxedge_x"])
    assert np.array_equal(sc, golden["mxedge_scale"])
    # rows 2/3 hold NaN codes whose sign differs between CPU and GPU division; compare magnitude
    g = golden["mxedge_codes"]
    assert np.array_equal(codes & 0x7F, g & 0x7F)
    finite = [0, 1, 4, 5, 6, 7]
    assert np.array_equal(codes[finite], g[finite])
    b = sc.flatten().tolist()
    assert b[0] <= 1 and b[3] == 255 and b[2] == 255  # reference :39-53


def test_known_block_max_500():
    # reference tests/test_blockscaled_quantize.py:28-36
    v = np.full((1, 32), 1.0, dtype=np.float32)
    v[0, 0] = 500.0
    qf, sf = orc.to_mx_e4m3(v, scaling_mode="floor")
    qc, sc = orc.to_mx_e4m3(v, scaling_mode="rceil")
    assert orc.e8m0_to_f32(sf).item() == 1.0 and orc.e4m3_to_f32(qf).max() == 448.0
    assert orc.e8m0_to_f32(sc).item() == 2.0 and orc.e4m3_to_f32(qc).max() == 256.0


def test_to_nvfp4_matches_reference(golden):
    x = _bf16(golden["nv_x_bf16"])
    pk, sf = orc.to_nvfp4(x, golden["nv_pts"][0])
    assert np.array_equal(sf, golden["nv_sf"])
    assert np.array_equal(pk, golden["nv_codes"])
    pk0, sf0 = orc.to_nvfp4(x, None)
    assert np.array_equal(sf0, golden["nv_sf_nopts"])
    assert np.array_equal(pk0, golden["nv_codes_nopts"])
    amax = x.float().abs().max().item()
    assert orc.nvfp4_per_tensor_scale(amax) == golden["nv_pts"][0]


def test_e2m1_encoder_sweep(golden):
    codes = orc.f32_to_e2m1_rne_sat(golden["e2m1_sweep_x"])
    assert np.array_equal(codes, golden["e2m1_sweep_codes"])
    assert np.array_equal(np.array(orc.FP4_E2M1FN_VALUES, dtype=np.float32).view(np.uint32),
                          golden["e2m1_values"].view(np.uint32))


def test_scale_layout(golden):
    s = golden["sf2d"]
    b = orc.pack_scale_blocked(s)
    assert np.array_equal(b, golden["sf2d_blocked"][0])
    assert np.array_equal(b.reshape(-1), golden["sf2d_to_blocked_flat"])
    assert np.array_equal(orc.unpack_scale_blocked(b, *s.shape), s)
    flat = b.reshape(-1)
    rk = b.shape[1]
    for m in (0, 1, 17, 31, 33, 127, 128, 299):
        for k in (0, 1, 3, 4, 7, 9):
            assert flat[orc.sf_byte_offset(m, k, rk)] == s[m, k]
    assert np.array_equal(orc.pack_scale_blocked(golden["mx_scale"]), golden["mx_scale_blocked"][0])
    assert np.array_equal(orc.pack_scale_blocked(golden["nv_sf"]), golden["nv_sf_blocked"][0])


def test_dequantize_matches_reference(golden):
    d = orc.dequant_mxfp8(golden["mx_codes"], golden["mx_scale"])
    assert np.array_equal(d.view(np.uint32), golden["mx_dequant"].view(np.uint32))
    dn = orc.dequant_nvfp4(golden["nv_codes"], golden["nv_sf"], golden["nv_pts"][0])
    assert np.array_equal(dn.view(np.uint32), golden["nv_dequant"].view(np.uint32))


def test_e4m3_codec_roundtrip():
    b = np.arange(256, dtype=np.uint8)
    v = orc.e4m3_to_f32(b)
    ok = ~np.isnan(v)
    assert np.array_equal(orc.f32_to_e4m3_rne_satfinite(v[ok]), b[ok])
    t = torch.from_numpy(b.copy()).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(v[ok], t[ok])
    # ties: halfway between 16 (0x58) and 18 (0x59) -> even mantissa
    assert orc.f32_to_e4m3_rne_satfinite(np.array([17.0, 19.0, 1000.0, -1000.0], np.float32)).tolist() == [
        0x58, 0x5A, 0x7E, 0xFE]


def test_quant_out_ref_properties():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((64, 128)).astype(np.float32)
    for fmt, vec, dmax in (("mxfp8_e4m3", 32, 448.0), ("nvfp4", 16, 6.0)):
        codes, sf, scale_q = orc.quant_out_ref(x, fmt)
        assert sf.shape == (64, 128 // vec)
        if fmt == "mxfp8_e4m3":
            deq = orc.e4m3_to_f32(codes) * np.repeat(scale_q, vec, -1)
            assert np.all(np.abs(deq - x) <= np.repeat(scale_q, vec, -1) * 16.0 + 1e-6)
            # e8m0 rounds the exponent up: amax/scale_q <= 448
            amax = np.abs(x.reshape(64, -1, vec)).max(-1)
            assert np.all(amax / scale_q <= 448.0)
        else:
            deq = orc.unpack_fp4(codes) * np.repeat(scale_q, vec, -1)
            assert np.all(np.abs(deq - x) <= np.repeat(scale_q, vec, -1) * 1.01 + 1e-6)


def test_to_nvfp4_inf_nan_blocks(golden):
    """inf blocks saturate (scale 448, codes +-6); a NaN anywhere in a block makes the scale byte the E4M3
    NaN and every code of the block 4 (quack/blockscaled/quantize.py:415-442 evaluated by the reference)."""
    x = golden["nvedge_x"]
    pk, sf = orc.to_nvfp4(x, golden["nvedge_pts"][0])
    assert np.array_equal(sf, golden["nvedge_sf"]) and np.array_equal(pk, golden["nvedge_codes"])
    pk0, sf0 = orc.to_nvfp4(x, None)
    assert np.array_equal(sf0, golden["nvedge_sf_nopts"]) and np.array_equal(pk0, golden["nvedge_codes_nopts"])
    assert sf[0, 0] == 0x7F and (pk[0, :8] == 0x44).all() and sf[2, 0] == 0x7E


def test_quant_out_ref_matches_reference_model(golden):
    """The output quantiser against the reference's own torch model (tests/test_gemm_quant_out.py:57-101,
    run by tests/golden/make_golden.py): scale bytes, dequantised scales and quantised values, with and
    without a norm constant, over 10 decades, zero / subnormal / huge blocks, exact block maxima, E2M1 ties
    and inf blocks.  E8M0 blocks whose maximum is inf are left out: the model takes their exponent from
    frexp(inf), which is unspecified (0 here: byte 127); the oracle and the kernel saturate to 2^127 (byte
    254) like the hardware conversion the model stands for."""
    x = golden["qo_x"]
    for fmt, vec in (("mxfp8_e4m3", 32), ("nvfp4", 16), ("mxfp4", 32)):
        for i, norm in enumerate(golden["qo_norms"]):
            codes, sf, scale_q = orc.quant_out_ref(x, fmt, float(norm))
            q = orc.e4m3_to_f32(codes) if fmt == "mxfp8_e4m3" else orc.unpack_fp4(codes)
            keep = np.ones(sf.shape, bool)
            if fmt != "nvfp4":
                keep = ~np.isinf(np.abs(x.reshape(x.shape[0], -1, vec)).max(-1))
                assert (~keep).sum() == 2 and (sf[~keep] == 254).all()
            keep_el = np.repeat(keep, vec, -1)
            assert np.array_equal(sf[keep], golden[f"qo_{fmt}_{i}_sf"][keep]), (fmt, i)
            assert np.array_equal(scale_q[keep], golden[f"qo_{fmt}_{i}_scale"][keep]), (fmt, i)
            gq = golden[f"qo_{fmt}_{i}_q"]
            if fmt != "nvfp4" and norm > 2:
                # E8M0 blocks that round to the smallest scale, 2^-127: the model's factor norm / 2^-127 overflows
                # to inf (0 * inf = NaN, subnormal * inf = inf), the device contract caps it at FLT_MAX
                # (quack/blockscaled/quantize_utils.py:9-22).  The API never pairs an E8M0 output with a norm.
                tiny = sf == 0
                assert tiny.sum() == 9 and (q[np.repeat(tiny, vec, -1)] == 0).all()
                keep &= ~tiny
                keep_el &= ~np.repeat(tiny, vec, -1)
            assert np.array_equal(q[keep_el].view(np.uint32), gq[keep_el].view(np.uint32)), (fmt, i)


def test_quant_out_ref_nan_blocks(golden):
    """NaN blocks of the E4M3-scaled format: scale byte 0x7F, finite elements multiplied by FLT_MAX (the
    model's branch for a scale that is not positive).  The model's treatment of the NaN element itself (and
    its E8M0 byte, frexp(NaN)) is an artefact of the torch functions it happens to use and is not pinned."""
    x = golden["qonan_x"]
    codes, sf, _ = orc.quant_out_ref(x, "nvfp4", 1.0)
    assert np.array_equal(sf, golden["qonan_nvfp4_sf"]) and sf[0, 0] == 0x7F and sf[2, 2] == 0x7F
    finite = ~np.isnan(x)
    assert np.array_equal(orc.unpack_fp4(codes)[finite], golden["qonan_nvfp4_q"][finite])


def test_mx_e5m2_and_mxfp4_match_reference(golden):
    """to_mx(elem_dtype=float8_e5m2) under both scale rules and to_mxfp4 (quack/blockscaled/quantize.py:47-114,
    :285-316): bf16 input with outlier channels, fp32 input over 12 decades, and the edge blocks (zero,
    subnormal, inf, NaN, maxima above the format range).  NaN codes are compared without the sign (CPU and GPU
    division produce opposite NaN signs); NaN elements of MXFP4 have no defined code."""
    x = _bf16(golden["mx_x_bf16"])
    for mode, suffix in (("rceil", ""), ("floor", "_floor")):
        c, s = orc.to_mx_e5m2(x, scaling_mode=mode)
        assert np.array_equal(s, golden["mx5_scale" + suffix]) and np.array_equal(c, golden["mx5_codes" + suffix])
    c, s = orc.to_mxfp4(x)
    assert np.array_equal(s, golden["mx4_scale"]) and np.array_equal(c, golden["mx4_codes"])
    c, s = orc.to_mx_e5m2(golden["mx32_x"])
    assert np.array_equal(s, golden["mx32_5_scale"]) and np.array_equal(c, golden["mx32_5_codes"])
    c, s = orc.to_mxfp4(golden["mx32_x"])
    assert np.array_equal(s, golden["mx32_4_scale"]) and np.array_equal(c, golden["mx32_4_codes"])
    e = golden["mxedge_x"]
    c, s = orc.to_mx_e5m2(e)
    assert np.array_equal(s, golden["mxedge_5_scale"]) and np.array_equal(c & 0x7F, golden["mxedge_5_codes"] & 0x7F)
    c, s = orc.to_mx_e4m3(e, scaling_mode="floor")
    assert np.array_equal(s, golden["mxedge_scale_floor"]) and np.array_equal(c & 0x7F, golden["mxedge_codes_floor"] & 0x7F)
    c, s = orc.to_mxfp4(e)
    not_nan_row = [0, 1, 2, 4, 5, 6, 7]
    assert np.array_equal(s, golden["mxedge_4_scale"]) and np.array_equal(c[not_nan_row], golden["mxedge_4_codes"][not_nan_row])
    # decode tables against torch
    b = np.arange(256, dtype=np.uint8)
    t = torch.from_numpy(b.copy()).view(torch.float8_e5m2).float().numpy()
    v = orc.e5m2_to_f32(b)
    assert np.array_equal(v[~np.isnan(t)], t[~np.isnan(t)])


def test_to_mx_dim0_matches_reference(golden):
    """to_mx_dim0 (quack/blockscaled/quantize.py:117-162): scale blocks run down the columns; the same numbers
    as quantising the transposed matrix."""
    x = _bf16(golden["mx_x_bf16"])
    for mode, suffix in (("rceil", ""), ("floor", "_floor")):
        c, s = orc.to_mx_dim0(x, scaling_mode=mode)
        assert np.array_equal(c, golden["mxd0_codes" + suffix]) and np.array_equal(s, golden["mxd0_scale" + suffix])
