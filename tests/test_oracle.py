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
