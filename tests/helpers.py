"""Shared builders for the GPU parity tests: seeded inputs -> oracle-quantised operands."""

import numpy as np
import torch

from oracle import blockscaled_oracle as orc


def oracle_quantize(x: torch.Tensor, fmt: str, pts=None):
    """-> (codes u8 ndarray, scales 2-D u8 ndarray, dequantised fp32 WITHOUT the tensor scale)."""
    if fmt == "mxfp8_e4m3":
        c, s = orc.to_mx_e4m3(x)
        return c, s, orc.dequant_mxfp8(c, s)
    if fmt == "mxfp8_e5m2":
        c, s = orc.to_mx_e5m2(x)
        return c, s, orc.dequant_mxfp8_e5m2(c, s)
    if fmt == "mxfp4":
        c, s = orc.to_mxfp4(x)
        return c, s, orc.dequant_mxfp4(c, s)
    c, s = orc.to_nvfp4(x, pts)
    return c, s, orc.dequant_nvfp4(c, s)


def dev(a, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def make_operand_pair(fmt: str, m: int, n: int, k: int, seed: int = 0, use_pts: bool = True, fmt_b: str = None):
    """Seeded (A, W) of the benchmark distributions, quantised by the ORACLE.  Returns a dict
    with raw bytes (numpy), dequantised values and per-tensor scales.  ``fmt_b``: format of W when it
    differs from A's."""
    a = orc.make_activation(m, k, seed)
    w = orc.make_weight(n, k, seed + 1)
    pa = pb = None
    if fmt == "nvfp4" and use_pts:
        pa = float(orc.nvfp4_per_tensor_scale(a.float().abs().max().item()))
        pb = float(orc.nvfp4_per_tensor_scale(w.float().abs().max().item()))
    ac, asf, adq = oracle_quantize(a, fmt, pa)
    bc, bsf, bdq = oracle_quantize(w, fmt_b or fmt, pb)
    return dict(a=a, w=w, ac=ac, asf=asf, adq=adq, bc=bc, bsf=bsf, bdq=bdq, pa=pa, pb=pb,
                asf_b=orc.pack_scale_blocked(asf), bsf_b=orc.pack_scale_blocked(bsf))


def containers(fmt: str, ops: dict, device="cuda"):
    """BlockScaledOperand pair (A (M,K), W (N,K)) from oracle bytes."""
    from quack_b200.blockscaled import BlockScaledFormat, BlockScaledOperand

    f = BlockScaledFormat.from_name(fmt)
    pa = None if ops["pa"] is None else torch.tensor([ops["pa"]], dtype=torch.float32, device=device)
    pb = None if ops["pb"] is None else torch.tensor([ops["pb"]], dtype=torch.float32, device=device)
    A = BlockScaledOperand.from_parts(dev(ops["ac"], device).view(f.qdata_dtype), dev(ops["asf_b"], device), f,
                                      per_tensor_scale=pa)
    W = BlockScaledOperand.from_parts(dev(ops["bc"], device).view(f.qdata_dtype), dev(ops["bsf_b"], device), f,
                                      per_tensor_scale=pb)
    return A, W


def identity_weight(fmt: str, n: int, k: int):
    """Exact identity as quantised bytes: code 1.0 on the diagonal, unit scales."""
    if fmt in ("mxfp8_e4m3", "mxfp8_e5m2"):
        bc = np.zeros((n, k), np.uint8)
        bc[np.arange(min(n, k)), np.arange(min(n, k))] = 0x38 if fmt == "mxfp8_e4m3" else 0x3C
        bsf = np.full((n, k // 32), 127, np.uint8)
        deq = orc.dequant_mxfp8 if fmt == "mxfp8_e4m3" else orc.dequant_mxfp8_e5m2
        assert np.array_equal(deq(bc, bsf), np.eye(n, k, dtype=np.float32))
    else:
        codes = np.zeros((n, k), np.uint8)
        codes[np.arange(min(n, k)), np.arange(min(n, k))] = 0x2
        bc = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
        if fmt == "mxfp4":
            bsf = np.full((n, k // 32), 127, np.uint8)
            assert np.array_equal(orc.dequant_mxfp4(bc, bsf), np.eye(n, k, dtype=np.float32))
        else:
            bsf = np.full((n, k // 16), 0x38, np.uint8)
            assert np.array_equal(orc.dequant_nvfp4(bc, bsf), np.eye(n, k, dtype=np.float32))
    return bc, bsf


def rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """max-normalised error, the reference's metric (tests/test_gemm_blockscaled_interface.py:88-89)."""
    return float(np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30))


# ---- torch (any device) statement of the reference's output-quantiser model --------------------------------
def torch_e2m1_codes(q: torch.Tensor) -> torch.Tensor:
    """fp32 values already clamped to [-6, 6] -> E2M1 codes (uint8, bit 3 = sign), round-half-to-even on the
    grid {0, .5, 1, 1.5, 2, 3, 4, 6}: the thresholds of oracle.f32_to_e2m1_rne_sat."""
    a = q.abs()
    code = torch.zeros_like(a, dtype=torch.uint8)
    for thr, strict, c in ((0.25, True, 1), (0.75, False, 2), (1.25, True, 3), (1.75, False, 4), (2.5, True, 5),
                           (3.5, False, 6), (5.0, True, 7)):
        code = torch.where((a > thr) if strict else (a >= thr), torch.full_like(code, c), code)
    sign = ((q.view(torch.int32) >> 28) & 0x8).to(torch.uint8)
    return code | sign


def torch_quant_out_nvfp4(x: torch.Tensor, norm: float):
    """The reference's quant_ref (tests/test_gemm_quant_out.py:57-101) for nvfp4 in torch ops on the tensor's
    device -> (packed codes uint8 (M, N/2), scale bytes uint8 (M, N/16))."""
    m, n = x.shape
    xb = x.reshape(m, n // 16, 16).float()
    amax = xb.abs().amax(-1)
    # IEEE divisions, as the CPU evaluation of the model performs them (the golden vectors come from it): on a
    # CUDA tensor torch turns "tensor / python_float" into a multiplication by the rounded reciprocal, which
    # differs in the last bit for some inputs, so the divisor is passed as a tensor
    scale = amax / torch.full_like(amax, 6.0) * norm
    sf = scale.clamp(max=448.0).to(torch.float8_e4m3fn)
    scale_q = sf.float()
    rcp = torch.where(scale_q > 0, torch.full_like(scale_q, norm) / scale_q,
                      torch.full_like(scale_q, torch.finfo(torch.float32).max))
    q = (xb * rcp.unsqueeze(-1)).clamp(-6.0, 6.0).reshape(m, n)
    codes = torch_e2m1_codes(q)
    return (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous(), sf.view(torch.uint8)
