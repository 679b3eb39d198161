"""Shared builders for the GPU parity tests: seeded inputs -> oracle-quantised operands."""

import numpy as np
import torch

from oracle import blockscaled_oracle as orc


def oracle_quantize(x: torch.Tensor, fmt: str, pts=None):
    """-> (codes u8 ndarray, scales 2-D u8 ndarray, dequantised fp32 WITHOUT the tensor scale)."""
    if fmt == "mxfp8_e4m3":
        c, s = orc.to_mx_e4m3(x)
        return c, s, orc.dequant_mxfp8(c, s)
    c, s = orc.to_nvfp4(x, pts)
    return c, s, orc.dequant_nvfp4(c, s)


def dev(a, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def make_operand_pair(fmt: str, m: int, n: int, k: int, seed: int = 0, use_pts: bool = True):
    """Seeded (A, W) of the benchmark distributions, quantised by the ORACLE.  Returns a dict
    with raw bytes (numpy), dequantised values and per-tensor scales."""
    a = orc.make_activation(m, k, seed)
    w = orc.make_weight(n, k, seed + 1)
    pa = pb = None
    if fmt == "nvfp4" and use_pts:
        pa = float(orc.nvfp4_per_tensor_scale(a.float().abs().max().item()))
        pb = float(orc.nvfp4_per_tensor_scale(w.float().abs().max().item()))
    ac, asf, adq = oracle_quantize(a, fmt, pa)
    bc, bsf, bdq = oracle_quantize(w, fmt, pb)
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
    if fmt == "mxfp8_e4m3":
        bc = np.zeros((n, k), np.uint8)
        bc[np.arange(min(n, k)), np.arange(min(n, k))] = 0x38
        bsf = np.full((n, k // 32), 127, np.uint8)
        assert np.array_equal(orc.dequant_mxfp8(bc, bsf), np.eye(n, k, dtype=np.float32))
    else:
        codes = np.zeros((n, k), np.uint8)
        codes[np.arange(min(n, k)), np.arange(min(n, k))] = 0x2
        bc = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
        bsf = np.full((n, k // 16), 0x38, np.uint8)
        assert np.array_equal(orc.dequant_nvfp4(bc, bsf), np.eye(n, k, dtype=np.float32))
    return bc, bsf


def rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """max-normalised error, the reference's metric (tests/test_gemm_blockscaled_interface.py:88-89)."""
    return float(np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30))
