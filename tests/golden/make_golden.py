"""Generate golden vectors from the reference's own pure-PyTorch quantizers.

Run once in a container that has the reference checked out (it is not needed at test
time):  ``python tests/golden/make_golden.py <path-to-reference>``.

The reference package's ``__init__`` imports its GPU kernel stack, which is not importable
without its JIT toolchain, so the two torch-only modules are imported through empty
namespace packages.  TORCHDYNAMO_DISABLE keeps ``BlockScaledOperand.quantize`` on the
eager functions (the reference's tests assert eager == compiled bit for bit).
"""

import os
import sys
import types

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")

import numpy as np
import torch


def import_reference(root):
    for name, sub in (("quack", "quack"), ("quack.blockscaled", "quack/blockscaled")):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(root, sub)]
        sys.modules[name] = mod
    import quack.blockscaled.quantize as q
    import quack.blockscaled.operand as o
    return q, o


def u8(t):
    return t.contiguous().view(torch.uint8).numpy().copy()


def extract_quant_ref(root, operand_module):
    """The reference's torch model of the fused output quantiser, ``quant_ref`` of
    tests/test_gemm_quant_out.py:57-101, without importing that module (its top-level
    ``import quack`` needs the GPU JIT stack): the function and the two helpers it uses are
    compiled from their own source text into a namespace that holds torch and the
    reference's ``BlockScaledFormat``."""
    import ast

    path = os.path.join(root, "tests", "test_gemm_quant_out.py")
    tree = ast.parse(open(path).read(), path)
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in ("quant_ref", "fmt_props"):
            keep.append(node)
        elif isinstance(node, ast.Assign) and any(getattr(t, "id", None) == "DTYPE_MAX" for t in node.targets):
            keep.append(node)
    assert len(keep) == 3, [getattr(n, "name", "DTYPE_MAX") for n in keep]
    ns = {"torch": torch, "BlockScaledFormat": operand_module.BlockScaledFormat}
    exec(compile(ast.Module(body=keep, type_ignores=[]), path, "exec"), ns)
    return ns["quant_ref"]


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QUACK_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py <checkout of Dao-AILab/quack>   (or QUACK_REFERENCE_ROOT)")
    q, o = import_reference(root)
    here = os.path.dirname(os.path.abspath(__file__))
    out = {}

    # ---- MXFP8: seeded activation with outlier channels, many magnitudes, edge rows -----
    g = torch.Generator().manual_seed(0)
    x = torch.randn(160, 256, generator=g).to(torch.bfloat16)
    x[:, torch.randperm(256, generator=g)[:2]] *= 20
    x[5] *= 1e-3
    x[6] *= 1e3
    x[7, :32] = 0
    x[8, 32:64] = -0.0
    codes, sc = q.to_mx(x, 32)
    out["mx_x_bf16"] = x.view(torch.int16).numpy().copy()
    out["mx_codes"] = u8(codes)
    out["mx_scale"] = u8(sc)
    out["mx_scale_blocked"] = u8(q.pack_scale_2d_to_blocked_contig(sc))
    codes_f, sc_f = q.to_mx(x, 32, scaling_mode="floor")
    out["mx_codes_floor"] = u8(codes_f)
    out["mx_scale_floor"] = u8(sc_f)

    # the other MX element types on the same input: E5M2 codes (both scale rules), packed E2M1 codes (MXFP4, floor)
    c5, s5 = q.to_mx(x, 32, elem_dtype=torch.float8_e5m2)
    out["mx5_codes"], out["mx5_scale"] = u8(c5), u8(s5)
    c5f, s5f = q.to_mx(x, 32, scaling_mode="floor", elem_dtype=torch.float8_e5m2)
    out["mx5_codes_floor"], out["mx5_scale_floor"] = u8(c5f), u8(s5f)
    c4, s4 = q.to_mxfp4(x, 32)
    out["mx4_codes"], out["mx4_scale"] = u8(c4), u8(s4)

    # quantisation along dim 0 (scale blocks down the columns), both scale rules
    cd0, sd0 = q.to_mx_dim0(x, 32)
    out["mxd0_codes"], out["mxd0_scale"] = u8(cd0), u8(sd0)
    cd0f, sd0f = q.to_mx_dim0(x, 32, scaling_mode="floor")
    out["mxd0_codes_floor"], out["mxd0_scale_floor"] = u8(cd0f), u8(sd0f)

    # fp32 input across magnitude decades (tests/test_blockscaled_quantize.py:15-26)
    x32 = torch.randn(64, 256, generator=g) * torch.logspace(-6, 6, 64).unsqueeze(1)
    c32, s32 = q.to_mx(x32, 32)
    out["mx32_x"] = x32.numpy().copy()
    out["mx32_codes"] = u8(c32)
    out["mx32_scale"] = u8(s32)
    c32_5, s32_5 = q.to_mx(x32, 32, elem_dtype=torch.float8_e5m2)
    out["mx32_5_codes"], out["mx32_5_scale"] = u8(c32_5), u8(s32_5)
    c32_4, s32_4 = q.to_mxfp4(x32, 32)
    out["mx32_4_codes"], out["mx32_4_scale"] = u8(c32_4), u8(s32_4)

    # edge blocks (tests/test_blockscaled_quantize.py:39-53) and the known block max 500
    e = torch.tensor([[0.0] * 32, [1e-40] * 32, [float("inf")] * 32, [float("nan")] * 32,
                      [500.0] + [1.0] * 31, [448.0] + [0.5] * 31, [-448.0 * 4] + [3.0] * 31,
                      [2.0 ** -130] * 32], dtype=torch.float32)
    ce, se = q.to_mx(e, 32)
    out["mxedge_x"] = e.numpy().copy()
    out["mxedge_codes"] = u8(ce)
    out["mxedge_scale"] = u8(se)
    ce5, se5 = q.to_mx(e, 32, elem_dtype=torch.float8_e5m2)
    out["mxedge_5_codes"], out["mxedge_5_scale"] = u8(ce5), u8(se5)
    ce4, se4 = q.to_mxfp4(e, 32)
    out["mxedge_4_codes"], out["mxedge_4_scale"] = u8(ce4), u8(se4)
    cef, sef = q.to_mx(e, 32, scaling_mode="floor")
    out["mxedge_codes_floor"], out["mxedge_scale_floor"] = u8(cef), u8(sef)

    # ---- NVFP4 with and without the per-tensor scale ------------------------------------
    xn = torch.randn(144, 192, generator=g).to(torch.bfloat16)
    xn[:, 3] *= 20
    xn[2, :16] = 0
    xn[3, 16:32] = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0,
                                 -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0]).to(torch.bfloat16)
    pts = q.nvfp4_per_tensor_scale(xn.abs().amax())
    pk, sf, _ = q.to_nvfp4(xn, 16, pts)
    out["nv_x_bf16"] = xn.view(torch.int16).numpy().copy()
    out["nv_pts"] = pts.reshape(1).numpy().copy()
    out["nv_codes"] = u8(pk)
    out["nv_sf"] = u8(sf)
    out["nv_sf_blocked"] = u8(q.pack_scale_2d_to_blocked_contig(sf))
    pk0, sf0, _ = q.to_nvfp4(xn, 16, None)
    out["nv_codes_nopts"] = u8(pk0)
    out["nv_sf_nopts"] = u8(sf0)

    # inf / NaN blocks (values, a NaN next to finite values, -inf, a whole NaN row, inf next to NaN)
    xe = torch.zeros(6, 32)
    xe[0, :16] = float("nan"); xe[0, 16:] = 1.0
    xe[1, 3] = float("nan"); xe[1, :3] = 2.0; xe[1, 20] = float("inf")
    xe[2, :] = float("inf"); xe[2, 5] = -float("inf"); xe[2, 7] = 1.0
    xe[3, 0] = float("inf"); xe[3, 1:] = 3.0
    xe[4, :] = -float("nan")
    xe[5, 2] = -float("inf"); xe[5, 18] = float("nan")
    out["nvedge_x"] = xe.numpy().copy()
    out["nvedge_pts"] = np.array([0.01], np.float32)
    pke, sfe, _ = q.to_nvfp4(xe, 16, torch.tensor(0.01))
    out["nvedge_codes"] = u8(pke)
    out["nvedge_sf"] = u8(sfe)
    pke0, sfe0, _ = q.to_nvfp4(xe, 16, None)
    out["nvedge_codes_nopts"] = u8(pke0)
    out["nvedge_sf_nopts"] = u8(sfe0)

    # ---- fused output quantiser: the reference's torch model (tests/test_gemm_quant_out.py:57-101) -----
    quant_ref = extract_quant_ref(root, o)
    g2 = torch.Generator().manual_seed(1)
    y = torch.randn(48, 128, generator=g2) * torch.logspace(-5, 5, 48).unsqueeze(1)
    y[3] = 0
    y[4, :32] = 0
    y[5, 0] = 448.0; y[5, 1:32] = 1.0           # block maximum exactly dmax
    y[6, 0] = 448.0 * 2 ** -7; y[6, 1:32] = 1e-3
    y[7, 0] = 6.0 * 2 ** 3; y[7, 1:16] = 0.5
    y[8, :16] = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0])
    y[9, 40] = float("inf")
    y[10, 64] = -float("inf"); y[10, 65] = 3.0
    y[11] = 1e-42                                 # subnormal block maximum
    y[12] = 3e38
    out["qo_x"] = y.numpy().copy()
    out["qo_norms"] = np.array([1.0, 1.0 / 0.37], np.float32)
    for fmt in ("mxfp8_e4m3", "nvfp4", "mxfp4"):
        for i, norm in enumerate((1.0, 1.0 / 0.37)):
            qf, sfb, sq = quant_ref(y, fmt, norm)
            out[f"qo_{fmt}_{i}_q"] = qf.numpy().copy()
            out[f"qo_{fmt}_{i}_sf"] = sfb.numpy().copy()
            out[f"qo_{fmt}_{i}_scale"] = sq.numpy().copy()
    # NaN blocks: the E4M3 scale byte is the format's NaN and finite elements are multiplied by FLT_MAX; the
    # E8M0 byte comes from frexp(NaN), whose exponent is unspecified, and is recorded only for reference
    yn = torch.randn(4, 64, generator=g2)
    yn[0, 3] = float("nan")
    yn[2, 40] = float("nan"); yn[2, 41] = 0.0
    out["qonan_x"] = yn.numpy().copy()
    for fmt in ("mxfp8_e4m3", "nvfp4"):
        qf, sfb, sq = quant_ref(yn, fmt, 1.0)
        out[f"qonan_{fmt}_q"] = qf.numpy().copy()
        out[f"qonan_{fmt}_sf"] = sfb.numpy().copy()

    # ---- container round trip: dequantize() of both formats ------------------------------
    opa = o.BlockScaledOperand.quantize(x, "mxfp8_e4m3")
    out["mx_dequant"] = opa.dequantize(torch.float32).numpy().copy()
    opn = o.BlockScaledOperand.quantize(xn, "nvfp4", per_tensor_scale=pts)
    out["nv_dequant"] = opn.dequantize(torch.float32).numpy().copy()

    # ---- scale layout on ragged shapes ----------------------------------------------------
    s2 = torch.randint(0, 255, (300, 10), generator=g, dtype=torch.uint8)
    out["sf2d"] = s2.numpy().copy()
    out["sf2d_blocked"] = u8(q.pack_scale_2d_to_blocked_contig(s2))
    out["sf2d_to_blocked_flat"] = u8(q.to_blocked(s2))

    # ---- E2M1 encoder on a dense sweep (quack/blockscaled/quantize.py:165-207) -----------
    sweep = torch.linspace(-7, 7, 4481, dtype=torch.float32)
    out["e2m1_sweep_x"] = sweep.numpy().copy()
    out["e2m1_sweep_codes"] = q._f32_to_floatx_unpacked(sweep.clone(), 2, 1).numpy().copy()
    out["e2m1_values"] = np.array(q.FP4_E2M1FN_VALUES, dtype=np.float32)

    np.savez_compressed(os.path.join(here, "blockscaled_golden.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
