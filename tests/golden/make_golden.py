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

    # fp32 input across magnitude decades (tests/test_blockscaled_quantize.py:15-26)
    x32 = torch.randn(64, 256, generator=g) * torch.logspace(-6, 6, 64).unsqueeze(1)
    c32, s32 = q.to_mx(x32, 32)
    out["mx32_x"] = x32.numpy().copy()
    out["mx32_codes"] = u8(c32)
    out["mx32_scale"] = u8(s32)

    # edge blocks (tests/test_blockscaled_quantize.py:39-53) and the known block max 500
    e = torch.tensor([[0.0] * 32, [1e-40] * 32, [float("inf")] * 32, [float("nan")] * 32,
                      [500.0] + [1.0] * 31, [448.0] + [0.5] * 31, [-448.0 * 4] + [3.0] * 31,
                      [2.0 ** -130] * 32], dtype=torch.float32)
    ce, se = q.to_mx(e, 32)
    out["mxedge_x"] = e.numpy().copy()
    out["mxedge_codes"] = u8(ce)
    out["mxedge_scale"] = u8(se)

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
