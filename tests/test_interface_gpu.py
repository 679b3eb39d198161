"""The reference-shaped Python API (quack_b200.gemm_interface) on the GPU: shapes, dtypes,
error messages and numerics, following tests/test_gemm_blockscaled_interface.py of the
reference.  Operands are quantised by the CUDA quantizer (checked bit-exact elsewhere) and
compared with the torch fp32 reference of the same API (``gemm_blockscaled_ref``) and with the
CPU oracle."""

import numpy as np
import pytest
import torch

from oracle import blockscaled_oracle as orc
from tests.helpers import containers, make_operand_pair, rel_err

pytestmark = pytest.mark.gpu


def _quant(fmt, m, n, k, seed=0, pts=True):
    from quack_b200.blockscaled import BlockScaledOperand, nvfp4_per_tensor_scale
    a = orc.make_activation(m, k, seed).cuda()
    w = orc.make_weight(n, k, seed + 1).cuda()
    kw_a, kw_w = {}, {}
    if fmt == "nvfp4" and pts:
        kw_a = dict(per_tensor_scale=nvfp4_per_tensor_scale(a.abs().amax()))
        kw_w = dict(per_tensor_scale=nvfp4_per_tensor_scale(w.abs().amax()))
    return BlockScaledOperand.quantize(a, fmt, **kw_a), BlockScaledOperand.quantize(w, fmt, **kw_w)


@pytest.mark.parametrize("fmt", ["mxfp8_e4m3", "nvfp4"])
@pytest.mark.parametrize("shape", [(256, 512, 256), (128, 128, 128), (384, 256, 768), (1024, 1024, 512), (100, 96, 64)])
def test_gemm_against_reference(fmt, shape):
    from quack_b200.gemm_interface import gemm, gemm_blockscaled_ref
    m, n, k = shape
    A, W = _quant(fmt, m, n, k)
    out = gemm(A, W.mT)
    assert out.shape == (m, n) and out.dtype == torch.bfloat16
    ref = gemm_blockscaled_ref(A, W.mT, out_dtype=torch.float32)
    assert (out.float() - ref).abs().max() / ref.abs().max() < 5e-3


@pytest.mark.parametrize("fmt", ["mxfp8_e4m3", "nvfp4"])
def test_quantize_then_gemm_equals_oracle_pipeline(fmt):
    """quantize (CUDA) -> gemm (CUDA) vs quantize (oracle) -> dequant -> fp32 matmul (oracle)."""
    from quack_b200.gemm_interface import gemm
    m, n, k = 512, 768, 1024
    ops = make_operand_pair(fmt, m, n, k, seed=4)
    A, W = _quant(fmt, m, n, k, seed=4)
    assert np.array_equal(A.qdata.view(torch.uint8).cpu().numpy(), ops["ac"])
    assert np.array_equal(W.scale.view(torch.uint8).cpu().numpy(), ops["bsf_b"])
    bias = orc.make_bias(n)
    out = gemm(A, W.mT, bias=bias.cuda(), alpha=0.5)
    scale = 0.5 if ops["pa"] is None else np.float32(ops["pa"]) * np.float32(ops["pb"]) * np.float32(0.5)
    ref = orc.gemm_blockscaled_ref(ops["adq"], ops["bdq"], alpha=float(scale), bias=bias)
    assert rel_err(out.float().cpu().numpy(), ref) < 5e-3


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_out_dtypes_alpha_and_preallocated_out(out_dtype):
    from quack_b200.gemm_interface import gemm, gemm_blockscaled_ref
    A, W = _quant("mxfp8_e4m3", 256, 384, 512)
    ref = gemm_blockscaled_ref(A, W.mT, alpha=2.0, out_dtype=torch.float32)
    out = torch.empty(256, 384, dtype=out_dtype, device="cuda")
    res = gemm(A, W.mT, out=out, alpha=2.0)
    assert res is out
    assert (out.float() - ref).abs().max() / ref.abs().max() < (1e-5 if out_dtype == torch.float32 else 5e-3)
    alpha_t = torch.tensor([2.0], device="cuda")
    out2 = gemm(A, W.mT, alpha=alpha_t, out_dtype=out_dtype)
    assert torch.equal(out2, out)


def test_batched_operands():
    from quack_b200.blockscaled import BlockScaledOperand
    from quack_b200.gemm_interface import gemm, gemm_blockscaled_ref
    a = torch.stack([orc.make_activation(256, 256, s) for s in range(3)]).cuda()
    w = torch.stack([orc.make_weight(384, 256, 10 + s) for s in range(3)]).cuda()
    A, W = BlockScaledOperand.quantize(a, "mxfp8_e4m3"), BlockScaledOperand.quantize(w, "mxfp8_e4m3")
    out = gemm(A, W.mT)
    assert out.shape == (3, 256, 384)
    ref = gemm_blockscaled_ref(A, W.mT, out_dtype=torch.float32)
    assert (out.float() - ref).abs().max() / ref.abs().max() < 5e-3


def test_nvfp4_per_tensor_scales_fold_into_alpha():
    """Per-tensor scales live on the operands and are folded on the device
    (reference tests/test_gemm_blockscaled_interface.py:615-645)."""
    from quack_b200.gemm_interface import gemm, gemm_blockscaled_ref
    A, W = _quant("nvfp4", 256, 256, 512)
    assert A.per_tensor_scale is not None and W.per_tensor_scale is not None
    out = gemm(A, W.mT, alpha=1.5)
    ref = gemm_blockscaled_ref(A, W.mT, alpha=1.5, out_dtype=torch.float32)
    assert (out.float() - ref).abs().max() / ref.abs().max() < 5e-3
    hp = orc.make_activation(256, 512, 0).float() @ orc.make_weight(256, 512, 1).float().T * 1.5
    assert (out.float().cpu() - hp).abs().max() / hp.abs().max() < 0.25   # fp4 quantisation error, not a scale slip


def test_operand_orientation_and_type_errors():
    from quack_b200.blockscaled import BlockScaledOperand
    from quack_b200.gemm_interface import gemm, gemm_act
    A, W = _quant("mxfp8_e4m3", 256, 256, 256)
    with pytest.raises(ValueError, match="B must be quantized along dim -2"):
        gemm(A, W)                       # square weight passed without .mT
    with pytest.raises(ValueError, match="A must be quantized along its last dim"):
        gemm(A.mT, W.mT)
    with pytest.raises(TypeError, match="no longer accepted"):
        gemm((A.qdata, A.scale), W.mT)
    with pytest.raises(TypeError, match="BlockScaledOperand"):
        gemm(A, [W.qdata, W.scale])
    A4, _ = _quant("nvfp4", 256, 256, 256)
    with pytest.raises(ValueError, match="cannot pair"):
        gemm(A4, W.mT)
    with pytest.raises(NotImplementedError, match="only supported by quack.gemm"):
        gemm_act(A, W.mT, activation="relu", postact_dtype="nvfp4")
    with pytest.raises(ValueError, match="unknown blockscaled format"):
        gemm(A, W.mT, out_dtype="fp3")
    with pytest.raises(NotImplementedError):
        gemm(torch.randn(4, 4, device="cuda"), torch.randn(4, 4, device="cuda"))
    u8 = BlockScaledOperand.from_parts(A.qdata, A.scale.view(torch.uint8), "mxfp8_e4m3")   # uint8 scale view
    assert torch.equal(gemm(u8, W.mT), gemm(A, W.mT))


@pytest.mark.parametrize("fmt", ["mxfp8_e4m3", "nvfp4"])
@pytest.mark.parametrize("activation", ["relu", "gelu_tanh_approx", "swiglu", "reglu"])
def test_gemm_act(fmt, activation):
    """postact rel error < 1e-2 (reference :303-328); bias + store_preact=False (:331-343)."""
    from quack_b200.gemm_interface import gated_to_pytorch_fn_map, gemm_act, gemm_blockscaled_ref, act_to_pytorch_fn_map
    m, n, k = 256, 512, 256
    A, W = _quant(fmt, m, n, k, seed=2)
    bias = orc.make_bias(n).cuda()
    pre_ref = gemm_blockscaled_ref(A, W.mT, alpha=2.0, out_dtype=torch.float32) + bias
    gated = activation in gated_to_pytorch_fn_map
    post_ref = (gated_to_pytorch_fn_map[activation](pre_ref[:, ::2], pre_ref[:, 1::2]) if gated
                else act_to_pytorch_fn_map[activation](pre_ref))
    pre, post = gemm_act(A, W.mT, bias=bias, activation=activation, alpha=2.0)
    assert pre.shape == (m, n) and post.shape == (m, n // 2 if gated else n)
    assert (pre.float() - pre_ref).abs().max() / pre_ref.abs().max() < 5e-3
    assert (post.float() - post_ref).abs().max() / post_ref.abs().max() < 1e-2
    none_pre, post2 = gemm_act(A, W.mT, bias=bias, activation=activation, alpha=2.0, store_preact=False)
    assert none_pre is None and torch.equal(post2, post)


@pytest.mark.parametrize("ofmt", ["mxfp8_e4m3", "nvfp4"])
def test_quantised_output_roundtrip_into_next_gemm(ofmt):
    """gemm(..., out_dtype=format) returns a container that feeds the next GEMM
    (reference tests/test_gemm_quant_out.py:187-227)."""
    from quack_b200.blockscaled import BlockScaledOperand
    from quack_b200.gemm_interface import gemm, gemm_blockscaled_ref
    m, n, k = 256, 512, 256
    A, W = _quant("nvfp4", m, n, k, seed=5)
    ref = gemm_blockscaled_ref(A, W.mT, out_dtype=torch.float32)
    kw = {}
    if ofmt == "nvfp4":
        kw["out_per_tensor_scale"] = float(ref.abs().max() / (448.0 * 6.0))
    res = gemm(A, W.mT, out_dtype=ofmt, **kw)
    assert isinstance(res, BlockScaledOperand) and res.format.name == ofmt and res.shape == (m, n) and res.quant_dim == -1
    if ofmt == "nvfp4":
        assert res.per_tensor_scale.item() == pytest.approx(kw["out_per_tensor_scale"])
    deq = res.dequantize(torch.float32)
    tol = 0.08 if ofmt == "mxfp8_e4m3" else 0.3
    assert (deq - ref).abs().max() / ref.abs().max() < tol
    W2 = BlockScaledOperand.quantize(orc.make_weight(128, n, 9).cuda(), ofmt,
                                     **({"per_tensor_scale": torch.tensor([1e-4], device="cuda")} if ofmt == "nvfp4" else {}))
    out2 = gemm(res, W2.mT)
    ref2 = gemm_blockscaled_ref(res, W2.mT, out_dtype=torch.float32)
    assert (out2.float() - ref2).abs().max() / ref2.abs().max() < 5e-3
    # preallocated container output
    res2 = gemm(A, W.mT, out=res.clone(), out_dtype=ofmt, **kw)
    assert torch.equal(res2.qdata.view(torch.uint8), res.qdata.view(torch.uint8))
    assert torch.equal(res2.scale.view(torch.uint8), res.scale.view(torch.uint8))


def test_fused_mlp_up_projection_quantised():
    """gemm_act_quant: SwiGLU + NVFP4 output in one kernel, consumed by the down projection."""
    from quack_b200.blockscaled import BlockScaledOperand, nvfp4_per_tensor_scale
    from quack_b200.gemm_interface import gemm, gemm_act, gemm_act_quant, gemm_blockscaled_ref
    m, k, n = 512, 512, 1024
    A, W = _quant("nvfp4", m, n, k, seed=12)
    bias = orc.make_bias(n).cuda()
    _, post_hp = gemm_act(A, W.mT, bias=bias, activation="swiglu", postact_dtype=torch.float32, store_preact=False)
    pts_out = nvfp4_per_tensor_scale(post_hp.abs().amax())
    h = gemm_act_quant(A, W.mT, bias=bias, activation="swiglu", postact_format="nvfp4", postact_per_tensor_scale=pts_out)
    assert isinstance(h, BlockScaledOperand) and h.shape == (m, n // 2) and h.format.name == "nvfp4"
    # identical to quantising the fp32 SwiGLU output with the stand-alone quantizer
    # (same arithmetic up to the rounding of rcp), so the dequantised tensors agree closely
    h_ref = BlockScaledOperand.quantize(post_hp, "nvfp4", per_tensor_scale=pts_out)
    d1, d2 = h.dequantize(torch.float32), h_ref.dequantize(torch.float32)
    assert (d1 - post_hp).abs().max() / post_hp.abs().max() < 0.3
    assert (d1 - d2).abs().max() / post_hp.abs().max() < 0.15
    Wd = BlockScaledOperand.quantize(orc.make_weight(256, n // 2, 13).cuda(), "nvfp4",
                                     per_tensor_scale=torch.tensor([2e-4], device="cuda"))
    y = gemm(h, Wd.mT)
    yref = gemm_blockscaled_ref(h, Wd.mT, out_dtype=torch.float32)
    assert (y.float() - yref).abs().max() / yref.abs().max() < 5e-3


def test_config1_nvfp4_8192_bias_properties():
    """Configuration 1 at full size (NVFP4, M=N=K=8192, fp32 bias).  The fp32 reference is
    computed on the GPU from the dequantised operands (TF32 off), and two size-independent
    properties are checked: linearity in alpha and exact bias separation."""
    from quack_b200.gemm_interface import gemm
    torch.backends.cuda.matmul.allow_tf32 = False
    m = n = k = 8192
    A, W = _quant("nvfp4", m, n, k)
    bias = orc.make_bias(n).cuda()
    out = gemm(A, W.mT, bias=bias)
    a_dq = A.dequantize(torch.float32)
    w_dq = W.dequantize(torch.float32)
    ref = a_dq @ w_dq.T + bias
    err = (out.float() - ref).abs().max() / ref.abs().max()
    assert err < 1e-2, err
    del a_dq, w_dq, ref
    o32 = gemm(A, W.mT, out_dtype=torch.float32)
    o32b = gemm(A, W.mT, bias=bias, out_dtype=torch.float32)
    assert torch.equal(o32b, o32 + bias)                       # bias is one fp32 add after alpha
    o32x2 = gemm(A, W.mT, alpha=2.0, out_dtype=torch.float32)
    assert torch.equal(o32x2, o32 * 2.0)                       # scaling by a power of two is exact


@pytest.mark.parametrize("fmt", ["mxfp8_e4m3", "nvfp4"])
def test_explicit_config_selects_the_dynamic_scheduler(fmt):
    """``GemmConfig(is_dynamic_persistent=True)`` runs the cluster-launch-control scheduler; the
    result is bit-identical to the static schedule of the same tile shape."""
    from quack_b200 import _lib
    from quack_b200.gemm_config import GemmConfig
    from quack_b200.gemm_interface import gemm
    m, n, k = 2048, 3072, 1024
    A, W = _quant(fmt, m, n, k)
    bias = orc.make_bias(n).cuda()
    base = gemm(A, W.mT, bias=bias)
    for tile_m, tile_n, cm in [(256, 256, 2), (128, 128, 1), (256, 192, 2)]:
        outs = []
        for dyn in (False, True):
            cfg = GemmConfig(tile_m=tile_m, tile_n=tile_n, cluster_m=cm, cluster_n=1, pingpong=False, is_dynamic_persistent=dyn)
            n0 = _lib.launch_count()
            outs.append(gemm(A, W.mT, bias=bias, config=cfg))
            assert _lib.launch_count() == n0 + 1
        assert torch.equal(outs[0], outs[1])
        assert (outs[0].float() - base.float()).abs().max() <= 1e-2 * base.float().abs().max()


@pytest.mark.parametrize("fmt", ["mxfp8_e4m3", "nvfp4"])
@pytest.mark.parametrize("cdt", [torch.bfloat16, torch.float16, torch.float32])
def test_gemm_add_residual(fmt, cdt):
    """gemm_add / gemm_add_inplace: D = alpha A B + beta C + bias, C of any float dtype, aligned and not,
    batched, tensor beta, and aliasing the output (reference tests of gemm_add in
    tests/test_gemm_blockscaled_interface.py)."""
    from quack_b200.gemm_interface import gemm, gemm_add, gemm_add_inplace, gemm_add_ref
    for (m, n, k) in [(256, 512, 256), (200, 456 if fmt == "mxfp8_e4m3" else 448, 384), (1, 128, 64), (1024, 2048, 512)]:
        A, W = _quant(fmt, m, n, k)
        g = torch.Generator(device="cuda").manual_seed(5)
        C = torch.randn(m, n, generator=g, device="cuda").to(cdt)
        bias = orc.make_bias(n).cuda()
        out = gemm_add(A, W.mT, C, bias=bias, alpha=0.5, beta=-1.25, out_dtype=torch.float32)
        ref = gemm_add_ref(A.dequantize(torch.float32), W.dequantize(torch.float32).mT, C, bias=bias, alpha=0.5, beta=-1.25,
                           out_dtype=torch.float32)
        assert (out - ref).abs().max() <= 1e-4 * ref.abs().max() + 1e-5, (m, n, k)
        # exactly the plain GEMM plus the residual when beta = 1 and the sum is exact in fp32
        plain = gemm(A, W.mT, out_dtype=torch.float32)
        again = gemm_add(A, W.mT, torch.zeros_like(C), out_dtype=torch.float32)
        assert torch.equal(plain, again)
        # in place, tensor beta
        acc = C.float().clone()
        gemm_add_inplace(A, W.mT, acc, beta=torch.tensor([2.0], device="cuda"))
        ref2 = gemm_add_ref(A.dequantize(torch.float32), W.dequantize(torch.float32).mT, C.float(), beta=2.0, out_dtype=torch.float32)
        assert (acc - ref2).abs().max() <= 1e-4 * ref2.abs().max() + 1e-5
    # a strided (unaligned rows) residual and a bf16 output
    A, W = _quant(fmt, 384, 256, 256)
    big = torch.randn(384, 256 + 3, device="cuda").to(cdt)
    Cs = big[:, 3:]
    out = gemm_add(A, W.mT, Cs)
    ref = gemm_add_ref(A.dequantize(torch.float32), W.dequantize(torch.float32).mT, Cs, out_dtype=torch.float32)
    assert out.dtype == torch.bfloat16 and (out.float() - ref).abs().max() <= 1e-2 * ref.abs().max()


def test_gemm_act_with_residual():
    from quack_b200.gemm_interface import gemm_act, gemm_act_ref
    A, W = _quant("mxfp8_e4m3", 512, 1024, 256)
    C = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16)
    pre, post = gemm_act(A, W.mT, C=C, activation="swiglu", out_dtype=torch.float32, postact_dtype=torch.float32)
    rpre, rpost = gemm_act_ref(A.dequantize(torch.float32), W.dequantize(torch.float32).mT, C=C, activation="swiglu",
                               out_dtype=torch.float32, postact_dtype=torch.float32)
    assert (pre - rpre).abs().max() <= 1e-4 * rpre.abs().max() + 1e-5
    assert (post - rpost).abs().max() <= 2e-3 * rpost.abs().max() + 1e-4
