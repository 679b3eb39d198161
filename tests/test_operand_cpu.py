"""Container / descriptor behaviour (host-only Python), mirroring the assertions of the
reference's tests/test_blockscaled_operand.py.  Operands are built with ``from_parts`` from
oracle-quantised bytes, so nothing here needs a GPU."""

import copy
import io
import pickle

import numpy as np
import pytest
import torch
import torch.utils._pytree as pytree

from oracle import blockscaled_oracle as orc
from quack_b200.blockscaled import (BLOCKSCALED_FORMAT_REGISTRY, MXFP4, MXFP4_BYTE, MXFP6_E2M3, MXFP6_E2M3_PACKED,
                                    MXFP8_E4M3, MXFP8_E5M2, NVFP4, BlockScaledFormat, BlockScaledOperand,
                                    mma_kind_for_pair, pack_scale_2d_to_blocked_contig, unpack_scale_blocked_to_2d)


def _operand(fmt="mxfp8_e4m3", mn=160, k=256, seed=0, pts=None):
    x = orc.make_activation(mn, k, seed)
    if fmt == "mxfp8_e4m3":
        c, s = orc.to_mx_e4m3(x)
        q = torch.from_numpy(c).view(torch.float8_e4m3fn)
        sf = torch.from_numpy(orc.pack_scale_blocked(s)).view(torch.float8_e8m0fnu)
        return x, BlockScaledOperand.from_parts(q, sf, fmt, orig_dtype=x.dtype)
    c, s = orc.to_nvfp4(x, pts)
    q = torch.from_numpy(c).view(torch.float4_e2m1fn_x2)
    sf = torch.from_numpy(orc.pack_scale_blocked(s)).view(torch.float8_e4m3fn)
    p = None if pts is None else torch.tensor([pts], dtype=torch.float32)
    return x, BlockScaledOperand.from_parts(q, sf, fmt, per_tensor_scale=p, orig_dtype=x.dtype)


def test_format_registry_and_legacy_names():
    assert BlockScaledFormat.from_name("mxfp8") is MXFP8_E4M3
    for name, fmt in BLOCKSCALED_FORMAT_REGISTRY.items():
        assert BlockScaledFormat.from_name(name) is fmt
    with pytest.raises(ValueError, match="unknown blockscaled format"):
        BlockScaledFormat.from_name("fp3")


def test_storage_logical_k():
    assert MXFP8_E4M3.storage_k(384) == 384 and MXFP8_E4M3.logical_k(384) == 384
    assert NVFP4.storage_k(384) == 192 and NVFP4.logical_k(192) == 384
    assert MXFP6_E2M3_PACKED.storage_k(128) == 96 and MXFP6_E2M3_PACKED.logical_k(96) == 128
    with pytest.raises(ValueError, match="whole storage"):
        MXFP6_E2M3_PACKED.storage_k(2)
    with pytest.raises(ValueError, match="whole packed groups"):
        MXFP6_E2M3_PACKED.logical_k(1)
    assert MXFP4_BYTE.is_byte_container and not MXFP4.is_byte_container and MXFP4.is_packed


def test_constructor_contract():
    f = BlockScaledFormat("x", torch.uint8, None, 8, 1, torch.float8_e8m0fnu, 32)
    assert f.elems_per_container == 1 and f.storage_layout is None
    with pytest.raises(TypeError, match="elems_per_container"):
        BlockScaledFormat("x", torch.uint8, None, 8, True, torch.float8_e8m0fnu, 32)
    with pytest.raises(ValueError, match="do not fit"):
        BlockScaledFormat("x", torch.uint8, None, 6, 2, torch.float8_e8m0fnu, 32)
    assert BlockScaledFormat.from_cutlass_dtypes("Float4E2M1FN", "Float8E4M3FN", 16) is NVFP4
    with pytest.raises(ValueError, match="no blockscaled format"):
        BlockScaledFormat.from_cutlass_dtypes("Float4E2M1FN", "Float8E4M3FN", 64)


def test_operand_metadata_and_roundtrip():
    x, op = _operand("mxfp8_e4m3")
    assert op.shape == tuple(x.shape) and op.dtype == x.dtype and op.quant_dim == -1
    assert op.qdata.dtype == torch.float8_e4m3fn and op.scale.dtype == torch.float8_e8m0fnu
    err = (op.dequantize(torch.float32) - x.float()).abs().max() / x.float().abs().max()
    assert err < 0.1
    pts = float(orc.nvfp4_per_tensor_scale(x.float().abs().max().item()))
    x4, op4 = _operand("nvfp4", pts=pts)
    assert op4.shape == tuple(x4.shape) and op4.qdata.shape == (160, 128)
    err4 = (op4.dequantize(torch.float32) - x4.float()).abs().max() / x4.float().abs().max()
    assert err4 < 0.6
    assert "nvfp4" in repr(op4) and "float4_e2m1fn_x2" in repr(op4) and "(160, 256)" in repr(op4)


def test_constructor_rejects():
    x, op = _operand()
    with pytest.raises(TypeError, match="qdata must be"):
        BlockScaledOperand.from_parts(op.qdata.view(torch.uint8), op.scale, "mxfp8_e4m3")
    with pytest.raises(TypeError, match="scale must be"):
        BlockScaledOperand.from_parts(op.qdata, op.scale.view(torch.float8_e4m3fn), "mxfp8_e4m3")
    with pytest.raises(ValueError, match="atom"):
        BlockScaledOperand.from_parts(op.qdata, op.scale.transpose(-1, -2), "mxfp8_e4m3")
    with pytest.raises(ValueError, match="32, 4, 4"):
        BlockScaledOperand.from_parts(op.qdata, op.scale.reshape(2, 2, 512), "mxfp8_e4m3")
    with pytest.raises(ValueError, match="per_tensor_scale"):
        BlockScaledOperand.from_parts(op.qdata, op.scale, "mxfp8_e4m3", per_tensor_scale=torch.ones(1))
    _, op4 = _operand("nvfp4")
    with pytest.raises(ValueError, match="scalar fp32"):
        BlockScaledOperand.from_parts(op4.qdata, op4.scale, "nvfp4", per_tensor_scale=torch.ones(2))
    with pytest.raises(ValueError, match="scalar fp32"):
        BlockScaledOperand.from_parts(op4.qdata, op4.scale, "nvfp4", per_tensor_scale=torch.ones(1, dtype=torch.float64))
    # uint8 scale views are re-viewed from the format, bytes unchanged
    op_u8 = BlockScaledOperand.from_parts(op4.qdata, op4.scale.view(torch.uint8), "nvfp4")
    assert op_u8.scale.dtype == torch.float8_e4m3fn
    assert torch.equal(op_u8.scale.view(torch.uint8), op4.scale.view(torch.uint8))


def test_padded_scale_dequantize_raises():
    x, op = _operand()
    padded = torch.zeros(3, 2, 32, 4, 4, dtype=torch.uint8).view(torch.float8_e8m0fnu)
    wide = BlockScaledOperand.from_parts(op.qdata, padded, "mxfp8_e4m3")  # shapes are not coupled at construction
    with pytest.raises(ValueError, match="Padded varlen scale buffers"):
        wide.dequantize()


def test_transpose_views():
    x, op = _operand()
    t = op.mT
    assert t.scale is op.scale and t.quant_dim == -2 and t.shape == (256, 160)
    assert t.qdata.stride() == (1, 256)
    assert torch.equal(t.dequantize(torch.float32), op.dequantize(torch.float32).mT)
    assert op.T.quant_dim == -2 and op.transpose(-2, -1).mT.quant_dim == -1
    b3 = BlockScaledOperand.from_parts(op.qdata.unsqueeze(0), op.scale.unsqueeze(0), "mxfp8_e4m3")
    with pytest.raises(ValueError, match="last two"):
        b3.transpose(0, 1)
    with pytest.raises(ValueError, match="2-D"):
        b3.T


def test_clone_to_deepcopy_and_torch_ops():
    x, op = _operand()
    c = op.clone()
    assert c.qdata.data_ptr() != op.qdata.data_ptr() and torch.equal(c.qdata.view(torch.uint8), op.qdata.view(torch.uint8))
    d = copy.deepcopy(op)
    assert torch.equal(d.scale.view(torch.uint8), op.scale.view(torch.uint8))
    assert op.to("cpu").device.type == "cpu"
    with pytest.raises(TypeError, match="dequantize"):
        op.to(torch.float16)
    with pytest.raises(TypeError):
        torch.mm(op, op.mT)
    with pytest.raises(TypeError):
        op + op


def test_save_load_and_pickle():
    _, op = _operand("nvfp4", pts=0.01)
    buf = io.BytesIO()
    torch.save({"w": op}, buf)
    buf.seek(0)
    back = torch.load(buf, weights_only=True)["w"]
    assert back.format == NVFP4 and back.quant_dim == -1
    assert torch.equal(back.qdata.view(torch.uint8), op.qdata.view(torch.uint8))
    assert torch.equal(back.per_tensor_scale, op.per_tensor_scale)
    assert pickle.loads(pickle.dumps(MXFP8_E4M3)) == MXFP8_E4M3
    # pickles that predate elems_per_container / storage_layout
    old = BlockScaledFormat.__new__(BlockScaledFormat)
    old.__setstate__({"name": "nvfp4", "qdata_dtype": torch.float4_e2m1fn_x2, "cutlass_dtype_name": "Float4E2M1FN",
                      "elem_bits": 4, "scale_dtype": torch.float8_e4m3fn, "sf_vec_size": 16, "has_per_tensor_scale": True})
    assert old == NVFP4
    fp6 = BlockScaledFormat.__new__(BlockScaledFormat)
    fp6.__setstate__({"name": "mxfp6_e2m3", "qdata_dtype": torch.uint8, "cutlass_dtype_name": "Float6E2M3FN",
                      "elem_bits": 6, "scale_dtype": torch.float8_e8m0fnu, "sf_vec_size": 32})
    assert fp6 == MXFP6_E2M3_PACKED


def test_pytree_roundtrip():
    _, op = _operand()
    for o in (op, op.mT):
        leaves, spec = pytree.tree_flatten(o)
        assert all(l is None or isinstance(l, torch.Tensor) for l in leaves)
        back = pytree.tree_unflatten(leaves, spec)
        assert back.format is MXFP8_E4M3 and back.shape == o.shape and back.quant_dim == o.quant_dim
        spec2 = pytree.treespec_loads(pytree.treespec_dumps(spec))
        assert pytree.tree_unflatten(leaves, spec2).shape == o.shape


def test_mma_kind_for_pair():
    assert mma_kind_for_pair(MXFP8_E4M3, MXFP8_E4M3) == "mxf8f6f4"
    assert mma_kind_for_pair(MXFP8_E4M3, MXFP8_E5M2) == "mxf8f6f4"
    assert mma_kind_for_pair(MXFP8_E4M3, MXFP4) == "mxf8f6f4"
    assert mma_kind_for_pair(NVFP4, NVFP4) == "mxf4nvf4" and mma_kind_for_pair(MXFP4, MXFP4) == "mxf4nvf4"
    with pytest.raises(ValueError, match="cannot pair"):
        mma_kind_for_pair(NVFP4, MXFP8_E4M3)
    with pytest.raises(ValueError, match="byte-per-element"):
        mma_kind_for_pair(MXFP4_BYTE, MXFP8_E4M3)
    with pytest.raises(ValueError, match="byte-per-element"):
        mma_kind_for_pair(MXFP6_E2M3, MXFP8_E4M3)
    e3m4 = BlockScaledFormat("mxfp8_e3m4", torch.uint8, None, 8, 1, torch.float8_e8m0fnu, 32)
    with pytest.raises(ValueError, match="no tcgen05 MMA element type"):
        mma_kind_for_pair(e3m4, MXFP8_E4M3)
    f128 = BlockScaledFormat("fp8_e4m3_1x128", torch.float8_e4m3fn, "Float8E4M3FN", 8, 1, torch.float32, 128)
    with pytest.raises(ValueError, match="no hardware MMA kind"):
        mma_kind_for_pair(f128, f128)


def test_from_parts_quant_dim():
    _, op = _operand()
    kn = BlockScaledOperand.from_parts(op.qdata.mT, op.scale, "mxfp8_e4m3", quant_dim=-2)
    assert kn.quant_dim == -2 and kn.shape == (256, 160)
    _, op4 = _operand("nvfp4")
    with pytest.raises(ValueError, match="packed dim"):
        BlockScaledOperand.from_parts(op4.qdata, op4.scale, "nvfp4", quant_dim=-2)
    assert BlockScaledOperand.from_parts(op4.qdata.mT, op4.scale, "nvfp4", quant_dim=-2).shape == (256, 160)
    with pytest.raises(ValueError, match="last two dims"):
        BlockScaledOperand.from_parts(op.qdata, op.scale, "mxfp8_e4m3", quant_dim=0 - 3)


def test_scale_layout_helpers_cpu(golden):
    s = torch.from_numpy(golden["sf2d"])
    b = pack_scale_2d_to_blocked_contig(s)
    assert np.array_equal(b.numpy(), golden["sf2d_blocked"])
    assert torch.equal(unpack_scale_blocked_to_2d(b, 300, 10)[0], s)


def test_quantize_needs_cuda_and_known_formats():
    x = torch.randn(128, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        BlockScaledOperand.quantize(x, "mxfp8_e4m3")
    with pytest.raises(NotImplementedError, match="no sm_100a quantizer"):
        BlockScaledOperand.quantize(x, "mxfp6_e2m3")
    with pytest.raises(ValueError, match="per_tensor_scale"):
        BlockScaledOperand.quantize(x, "mxfp8_e4m3", per_tensor_scale=torch.ones(1))
