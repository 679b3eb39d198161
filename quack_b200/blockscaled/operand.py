"""Block-scaled format descriptors and the operand container.

Host-only Python with the observable behaviour of ``quack/blockscaled/operand.py``
(reference): ``BlockScaledFormat`` (:65-278) describes a quantisation format,
``BlockScaledOperand`` (:550-946) bundles quantised values, blocked scale factors, the format,
the optional NVFP4 per-tensor scale, the original dtype and the quantised axis.  Quantising
runs the CUDA kernels of this package; ``dequantize`` is a torch helper for tests.
"""

from __future__ import annotations

import copy as _copy
import dataclasses
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.utils._pytree as _pytree

from .quantize import QUANTIZERS, check_blocked_scale_atom, quantize_to_blocked

__all__ = [
    "BlockScaledFormat", "BlockScaledOperand", "BLOCKSCALED_FORMAT_REGISTRY", "mma_kind_for_pair",
    "MXFP8_E4M3", "MXFP8_E5M2", "MXFP4", "MXFP4_BYTE", "NVFP4", "MXFP6_E2M3", "MXFP6_E3M2",
    "MXFP6_E2M3_PACKED", "MXFP6_E3M2_PACKED", "MXFP6_E2M3_BYTE", "MXFP6_E3M2_BYTE",
]

_LAYOUTS = (None, "container_v1", "packed_lsb_v1")
_FIELD_ORDER = ("name", "qdata_dtype", "cutlass_dtype_name", "elem_bits", "elems_per_container", "scale_dtype",
                "sf_vec_size", "has_per_tensor_scale", "storage_layout")


def _positive_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) and v > 0


@dataclass(frozen=True)
class BlockScaledFormat:
    """Frozen, hashable descriptor of a block-scaled format.  Field order is part of the
    public constructor / pickle contract."""

    name: str
    qdata_dtype: torch.dtype
    cutlass_dtype_name: Optional[str]   # MMA element type name; None = host-only format
    elem_bits: int
    elems_per_container: int            # fp4x2: 2; one code per storage element: 1
    scale_dtype: torch.dtype
    sf_vec_size: int                    # logical K elements per scale factor
    has_per_tensor_scale: bool = False
    storage_layout: Optional[str] = None  # None (legacy container) | container_v1 | packed_lsb_v1

    def __post_init__(self):
        if not isinstance(self.name, str) or not self.name:
            raise TypeError("format name must be a non-empty str")
        if not isinstance(self.qdata_dtype, torch.dtype):
            raise TypeError(f"qdata_dtype must be a torch.dtype, got {self.qdata_dtype!r}")
        if self.cutlass_dtype_name is not None and not isinstance(self.cutlass_dtype_name, str):
            raise TypeError("cutlass_dtype_name must be a str or None")
        for field in ("elem_bits", "elems_per_container", "sf_vec_size"):
            if not _positive_int(getattr(self, field)):
                raise TypeError(f"{field} must be a positive int, got {getattr(self, field)!r}")
        if not isinstance(self.scale_dtype, torch.dtype):
            raise TypeError(f"scale_dtype must be a torch.dtype, got {self.scale_dtype!r}")
        if not isinstance(self.has_per_tensor_scale, bool):
            raise TypeError("has_per_tensor_scale must be bool")
        if self.storage_layout not in _LAYOUTS:
            raise ValueError("storage_layout must be None, 'container_v1', or 'packed_lsb_v1', "
                             f"got {self.storage_layout!r}")
        if self.storage_layout != "packed_lsb_v1" and self.elem_bits * self.elems_per_container > self.storage_elem_bits:
            raise ValueError(
                f"{self.name}: {self.elems_per_container} x {self.elem_bits}-bit values do not fit in a "
                f"{self.storage_elem_bits}-bit storage element")

    def __setstate__(self, state):
        """Accept pickles written before ``elems_per_container`` / ``storage_layout`` existed
        (reference :94-142): derive the missing fields, rename the short-lived unversioned
        packed-fp6 descriptors, then validate."""
        if not isinstance(state, dict):
            raise TypeError(f"invalid BlockScaledFormat pickle state: {type(state)}")
        s = dict(state)
        had_layout = "storage_layout" in s
        if "elems_per_container" not in s:
            sbits, ebits = s["qdata_dtype"].itemsize * 8, s["elem_bits"]
            if s.get("storage_layout") == "packed_lsb_v1" or (not had_layout and sbits % ebits):
                s["elems_per_container"] = 1
                s.setdefault("storage_layout", "packed_lsb_v1")
            elif sbits % ebits == 0:
                s["elems_per_container"] = sbits // ebits
            else:
                raise ValueError("cannot infer elems_per_container from serialized format state")
        s.setdefault("has_per_tensor_scale", False)
        s.setdefault("storage_layout", None)
        if s["storage_layout"] == "packed_lsb_v1":
            s["name"] = {"mxfp6_e2m3": "mxfp6_e2m3_packed", "mxfp6_e3m2": "mxfp6_e3m2_packed"}.get(s["name"], s["name"])
        for f in _FIELD_ORDER:
            if f not in s:
                raise ValueError(f"BlockScaledFormat pickle is missing {f!r}")
            object.__setattr__(self, f, s[f])
        self.__post_init__()

    # ---- storage <-> logical K ----
    @property
    def storage_elem_bits(self) -> int:
        return self.qdata_dtype.itemsize * 8

    @property
    def is_packed(self) -> bool:
        """True when a qdata row holds more logical elements than storage elements."""
        return getattr(self, "storage_layout", None) == "packed_lsb_v1" or self.elems_per_container > 1

    @property
    def is_byte_container(self) -> bool:
        """Deprecated one-code-per-storage-element sub-byte storage."""
        return not self.is_packed and self.elem_bits < self.storage_elem_bits

    def storage_k(self, logical_k: int) -> int:
        if getattr(self, "storage_layout", None) == "packed_lsb_v1":
            bits = logical_k * self.elem_bits
            if bits % self.storage_elem_bits:
                raise ValueError(f"{self.name}: logical K={logical_k} does not fill whole storage elements "
                                 f"({self.elem_bits}-bit codes in {self.storage_elem_bits}-bit units)")
            return bits // self.storage_elem_bits
        if logical_k % self.elems_per_container:
            raise ValueError(f"{self.name}: logical K={logical_k} is not divisible by "
                             f"elems_per_container={self.elems_per_container}")
        return logical_k // self.elems_per_container

    def logical_k(self, storage_k: int) -> int:
        if getattr(self, "storage_layout", None) == "packed_lsb_v1":
            bits = storage_k * self.storage_elem_bits
            if bits % self.elem_bits:
                raise ValueError(f"{self.name}: storage K={storage_k} is not whole packed groups "
                                 f"({self.storage_elem_bits}-bit units of {self.elem_bits}-bit codes)")
            return bits // self.elem_bits
        return storage_k * self.elems_per_container

    def to_cutlass_dtype(self):
        """The reference resolves the CuTe-DSL element type here; this package has no DSL."""
        if self.cutlass_dtype_name is None:
            raise ValueError(f"{self.name} has no CuTe-DSL element type")
        import cutlass  # optional dependency, only for callers that still want the DSL type

        return getattr(cutlass, self.cutlass_dtype_name)

    @classmethod
    def from_name(cls, name: str) -> "BlockScaledFormat":
        key = _LEGACY_FORMAT_NAMES.get(name, name)
        fmt = BLOCKSCALED_FORMAT_REGISTRY.get(key)
        if fmt is None:
            raise ValueError(f"unknown blockscaled format {name!r}; known: {sorted(BLOCKSCALED_FORMAT_REGISTRY)}")
        return fmt

    @classmethod
    def from_cutlass_dtypes(cls, ab_dtype, sf_dtype, sf_vec_size: int) -> "BlockScaledFormat":
        """Look a format up by (MMA element type, scale type, vector size).  Accepts DSL type
        objects or their names."""
        def _n(t):
            return t if isinstance(t, str) else getattr(t, "__name__", str(t))
        scale_names = {torch.float8_e8m0fnu: "Float8E8M0FNU", torch.float8_e4m3fn: "Float8E4M3FN"}
        for fmt in BLOCKSCALED_FORMAT_REGISTRY.values():
            if (fmt.cutlass_dtype_name is not None and not fmt.is_byte_container
                    and fmt.cutlass_dtype_name == _n(ab_dtype) and scale_names.get(fmt.scale_dtype) == _n(sf_dtype)
                    and fmt.sf_vec_size == sf_vec_size):
                return fmt
        raise ValueError(f"no blockscaled format matches (ab={ab_dtype}, sf={sf_dtype}, vec={sf_vec_size})")


_E8 = torch.float8_e8m0fnu
MXFP8_E4M3 = BlockScaledFormat("mxfp8_e4m3", torch.float8_e4m3fn, "Float8E4M3FN", 8, 1, _E8, 32)
MXFP8_E5M2 = BlockScaledFormat("mxfp8_e5m2", torch.float8_e5m2, "Float8E5M2", 8, 1, _E8, 32)
MXFP4 = BlockScaledFormat("mxfp4", torch.float4_e2m1fn_x2, "Float4E2M1FN", 4, 2, _E8, 32)
NVFP4 = BlockScaledFormat("nvfp4", torch.float4_e2m1fn_x2, "Float4E2M1FN", 4, 2, torch.float8_e4m3fn, 16,
                          has_per_tensor_scale=True)
MXFP6_E2M3 = BlockScaledFormat("mxfp6_e2m3", torch.uint8, "Float6E2M3FN", 6, 1, _E8, 32)
MXFP6_E3M2 = BlockScaledFormat("mxfp6_e3m2", torch.uint8, "Float6E3M2FN", 6, 1, _E8, 32)
MXFP6_E2M3_PACKED = BlockScaledFormat("mxfp6_e2m3_packed", torch.uint8, "Float6E2M3FN", 6, 1, _E8, 32,
                                      storage_layout="packed_lsb_v1")
MXFP6_E3M2_PACKED = BlockScaledFormat("mxfp6_e3m2_packed", torch.uint8, "Float6E3M2FN", 6, 1, _E8, 32,
                                      storage_layout="packed_lsb_v1")
MXFP4_BYTE = BlockScaledFormat("mxfp4_byte", torch.uint8, "Float4E2M1FN", 4, 1, _E8, 32)
MXFP6_E2M3_BYTE = MXFP6_E2M3
MXFP6_E3M2_BYTE = MXFP6_E3M2

BLOCKSCALED_FORMAT_REGISTRY = {f.name: f for f in (
    MXFP8_E4M3, MXFP8_E5M2, MXFP4, NVFP4, MXFP6_E2M3, MXFP6_E3M2, MXFP6_E2M3_PACKED, MXFP6_E3M2_PACKED, MXFP4_BYTE)}

_LEGACY_FORMAT_NAMES = {"mxfp8": "mxfp8_e4m3", "mxfp6_e2m3_byte": "mxfp6_e2m3", "mxfp6_e3m2_byte": "mxfp6_e3m2"}
_CANONICAL_TO_LEGACY = {"mxfp8_e4m3": "mxfp8"}


def legacy_format_name(fmt: BlockScaledFormat) -> str:
    return _CANONICAL_TO_LEGACY.get(fmt.name, fmt.name)


def _mma_element_class(fmt: BlockScaledFormat) -> Optional[str]:
    name = fmt.cutlass_dtype_name or ""
    for prefix, cls in (("Float8", "f8"), ("Float6", "f6"), ("Float4", "f4")):
        if name.startswith(prefix):
            return cls
    return None


def mma_kind_for_pair(fmt_a: BlockScaledFormat, fmt_b: BlockScaledFormat) -> str:
    """tcgen05 MMA kind of an (A, B) format pair, or ValueError when the hardware cannot
    express it (reference :418-483).  nvfp4 pairs only with nvfp4 (``mxf4nvf4``); mxfp4 x
    mxfp4 is ``mxf4nvf4`` too; every other e8m0 / vec-32 pair of fp8/fp6/fp4 elements is
    ``mxf8f6f4``.  This is legality only: which kinds have a kernel is decided at dispatch."""
    for f in (fmt_a, fmt_b):
        if f.is_byte_container:
            raise ValueError(f"{f.name} uses deprecated byte-per-element sub-byte storage and is host-side "
                             "compatibility only; call operand.to_packed() before GEMM")
    if "nvfp4" in (fmt_a.name, fmt_b.name):
        if fmt_a.name == fmt_b.name:
            return "mxf4nvf4"
        other = fmt_b.name if fmt_a.name == "nvfp4" else fmt_a.name
        raise ValueError(f"nvfp4 (e4m3 scales, vec 16) cannot pair with {other}: the mxf4nvf4 MMA kind's scale "
                         "config is instruction-wide, so it requires nvfp4 on both operands")
    if fmt_a.name == fmt_b.name == "mxfp4":
        return "mxf4nvf4"
    for f in (fmt_a, fmt_b):
        if _mma_element_class(f) is None:
            raise ValueError(f"{f.name} has no tcgen05 MMA element type (cutlass_dtype_name={f.cutlass_dtype_name}): "
                             "no hardware blockscaled MMA kind exists for this format")
        if f.scale_dtype != torch.float8_e8m0fnu or f.sf_vec_size != 32:
            raise ValueError(f"{f.name} (scales {f.scale_dtype}, vec {f.sf_vec_size}) has no hardware MMA kind: "
                             "kind::mxf8f6f4 requires e8m0 scales with vec size 32")
    return "mxf8f6f4"


_INTERIM_PACKED = {("mxfp6_e2m3", "packed_lsb_v1"): MXFP6_E2M3_PACKED, ("mxfp6_e3m2", "packed_lsb_v1"): MXFP6_E3M2_PACKED}


def _coerce_format(format) -> BlockScaledFormat:
    if isinstance(format, str):
        return BlockScaledFormat.from_name(format)
    if not isinstance(format, BlockScaledFormat):
        raise TypeError(f"format must be a BlockScaledFormat or str, got {type(format)}")
    target = _INTERIM_PACKED.get((format.name, getattr(format, "storage_layout", None)))
    if target is None:
        return format
    if dataclasses.replace(format, name=target.name) != target:
        raise ValueError(f"ambiguous interim packed FP6 descriptor {format.name}: fields do not match {target.name}")
    return target


def _normalize_quant_dim(dim: int, ndim: int) -> int:
    d = dim if dim < 0 else dim - ndim
    if d not in (-1, -2):
        raise ValueError(f"quant_dim must be one of the last two dims, got {dim}")
    return d


def _packed_dim(qdata: torch.Tensor, fmt: BlockScaledFormat) -> int:
    """The unit-stride dim (packing runs along it).  Dims of extent 1 report arbitrary
    strides, so longer dims win; the innermost dim wins ties."""
    fallback = None
    for d in reversed(range(qdata.ndim)):
        if qdata.stride(d) == 1:
            if qdata.shape[d] != 1:
                return d
            if fallback is None:
                fallback = d
    if fallback is None:
        raise ValueError(f"qdata has no unit-stride dim: shape={tuple(qdata.shape)}, stride={qdata.stride()}")
    return fallback


@dataclass(frozen=True, eq=False)
class BlockScaledOperand:
    """Quantised GEMM operand: a plain container, not a tensor.  ``shape`` / ``dtype``
    describe the logical (unpacked, high-precision) view; torch ops reject it."""

    qdata: torch.Tensor
    scale: torch.Tensor
    format: BlockScaledFormat
    per_tensor_scale: Optional[torch.Tensor] = None
    orig_dtype: torch.dtype = torch.bfloat16
    quant_dim: Optional[int] = None   # -1 or -2: the logical dim the scale vectors run along

    def __post_init__(self):
        fmt = _coerce_format(self.format)
        object.__setattr__(self, "format", fmt)
        if self.qdata.dtype != fmt.qdata_dtype:
            raise TypeError(f"{fmt.name} qdata must be {fmt.qdata_dtype}, got {self.qdata.dtype}")
        check_blocked_scale_atom(self.scale, "scale")
        if self.scale.dtype == torch.uint8:  # scales that crossed a collective arrive as bytes
            object.__setattr__(self, "scale", self.scale.view(fmt.scale_dtype))
        elif self.scale.dtype != fmt.scale_dtype:
            raise TypeError(f"{fmt.name} scale must be {fmt.scale_dtype}, got {self.scale.dtype}")
        pts = self.per_tensor_scale
        if pts is not None:
            if not fmt.has_per_tensor_scale:
                raise ValueError(f"{fmt.name} does not take a per_tensor_scale")
            if pts.numel() != 1 or pts.dtype != torch.float32:
                raise ValueError(f"per_tensor_scale must be a scalar fp32 tensor, got {pts.dtype} with "
                                 f"{pts.numel()} elements")
            object.__setattr__(self, "per_tensor_scale", pts.reshape(1))
        if self.qdata.device != self.scale.device:
            raise ValueError(f"qdata on {self.qdata.device} but scale on {self.scale.device}")
        if pts is not None and self.qdata.device != pts.device:
            raise ValueError(f"qdata on {self.qdata.device} but per_tensor_scale on {pts.device}")
        want = None if self.quant_dim is None else _normalize_quant_dim(self.quant_dim, self.ndim)
        if fmt.is_packed:
            derived = -1 if _packed_dim(self.qdata, fmt) == self.qdata.ndim - 1 else -2
            if want is not None and want != derived:
                raise ValueError(f"quant_dim={self.quant_dim} conflicts with the {fmt.name} packed dim "
                                 f"(packing runs along the quantized axis, here dim {derived})")
            want = derived
        object.__setattr__(self, "quant_dim", -1 if want is None else want)

    # ---- logical metadata ----
    @property
    def ndim(self) -> int:
        return self.qdata.ndim

    @property
    def shape(self) -> Tuple[int, ...]:
        if not self.format.is_packed:
            return tuple(self.qdata.shape)
        k_dim = self._mn_k_dims()[1]
        return tuple(self.format.logical_k(s) if d == k_dim else s for d, s in enumerate(self.qdata.shape))

    @property
    def dtype(self) -> torch.dtype:
        return self.orig_dtype

    @property
    def device(self) -> torch.device:
        return self.qdata.device

    def _mn_k_dims(self) -> Tuple[int, int]:
        lo, hi = self.ndim - 2, self.ndim - 1
        return (lo, hi) if self.quant_dim == -1 else (hi, lo)

    # ---- views ----
    def _view(self, qdata: torch.Tensor, quant_dim: int) -> "BlockScaledOperand":
        # a stride swap cannot break an invariant checked at construction: skip re-validation
        new = object.__new__(BlockScaledOperand)
        for k, v in (("qdata", qdata), ("scale", self.scale), ("format", self.format),
                     ("per_tensor_scale", self.per_tensor_scale), ("orig_dtype", self.orig_dtype),
                     ("quant_dim", quant_dim)):
            object.__setattr__(new, k, v)
        return new

    @property
    def mT(self) -> "BlockScaledOperand":
        """Swap the last two logical dims: qdata stride swap, the SAME scale object, and the
        quantised axis flips (-1 <-> -2)."""
        return self._view(self.qdata.transpose(-2, -1), -3 - self.quant_dim)

    @property
    def T(self) -> "BlockScaledOperand":
        if self.ndim != 2:
            raise ValueError(f"BlockScaledOperand.T requires 2-D, got {self.ndim}-D")
        return self.mT

    def transpose(self, dim0: int, dim1: int) -> "BlockScaledOperand":
        d0, d1 = dim0 % self.ndim, dim1 % self.ndim
        if {d0, d1} != {self.ndim - 2, self.ndim - 1}:
            raise ValueError(f"BlockScaledOperand.transpose({d0}, {d1}): only the last two dims may swap "
                             "(scale blocks along K; other permutations are not representable)")
        return self.mT

    # ---- constructors ----
    @classmethod
    def from_parts(cls, qdata, scale, format, *, per_tensor_scale=None, orig_dtype=torch.bfloat16, quant_dim=-1):
        """Wrap already-quantised storage (checkpoints, external quantizers)."""
        return cls(qdata, scale, _coerce_format(format), per_tensor_scale, orig_dtype, quant_dim)

    @classmethod
    def quantize(cls, x: torch.Tensor, format, *, dim: int = -1,
                 per_tensor_scale: Optional[torch.Tensor] = None) -> "BlockScaledOperand":
        """Quantise a 2-D / 3-D bf16 / fp32 CUDA tensor along ``dim``: -1 (default) or -2 (the result equals
        quantising the transposed copy and viewing it back; 2-D inputs go through a kernel that transposes
        while it quantises, batched ones through a transposed copy).  One kernel launch writes codes and
        blocked scale factors."""
        fmt = _coerce_format(format)
        if _normalize_quant_dim(dim, x.ndim) == -2:
            from .. import _ops
            rows = x.shape[-2]
            if (x.ndim == 2 and x.is_cuda and fmt.name in _ops._FMT_ID and rows % 32 == 0
                    and (rows * (1 if fmt.elems_per_container == 1 else 0.5)) % 16 == 0):
                # one kernel reads x once and writes the codes of the transposed matrix and its blocked scales
                if per_tensor_scale is not None and not fmt.has_per_tensor_scale:
                    raise ValueError(f"{fmt.name} does not take a per_tensor_scale")
                pts = None if per_tensor_scale is None else per_tensor_scale.to(device=x.device, dtype=torch.float32).reshape(1)
                c, s = _ops.quantize_cols(x, _ops.format_id(fmt.name), pts)
                return cls(c.view(fmt.qdata_dtype), s.view(fmt.scale_dtype), fmt, pts, x.dtype, -1).mT
            return cls.quantize(x.transpose(-1, -2).contiguous(), fmt, per_tensor_scale=per_tensor_scale).mT
        if fmt.name not in QUANTIZERS:
            if fmt.name in BLOCKSCALED_FORMAT_REGISTRY:
                raise NotImplementedError(
                    f"quack_b200 has no sm_100a quantizer for {fmt.name} (implemented: {sorted(QUANTIZERS)}); "
                    "construct pre-quantized data via from_parts")
            raise NotImplementedError(f"no in-repo quantizer for {fmt.name}; construct pre-quantized data via from_parts")
        if per_tensor_scale is not None and not fmt.has_per_tensor_scale:
            raise ValueError(f"{fmt.name} does not take a per_tensor_scale")
        assert x.ndim in (2, 3), f"expected (M, K) or (L, M, K), got shape {tuple(x.shape)}"
        assert x.shape[-1] % fmt.sf_vec_size == 0, (
            f"K ({x.shape[-1]}) must be divisible by {fmt.sf_vec_size} for {fmt.name}")
        if not x.is_cuda:
            raise RuntimeError("BlockScaledOperand.quantize needs a CUDA tensor: quack_b200 has no CPU quantizer")
        batched = x.ndim == 3
        l, mn, k = x.shape if batched else (1, *x.shape)
        pts = None
        if per_tensor_scale is not None:
            pts = per_tensor_scale.to(device=x.device, dtype=torch.float32).reshape(1)
        if not batched or mn % 128 == 0:
            # one launch: with mn a multiple of 128 no scale atom straddles two batch entries
            c, s = quantize_to_blocked(x.reshape(l * mn, k), fmt.name, pts)
            q = c.reshape(*x.shape[:-1], -1)
            sf = s.reshape(l, -1, *s.shape[1:]) if batched else s
        else:
            parts = [quantize_to_blocked(x[i], fmt.name, pts) for i in range(l)]
            q, sf = torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts])
        return cls(q.view(fmt.qdata_dtype), sf.view(fmt.scale_dtype), fmt, pts, x.dtype, -1)

    def to_packed(self) -> "BlockScaledOperand":
        """Canonical packed operands are returned unchanged; byte-container formats have no
        repacking kernel here."""
        if not self.format.is_byte_container:
            return self
        raise NotImplementedError(f"no repacking kernel for {self.format.name} in quack_b200")

    def dequantize(self, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """codes x scales (x per-tensor scale) as a plain tensor (torch ops; a test helper)."""
        from .quantize import dequant_operand, unpack_scale_blocked_to_2d

        fmt = self.format
        mn_dim, k_dim = self._mn_k_dims()
        q = self.qdata if k_dim == self.ndim - 1 else self.qdata.transpose(mn_dim, k_dim)
        batched = self.ndim == 3
        vals = dequant_operand(q if batched else q.unsqueeze(0), fmt)
        l, mn, k = vals.shape
        scale = self.scale if self.scale.ndim == 6 else self.scale.unsqueeze(0)
        sf_k = -(-k // fmt.sf_vec_size)
        expect = (l, -(-mn // 128), -(-sf_k // 4), 32, 4, 4)
        if tuple(scale.shape) != expect:
            raise ValueError("dequantize requires dense scale factors matching qdata; "
                             f"got {tuple(scale.shape)}, expected {expect}. Padded varlen scale buffers require "
                             "sequence offsets, which BlockScaledOperand does not carry")
        sf2d = unpack_scale_blocked_to_2d(scale.contiguous(), mn, sf_k).float()
        out = vals * sf2d.repeat_interleave(fmt.sf_vec_size, dim=-1)[..., :k]
        if self.per_tensor_scale is not None:
            out = out * self.per_tensor_scale
        if not batched:
            out = out.squeeze(0)
        if k_dim != self.ndim - 1:
            out = out.transpose(mn_dim, k_dim)
        return out.to(self.dtype if dtype is None else dtype)

    def _map(self, fn) -> "BlockScaledOperand":
        return dataclasses.replace(self, qdata=fn(self.qdata), scale=fn(self.scale),
                                   per_tensor_scale=None if self.per_tensor_scale is None else fn(self.per_tensor_scale))

    def to(self, device, non_blocking: bool = False) -> "BlockScaledOperand":
        if isinstance(device, torch.dtype):
            raise TypeError(f"BlockScaledOperand.to({device}): dtype conversion of quantized storage is not "
                            "supported; call .dequantize(dtype) explicitly")
        return self._map(lambda t: t.to(device, non_blocking=non_blocking))

    def clone(self) -> "BlockScaledOperand":
        return self._map(lambda t: t.clone())

    def __deepcopy__(self, memo):
        return self._map(lambda t: _copy.deepcopy(t, memo))

    def __repr__(self):
        pts = "" if self.per_tensor_scale is None else f", per_tensor_scale={self.per_tensor_scale}"
        return (f"BlockScaledOperand(format={self.format.name}, shape={self.shape}, quant_dim={self.quant_dim}, "
                f"dtype={self.dtype}, qdata={self.qdata.dtype}{tuple(self.qdata.shape)}, "
                f"scale={tuple(self.scale.shape)}{pts}, device={self.device})")


# ---- pytree: the container crosses functional transforms as (qdata, scale, pts) leaves ----
_CTX_VERSION = 1


def _dt_name(dt: torch.dtype) -> str:
    return str(dt).removeprefix("torch.")


def _dt_from(name) -> torch.dtype:
    if isinstance(name, torch.dtype):
        return name
    if not isinstance(name, str):
        raise TypeError(f"invalid serialized torch dtype {name!r}")
    dt = getattr(torch, name.removeprefix("torch."), None)
    if not isinstance(dt, torch.dtype):
        raise ValueError(f"unknown serialized torch dtype {name!r}")
    return dt


def _fmt_ctx(fmt: BlockScaledFormat) -> dict:
    d = {f: getattr(fmt, f, None) for f in _FIELD_ORDER}
    d["qdata_dtype"], d["scale_dtype"] = _dt_name(fmt.qdata_dtype), _dt_name(fmt.scale_dtype)
    return d


def _fmt_from_ctx(ctx: dict) -> BlockScaledFormat:
    if not isinstance(ctx, dict):
        raise TypeError(f"invalid serialized BlockScaledFormat context {ctx!r}")
    kw = {f: ctx.get(f) for f in _FIELD_ORDER}
    kw["qdata_dtype"], kw["scale_dtype"] = _dt_from(ctx["qdata_dtype"]), _dt_from(ctx["scale_dtype"])
    fmt = BlockScaledFormat(**kw)
    reg = BLOCKSCALED_FORMAT_REGISTRY.get(fmt.name)
    return reg if reg == fmt else fmt


def _flatten(op: BlockScaledOperand):
    return (op.qdata, op.scale, op.per_tensor_scale), {
        "version": _CTX_VERSION, "format": _fmt_ctx(op.format), "orig_dtype": _dt_name(op.orig_dtype),
        "quant_dim": op.quant_dim}


def _unflatten(children, ctx):
    qdata, scale, pts = children
    if isinstance(ctx, dict):
        if ctx.get("version") != _CTX_VERSION:
            raise ValueError(f"unsupported BlockScaledOperand pytree context version {ctx.get('version')!r}")
        fmt, odt, qd = _fmt_from_ctx(ctx["format"]), _dt_from(ctx["orig_dtype"]), ctx["quant_dim"]
    else:  # legacy (format name | descriptor, dtype, quant_dim) triple
        if not isinstance(ctx, (tuple, list)) or len(ctx) != 3:
            raise TypeError(f"invalid legacy BlockScaledOperand pytree context {ctx!r}")
        f, odt, qd = ctx
        fmt = f if isinstance(f, BlockScaledFormat) else BlockScaledFormat.from_name(f)
        odt = _dt_from(odt)
    return BlockScaledOperand(qdata, scale, fmt, pts, odt, qd)


_pytree.register_pytree_node(
    BlockScaledOperand, _flatten, _unflatten,
    serialized_type_name="quack_b200.blockscaled.operand.BlockScaledOperand",
    to_dumpable_context=lambda c: c, from_dumpable_context=lambda c: c)

torch.serialization.add_safe_globals([BlockScaledOperand, BlockScaledFormat])
