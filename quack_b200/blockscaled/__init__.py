"""Block-scaled (MXFP8 / NVFP4) operand support: format descriptors, the operand container,
CUDA quantizers and scale-layout helpers.  Mirrors ``quack.blockscaled`` of the reference;
formats without a B200 kernel in this package keep their descriptors (``from_parts`` works)
and raise ``NotImplementedError`` from ``quantize``."""

from .operand import (  # noqa: F401
    BLOCKSCALED_FORMAT_REGISTRY, MXFP4, MXFP4_BYTE, MXFP6_E2M3, MXFP6_E2M3_BYTE, MXFP6_E2M3_PACKED, MXFP6_E3M2,
    MXFP6_E3M2_BYTE, MXFP6_E3M2_PACKED, MXFP8_E4M3, MXFP8_E5M2, NVFP4, BlockScaledFormat, BlockScaledOperand,
    mma_kind_for_pair,
)
from .quantize import (  # noqa: F401
    nvfp4_per_tensor_scale, to_blocked, to_mx, to_mx_compiled, to_mx_dim0, to_mx_dim0_compiled, to_mx_e5m2, to_mxfp4, to_mxfp4_compiled, to_nvfp4,
    to_nvfp4_compiled,
)
from .utils import (  # noqa: F401
    BLOCKSCALED_FORMATS, blockscaled_gemm_reference, blockscaled_quantize, blockscaled_quantize_dim0, dequant_operand,
    pack_scale_2d_to_blocked_contig, scale_blocked_for_cublas, scale_view_for_kernel, unpack_scale_blocked_to_2d,
)
