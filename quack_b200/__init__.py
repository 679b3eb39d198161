"""quack_b200: B200-native (sm_100a) block-scale quantizer, block-scaled GEMM with fused
epilogue and all-gather GEMM, behind the Python API of Dao-AILab/quack's quantised-linear
path (``quack.blockscaled``, ``quack.gemm_interface``, ``quack.gemm``, ``quack.distributed``).

All numerics run in hand-written CUDA kernels reached through the C ABI of
``libquack_b200.so`` (``include/quack_b200.h``).  There is no CPU or PyTorch fallback: if the
library is missing, importing this package raises.
"""

from . import _lib  # noqa: F401  (loads libquack_b200.so; raises when it is missing)
from .blockscaled import BlockScaledFormat, BlockScaledOperand  # noqa: F401
from .gemm import AllGatherArguments  # noqa: F401
from . import gemm, gemm_interface  # noqa: F401  (`quack_b200.gemm` is the kernel-level MODULE, as in the reference)

__version__ = "0.1.0"
