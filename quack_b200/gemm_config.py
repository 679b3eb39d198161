"""Tile configuration of the block-scaled GEMM (``quack/gemm_config.py`` in the reference:
``GemmConfig`` :36-54, ``cta_tile_shape_m`` :57-68, ``blockscaled_config_ok`` :71-95,
``blockscaled_default_config`` :288-314).  The kernels here are compiled ahead of time for a
fixed set of tile shapes, so a config names one of them instead of driving a JIT."""

from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum
from functools import lru_cache
from typing import Optional


class SplitKMode(IntEnum):
    SERIAL = 0
    PARALLEL = 1
    SEPARATE = 2


@dataclass(frozen=True)
class GemmConfig:
    tile_m: int = 128
    tile_n: int = 192
    tile_k: Optional[int] = None
    num_warps: Optional[int] = None
    pingpong: bool = True
    is_dynamic_persistent: bool = True
    cluster_m: int = 2
    cluster_n: int = 1
    cluster_k: int = 1
    split_k: int = 1
    swap_ab: bool = False
    max_swizzle_size: int = 8
    device_capacity: int = 10
    use_tma_gather: bool = False


# (tile_n, CTAs per MMA) pairs with a compiled kernel
COMPILED_TILES = {(64, 1), (128, 1), (256, 1), (128, 2), (192, 2), (256, 2)}


def cta_tile_shape_m(tile_m: int, cluster_m: int, device_capacity: int = 10, blockscaled: bool = False) -> int:
    """Rows per CTA: an even cluster_m with a 256-row MMA tile (128 too when not block-scaled)
    splits the tile across a CTA pair."""
    if device_capacity not in (10, 11) or cluster_m % 2:
        return tile_m
    return tile_m // 2 if tile_m in ((256,) if blockscaled else (128, 256)) else tile_m


def blockscaled_config_ok(c: GemmConfig) -> bool:
    """Hardware constraints of the tcgen05 block-scaled MMA path (reference :71-95)."""
    return (c.device_capacity in (10, 11) and not c.swap_ab and c.tile_k is None and c.tile_m in (128, 256)
            and c.tile_n % 64 == 0 and 64 <= c.tile_n <= 256 and c.cluster_m <= 4 and c.cluster_n <= 4)


def config_to_kernel(c: GemmConfig):
    """(tile_n, cta_group) of the compiled kernel that implements ``c``; ValueError if the
    config is legal for the hardware but was not compiled into this library."""
    if not blockscaled_config_ok(c):
        raise ValueError(f"config {c} is not valid for a block-scaled GEMM")
    cg = 2 if (c.tile_m == 256 and c.cluster_m % 2 == 0) else 1
    if c.tile_m == 256 and cg == 1:
        raise ValueError("tile_m=256 needs an even cluster_m (the MMA tile spans a CTA pair)")
    if c.cluster_n != 1 or c.cluster_m not in (1, 2):
        raise ValueError("quack_b200 kernels use clusters (1,1) or (2,1): no operand multicast")
    if (c.tile_n, cg) not in COMPILED_TILES:
        raise ValueError(f"no compiled kernel for tile_n={c.tile_n} with {cg} CTA(s) per MMA; "
                         f"available: {sorted(COMPILED_TILES)}")
    return c.tile_n, cg


@lru_cache(maxsize=None)
def _blockscaled_config(tile_m, tile_n, cluster, device_capacity=10, pingpong=False):
    return GemmConfig(tile_m=tile_m, tile_n=tile_n, cluster_m=cluster[0], cluster_n=cluster[1], pingpong=pingpong,
                      is_dynamic_persistent=False, device_capacity=device_capacity)


def blockscaled_default_config(m: int, n: int, device_capacity: int = 10) -> GemmConfig:
    """The reference's rule (:308-314): large problems use a 256-row MMA tile on a CTA pair."""
    if m >= 512 and n >= 256:
        return _blockscaled_config(256, 256, (2, 1))
    if m >= 512 and n >= 128:
        return _blockscaled_config(256, 128, (2, 1))
    return _blockscaled_config(128, 128, (1, 1))
