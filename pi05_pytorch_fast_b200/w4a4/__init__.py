"""B200 W4A4 path behind the reference's ``pi05_fast.w4a4`` interface."""

from .extension import (
    int4_gemm,
    int4_gemm2,
    int4_gemm2_tiled,
    int4_gemm3,
    int4_gemm_tiled,
    preload,
)
from .linear import W4A4Linear
from .pack import pack_linear_weight, preshuffle_wmma_weight
from .apply import apply_w4a4_from_dir, maybe_apply_w4a4_from_env

__all__ = [
    "W4A4Linear",
    "apply_w4a4_from_dir",
    "maybe_apply_w4a4_from_env",
    "pack_linear_weight",
    "preshuffle_wmma_weight",
    "int4_gemm",
    "int4_gemm_tiled",
    "int4_gemm2",
    "int4_gemm2_tiled",
    "int4_gemm3",
    "preload",
]
