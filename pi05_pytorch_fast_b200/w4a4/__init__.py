"""B200 W4A4 ops behind the reference's ``pi05_fast.w4a4`` op interface.

Importing registers the five ``pi05_w4a4::*`` custom ops on the sm_100a
kernels.  The reference's own model glue (``pi05_fast/w4a4/linear.py``,
``apply.py``) then runs unmodified on them; this package's own caller of
the path is ``pi05_pytorch_fast_b200.prefix_lm``.
"""

from .extension import (
    int4_gemm,
    int4_gemm2,
    int4_gemm2_tiled,
    int4_gemm3,
    int4_gemm_tiled,
    preload,
)
from .pack import pack_linear_weight, preshuffle_wmma_weight

__all__ = [
    "pack_linear_weight",
    "preshuffle_wmma_weight",
    "int4_gemm",
    "int4_gemm_tiled",
    "int4_gemm2",
    "int4_gemm2_tiled",
    "int4_gemm3",
    "preload",
]
