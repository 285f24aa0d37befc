"""ctypes binding of libw4a4_sm100.so (the C ABI in include/w4a4_sm100.h).

The library is built in-tree by ``pi05_pytorch_fast_b200.build`` (``nvcc`` for
sm_100a).  There is no fallback: if the library is missing every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_NAME = "libw4a4_sm100.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

W4A4_OK = 0
W4A4_ERR_INVALID = 1
W4A4_ERR_UNSUPPORTED = 2
W4A4_ERR_CUDA = 3

STAGING_FP16 = 0
STAGING_FP32 = 1
CODES_INT8 = 0
CODES_PACKED = 1
CODES_GEMM = 2
LAYOUT_ROW_MAJOR = 0
LAYOUT_FRAGMENT_MAJOR = 1
LAYOUT_INT8 = 2
ROTATE_BY_K = -1
GEMM_SINGLE_CTA = 0
GEMM_CTA_PAIR = 1
GEMM_NO_SPLIT = 2
GEMM_SPLIT_K = 3
ATTN_MAX_SEQ = 4096
NOALLOC_MAX_ROWS = 65536
NOALLOC_MAX_CODES = 16 * 1024 * 1024

# Every symbol include/w4a4_sm100.h declares.
EXPORTED_SYMBOLS = (
    "w4a4_quant",
    "w4a4_gemm",
    "w4a4_gemm_accumulators",
    "w4a4_int4_gemm",
    "w4a4_int4_gemm_noalloc",
    "w4a4_rmsnorm_quant",
    "w4a4_geglu_quant",
    "w4a4_prefix_tables",
    "w4a4_rope",
    "w4a4_prefix_attention",
    "w4a4_geglu",
    "w4a4_quant_segments",
    "w4a4_pad_rows",
    "w4a4_repack_int8",
    "w4a4_pack_weight",
    "w4a4_ada_rms_norm_bf16",
    "w4a4_rope_qk_bf16",
    "w4a4_layer_norm_bf16",
    "w4a4_last_error",
    "w4a4_device_error",
    "w4a4_set_wait_limit_ns",
    "w4a4_set_gemm_variant",
    "w4a4_gemm_plan",
    "w4a4_selftest_wait_timeout",
    "w4a4_version",
)


class W4A4Weight(ctypes.Structure):
    """Mirror of ``w4a4_weight``."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("n", ctypes.c_int32),
        ("row_words", ctypes.c_int32),
        ("layout", ctypes.c_int32),
    ]


_lib = None
_lock = threading.Lock()


class W4A4Error(RuntimeError):
    """An error status returned by the native library."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def _declare(lib: ctypes.CDLL) -> None:
    c_i32, c_i64, c_u64, vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_void_p
    lib.w4a4_quant.argtypes = [vp, c_i64, c_i32, c_i64, c_i32, c_i32, c_i32, vp, vp, vp]
    lib.w4a4_gemm.argtypes = [vp, vp, c_i64, c_i32, c_i32, ctypes.POINTER(W4A4Weight),
                              ctypes.POINTER(vp), vp]
    lib.w4a4_gemm_accumulators.argtypes = [vp, c_i64, c_i32, c_i32, ctypes.POINTER(W4A4Weight),
                                           ctypes.POINTER(vp), vp]
    lib.w4a4_int4_gemm.argtypes = [vp, c_i64, c_i32, c_i64, c_i32, c_i32, c_i32,
                                   ctypes.POINTER(W4A4Weight), ctypes.POINTER(vp), vp, vp, vp]
    lib.w4a4_int4_gemm_noalloc.argtypes = [vp, c_i64, c_i32, c_i64, c_i32, c_i32, c_i32,
                                           ctypes.POINTER(W4A4Weight), ctypes.POINTER(vp), vp]
    lib.w4a4_rmsnorm_quant.argtypes = [vp, c_i64, vp, c_i64, vp, ctypes.c_float, vp, c_i64, vp,
                                       c_i64, c_i64, c_i32, c_i32, c_i32, vp, vp, vp]
    lib.w4a4_geglu_quant.argtypes = [vp, vp, c_i64, c_i32, c_i64, c_i32, c_i32, vp, vp, vp, c_i64, vp]
    lib.w4a4_prefix_tables.argtypes = [vp, c_i32, c_i32, vp, c_i32, vp, vp, vp, vp, vp]
    lib.w4a4_rope.argtypes = [vp, c_i64, vp, c_i64, vp, vp, c_i64, c_i32, vp]
    lib.w4a4_prefix_attention.argtypes = [vp, c_i64, vp, c_i64, vp, c_i64, vp, vp, c_i32, c_i32, c_i32,
                                          vp, vp, c_i64, vp, vp, vp, c_i64, vp]
    lib.w4a4_geglu.argtypes = [vp, vp, c_i64, c_i32, c_i64, vp, c_i64, vp]
    lib.w4a4_quant_segments.argtypes = [vp, c_i64, c_i32, c_i32, c_i64, c_i64, c_i32, c_i32, vp, vp, vp]
    lib.w4a4_pad_rows.argtypes = [vp, c_i32, c_i32, c_i32, vp, vp]
    lib.w4a4_repack_int8.argtypes = [vp, c_i32, vp, vp]
    lib.w4a4_pack_weight.argtypes = [vp, c_i32, c_i64, c_i32, c_i32, c_i32, c_i32, vp, c_i32, vp]
    lib.w4a4_ada_rms_norm_bf16.argtypes = [vp, vp, c_i64, c_i32, c_i32, vp, vp, c_i64, ctypes.c_float, vp]
    lib.w4a4_rope_qk_bf16.argtypes = [vp, c_i64, c_i32, vp, c_i64, c_i32, vp, vp, c_i64, c_i32, vp]
    lib.w4a4_layer_norm_bf16.argtypes = [vp, vp, c_i64, c_i32, vp, vp, ctypes.c_float, vp]
    lib.w4a4_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    lib.w4a4_device_error.argtypes = [ctypes.POINTER(ctypes.c_uint32), c_i32]
    lib.w4a4_set_wait_limit_ns.argtypes = [c_u64]
    lib.w4a4_set_gemm_variant.argtypes = [c_i32]
    lib.w4a4_gemm_plan.argtypes = [c_i64, c_i32, c_i32, ctypes.POINTER(c_i32), c_i32, c_i32,
                                   c_i32, ctypes.POINTER(c_i32)]
    lib.w4a4_selftest_wait_timeout.argtypes = [c_u64, vp]
    lib.w4a4_version.argtypes = []
    for name in EXPORTED_SYMBOLS:
        getattr(lib, name).restype = ctypes.c_int


def lib() -> ctypes.CDLL:
    """The loaded native library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.isfile(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_NAME} is not built (expected at {LIB_PATH}); run "
                    "`python -m pi05_pytorch_fast_b200.build`. The W4A4 path has no CPU fallback."
                )
            handle = ctypes.CDLL(LIB_PATH)
            _declare(handle)
            _lib = handle
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().w4a4_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


def check(status: int) -> None:
    """Raise the library's message as a RuntimeError on a non-zero status."""
    if status != W4A4_OK:
        raise W4A4Error(status, last_error())


def device_error(clear: bool = False) -> int:
    """Device error word of the current device (synchronises the device)."""
    bits = ctypes.c_uint32(0)
    check(lib().w4a4_device_error(ctypes.byref(bits), 1 if clear else 0))
    return bits.value


def set_wait_limit_ns(limit_ns: int) -> None:
    check(lib().w4a4_set_wait_limit_ns(int(limit_ns)))


def set_gemm_variant(variant: int) -> None:
    """GEMM_SINGLE_CTA (default, split-K where faster), GEMM_CTA_PAIR,
    GEMM_NO_SPLIT or GEMM_SPLIT_K for launches after this call."""
    check(lib().w4a4_set_gemm_variant(int(variant)))


def gemm_plan(m: int, k: int, ns, sms: int = 148, variant: int = GEMM_SINGLE_CTA,
              layout: int = LAYOUT_ROW_MAJOR) -> dict:
    """The launch shape w4a4_gemm would choose (host computation, no GPU)."""
    n_arr = (ctypes.c_int32 * len(ns))(*ns)
    out = (ctypes.c_int32 * 6)()
    check(lib().w4a4_gemm_plan(m, k, len(ns), n_arr, sms, variant, layout, out))
    return {"tok_tile": out[0], "split": bool(out[1]), "grid": out[2], "tok_tiles": out[3],
            "tok_group": out[4], "w_tiles": out[5]}


def attn_vt_stride(seq: int) -> int:
    """Row stride (elements) of the V^T scratch of w4a4_prefix_attention."""
    return (seq + 7) // 8 * 8


def weights_array(descs) -> ctypes.Array:
    arr = (W4A4Weight * len(descs))()
    for i, (ptr, n, row_words, layout) in enumerate(descs):
        arr[i].data = ptr
        arr[i].n = n
        arr[i].row_words = row_words
        arr[i].layout = layout
    return arr


def pointer_array(ptrs) -> ctypes.Array:
    arr = (ctypes.c_void_p * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = p
    return arr
