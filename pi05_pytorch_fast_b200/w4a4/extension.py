"""``pi05_w4a4::*`` PyTorch custom ops on the B200 W4A4 path.

Same op names, schemas, fake (meta) implementations, Python wrappers and
error messages as the reference's ``pi05_fast/w4a4/extension.py:78-178``
(argument checks follow ``pi05_fast/w4a4/csrc/int4_gemm.cu:487-501, :570-577``),
but every op runs the sm_100a kernels of ``libw4a4_sm100.so``: the schemas
and fakes are registered here, the op bodies are C++ (``_w4a4_ops.so``, built
from ``csrc/torch_ops.cpp``) calling the library's C ABI.  There is no CPU
path: CPU tensors raise, a missing library raises.

Importing this module before the reference's ``pi05_fast.w4a4.extension``
makes the reference's ``_register_custom_op`` see the ops as registered
(extension.py:82-87), so the reference's ``apply.py`` / ``linear.py`` call
these kernels unmodified.

Environment:
  PI05_W4A4_STAGING = fp16 (default) | fp32
      fp16: the activation FWHT rounds to fp16 like the reference HIP kernel
            (int4_gemm.cu:404-426);
      fp32: all-fp32 FWHT like the reference CPU emulation (pack.py:113-131).
"""

from __future__ import annotations

import os
import warnings

import torch

from .. import _native as nat

STAGING_ENV = "PI05_W4A4_STAGING"

_op_registered = False
_warned_pad = False


def staging_mode() -> int:
    """The FWHT staging selected by PI05_W4A4_STAGING."""
    v = os.environ.get(STAGING_ENV, "fp16").strip().lower()
    if v in ("fp16", ""):
        return nat.STAGING_FP16
    if v == "fp32":
        return nat.STAGING_FP32
    raise RuntimeError(f"{STAGING_ENV} must be 'fp16' or 'fp32', got {v!r}")


def _check_activation(x: torch.Tensor) -> int:
    if not x.is_cuda:
        raise RuntimeError("int4_gemm expects CUDA/HIP tensors")
    if x.dtype != torch.float16:
        raise RuntimeError("int4_gemm activations must be float16")
    if x.dim() == 0 or x.size(-1) <= 0:
        raise RuntimeError("int4_gemm activations need a non-empty last dimension")
    k = int(x.size(-1))
    if k % 64 != 0:
        raise RuntimeError(f"K must be a multiple of 64, got {k}")
    return k


def _check_packed(w: torch.Tensor, k: int, device: torch.device) -> None:
    if not w.is_cuda:
        raise RuntimeError("packed W must be on CUDA/HIP")
    if w.dtype != torch.int32 or w.dim() != 2:
        raise RuntimeError("packed W must be int32 [N, K/8+1]")
    if w.size(1) < k // 8 + 1:
        raise RuntimeError("packed W second dim must contain K/8 packed words plus a scale")
    if w.device != device:
        raise RuntimeError(f"packed W is on {w.device} but the activations are on {device}")


def pad_rows_cuda(w: torch.Tensor, row_words: int) -> torch.Tensor:
    """Row-major packed weight [N, R] -> [N, row_words] with zero words appended
    (the load-time pad of apply.py:68-69), on the device."""
    if w.size(1) > row_words:
        raise ValueError("row_words must not shrink the rows")
    out = torch.empty((w.size(0), row_words), dtype=torch.int32, device=w.device)
    w = w.contiguous()
    with torch.cuda.device(w.device):
        stream = torch.cuda.current_stream(w.device).cuda_stream
        nat.check(nat.lib().w4a4_pad_rows(w.data_ptr(), w.size(0), w.size(1), row_words,
                                          out.data_ptr(), stream))
    return out


def _prepare_row_major(w: torch.Tensor) -> torch.Tensor:
    """The GEMM streams weights with TMA, whose row stride must be a multiple of
    16 bytes.  The reference's default load path already pads rows to K/8+8
    (apply.py:51, :68-69); other strides are padded here, per call."""
    global _warned_pad
    w = w.contiguous()
    if (w.size(1) * 4) % 16 == 0:
        return w
    if not _warned_pad:
        warnings.warn(
            "pi05_w4a4: packed weight row stride is not a multiple of 4 words; padding it on every "
            "call. Pad once at load (PI05_W4A4_ROW_PAD_WORDS=8, the default) to avoid the copy.",
            stacklevel=3,
        )
        _warned_pad = True
    return pad_rows_cuda(w, (w.size(1) + 3) // 4 * 4)


def _fake_out(x: torch.Tensor, packed: torch.Tensor) -> torch.Tensor:
    return torch.empty(*x.shape[:-1], packed.shape[0], device=x.device, dtype=torch.float16)


def _ops_exist() -> bool:
    try:
        torch.ops.pi05_w4a4.int4_gemm2_tiled  # noqa: B018
        return True
    except (AttributeError, RuntimeError):
        return False


# The op library; kept alive for the life of the process.
_library = None
# Raising stubs, registered while the C++ op library is not built; dropped
# before that library registers the real bodies.
_stub_library = None
_ops_loaded = False

# name, schema arguments / returns, fake implementation
_OPS = (
    ("int4_gemm", "(Tensor x, Tensor packed) -> Tensor",
     lambda x, packed: _fake_out(x, packed)),
    ("int4_gemm_tiled", "(Tensor x, Tensor packed) -> Tensor",
     lambda x, packed: _fake_out(x, packed)),
    ("int4_gemm2", "(Tensor x, Tensor w0, Tensor w1) -> (Tensor, Tensor)",
     lambda x, w0, w1: (_fake_out(x, w0), _fake_out(x, w1))),
    ("int4_gemm2_tiled", "(Tensor x, Tensor w0, Tensor w1) -> (Tensor, Tensor)",
     lambda x, w0, w1: (_fake_out(x, w0), _fake_out(x, w1))),
    ("int4_gemm3", "(Tensor x, Tensor w0, Tensor w1, Tensor w2) -> (Tensor, Tensor, Tensor)",
     lambda x, w0, w1, w2: (_fake_out(x, w0), _fake_out(x, w1), _fake_out(x, w2))),
)

OPS_LIB_NAME = "_w4a4_ops.so"
OPS_LIB_PATH = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), OPS_LIB_NAME)


def _not_built(*_args):
    raise RuntimeError(
        f"{OPS_LIB_NAME} is not built (expected at {OPS_LIB_PATH}); run "
        "`python -m pi05_pytorch_fast_b200.build`. The W4A4 path has no CPU fallback.")


def _load_ops() -> bool:
    """Loads the C++ op bodies (csrc/torch_ops.cpp, registered under
    CompositeExplicitAutograd) if the library is built; they replace the
    not-built stubs."""
    global _ops_loaded, _stub_library
    if not _ops_loaded and os.path.isfile(OPS_LIB_PATH):
        if _stub_library is not None:
            _stub_library._destroy()
            _stub_library = None
        torch.ops.load_library(OPS_LIB_PATH)
        _ops_loaded = True
    return _ops_loaded


def _register_custom_op() -> None:
    """Registers the five pi05_w4a4 ops with the reference's schemas (the
    schemas torch.library.custom_op(..., mutates_args=()) gives them,
    extension.py:92-138) and fake implementations for tracing.  The op
    bodies are C++ (_w4a4_ops.so): checks, output allocation and the call
    into libw4a4_sm100.so cost about 2 us of host time per op.  Without that
    library every op raises."""
    global _op_registered, _library, _stub_library
    if _op_registered:
        return
    if _ops_exist():
        raise RuntimeError(
            "pi05_w4a4 ops are already registered by another backend. Import "
            "pi05_pytorch_fast_b200 before pi05_fast.w4a4.extension so the B200 kernels serve them."
        )
    lib = torch.library.Library("pi05_w4a4", "DEF")
    for name, schema, fake in _OPS:
        lib.define(name + schema)
        torch.library.register_fake("pi05_w4a4::" + name, fake, lib=lib)
    _library = lib
    _op_registered = True
    if not _load_ops():
        _stub_library = torch.library.Library("pi05_w4a4", "IMPL")
        for name, _, _ in _OPS:
            _stub_library.impl(name, _not_built, "CompositeExplicitAutograd")


_register_custom_op()


def int4_gemm(x: torch.Tensor, packed_w: torch.Tensor) -> torch.Tensor:
    """W4A4 GEMM. x: fp16 [..., K]; packed_w: int32 [N, K/8+1 (+pad)] -> fp16 [..., N]."""
    return torch.ops.pi05_w4a4.int4_gemm(x, packed_w)


def int4_gemm_tiled(x: torch.Tensor, packed_w: torch.Tensor) -> torch.Tensor:
    """W4A4 GEMM with fragment-major weights [N, K/8+9]."""
    return torch.ops.pi05_w4a4.int4_gemm_tiled(x, packed_w)


def int4_gemm2(x: torch.Tensor, w0: torch.Tensor, w1: torch.Tensor):
    """One shared activation quant, two GEMMs (one launch)."""
    return torch.ops.pi05_w4a4.int4_gemm2(x, w0, w1)


def int4_gemm2_tiled(x: torch.Tensor, w0: torch.Tensor, w1: torch.Tensor):
    """One shared activation quant, two fragment-major GEMMs (one launch)."""
    return torch.ops.pi05_w4a4.int4_gemm2_tiled(x, w0, w1)


def int4_gemm3(x: torch.Tensor, w0: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor):
    """One shared activation quant, three GEMMs (one launch)."""
    return torch.ops.pi05_w4a4.int4_gemm3(x, w0, w1, w2)


def preload() -> None:
    """Load the native libraries up front (the reference JIT-compiles here)."""
    nat.lib()
    _register_custom_op()
    if not _load_ops():
        _not_built()


# ---------------------------------------------------------------------------
# Lower-level entry points (used by tests and the benchmark)
# ---------------------------------------------------------------------------
_CODE_FORMATS = {"int8": nat.CODES_INT8, "packed": nat.CODES_PACKED, "gemm": nat.CODES_GEMM}
# Byte order of each group of 8 codes in the GEMM format (include/w4a4_sm100.h).
GEMM_GROUP_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)


def to_gemm_order(codes: torch.Tensor) -> torch.Tensor:
    """int8 codes [..., K] in natural order -> the GEMM's byte order."""
    k = codes.shape[-1]
    idx = torch.tensor(GEMM_GROUP_ORDER, device=codes.device)
    return codes.reshape(*codes.shape[:-1], k // 8, 8).index_select(-1, idx).reshape(codes.shape).contiguous()


def quantize(x: torch.Tensor, staging: int | None = None, fmt: str = "int8",
             rotate: int = nat.ROTATE_BY_K) -> tuple[torch.Tensor, torch.Tensor]:
    """Activation codes of x [..., K] and row scales fp32 [M].  ``fmt``:
    "int8" (natural order int8 [M, K]), "gemm" (int8 [M, K] in the GEMM's
    byte order) or "packed" (the reference's int32 words [M, K/8])."""
    k = _check_activation(x)
    x2 = x.contiguous()
    if x2.data_ptr() % 16:
        x2 = x2.clone()
    m = x2.numel() // k
    dev = x.device
    with torch.cuda.device(dev):
        if fmt == "packed":
            codes = torch.empty((m, k // 8), dtype=torch.int32, device=dev)
        else:
            codes = torch.empty((m, k), dtype=torch.int8, device=dev)
        scales = torch.empty((m,), dtype=torch.float32, device=dev)
        st = staging_mode() if staging is None else staging
        nat.check(nat.lib().w4a4_quant(
            x2.data_ptr(), m, k, k, rotate, st, _CODE_FORMATS[fmt],
            codes.data_ptr(), scales.data_ptr(), torch.cuda.current_stream(dev).cuda_stream))
    return codes, scales


def gemm_from_codes(codes: torch.Tensor, scales: torch.Tensor, weights, fragment_major=False):
    """GEMM of int8 codes [M, K] in the GEMM byte order (``quantize(fmt="gemm")``)
    + scales [M] against 1..3 packed weights."""
    if codes.dim() != 2 or codes.dtype != torch.int8 or not codes.is_contiguous():
        raise ValueError("gemm_from_codes: codes must be a contiguous int8 [M, K] tensor")
    m, k = codes.shape
    if (scales.dtype != torch.float32 or scales.numel() != m or not scales.is_contiguous()
            or scales.device != codes.device):
        raise ValueError("gemm_from_codes: scales must be a contiguous fp32 [M] tensor on the codes' device")
    layout = nat.LAYOUT_FRAGMENT_MAJOR if fragment_major else nat.LAYOUT_ROW_MAJOR
    dev = codes.device
    with torch.cuda.device(dev):
        ws = [w.contiguous() if fragment_major else _prepare_row_major(w) for w in weights]
        ys = [torch.empty((m, int(w.size(0))), dtype=torch.float16, device=dev) for w in ws]
        descs = nat.weights_array(
            [(w.data_ptr(), int(w.size(0)), int(w.size(1)), layout) for w in ws])
        outs = nat.pointer_array([y.data_ptr() for y in ys])
        nat.check(nat.lib().w4a4_gemm(codes.data_ptr(), scales.data_ptr(), m, k, len(ws), descs,
                                      outs, torch.cuda.current_stream(dev).cuda_stream))
    return ys
