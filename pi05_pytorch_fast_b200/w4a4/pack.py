"""Packed W4A4 weight format (offline / load-time host code).

The on-disk and in-memory formats are the reference's, so checkpoints packed
by ``scripts/pack_w4a4_prefix.py`` load unchanged:

* row-major: int32 [N, K/8 + 1]; word p of row n holds k = 8p..8p+7 with
  element j at bits 4j..4j+3 (two's-complement nibbles); word K/8 holds the
  fp32 row scale's bits (pack.py:85-101);
* padded row-major: the same rows with extra zero words, e.g. K/8 + 8
  (apply.py:51, :68-69);
* fragment-major: payload flat as [K/16][N][2 words] followed by the N
  scales, declared [N, K/8 + 9] (pack.py:45-68).

Weight packing runs in fp32, on the CPU as the reference's does, or on the
GPU by this library's ``w4a4_pack_weight`` kernel (``pack_weight_cuda``); both
are bit-identical to the reference's pack.  None of this is on the inference
path; the GEMM reads these layouts directly on the GPU.
"""

from __future__ import annotations

import math
from typing import Any

import torch

ROTATE_K = frozenset({1024, 2048, 16384})
WMMA_PRESHUFFLE_PAD_WORDS = 9
DEFAULT_ROW_PAD_WORDS = 8


def should_rotate(k: int, rotate: bool | None = None) -> bool:
    """Hadamard rotation applies to K in {1024, 2048, 16384} unless overridden."""
    return bool(rotate) if rotate is not None else k in ROTATE_K


def fwht_unnormalized(x: torch.Tensor) -> torch.Tensor:
    """Unnormalised Walsh-Hadamard transform along the last dimension, fp32
    butterflies in ascending stride order."""
    n = x.shape[-1]
    if n <= 0 or n & (n - 1):
        raise ValueError(f"FWHT length must be a power of 2, got {n}")
    lead = x.shape[:-1]
    y = x.contiguous().clone().reshape(-1, n)
    h = 1
    while h < n:
        v = y.view(-1, n // (2 * h), 2, h)
        lo = v[:, :, 0, :].clone()
        hi = v[:, :, 1, :]
        v[:, :, 0, :] = lo + hi
        v[:, :, 1, :] = lo - hi
        h <<= 1
    return y.reshape(*lead, n)


def pack_nibbles(q: torch.Tensor) -> torch.Tensor:
    """int codes [..., K] in [-8, 7] -> int32 words [..., K/8]."""
    if q.shape[-1] % 8:
        raise ValueError(f"K must be a multiple of 8, got {q.shape[-1]}")
    g = (q.to(torch.int64) & 0xF).reshape(*q.shape[:-1], q.shape[-1] // 8, 8)
    shifts = torch.arange(0, 32, 4, dtype=torch.int64, device=q.device)
    words = (g << shifts).sum(dim=-1)
    return torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)


def unpack_nibbles(packed: torch.Tensor, k: int) -> torch.Tensor:
    """int32 words [..., K/8] -> int32 codes [..., K] in [-8, 7]."""
    w = packed.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(0, 32, 4, dtype=torch.int64, device=packed.device)
    nib = (w.unsqueeze(-1) >> shifts) & 0xF
    return torch.where(nib >= 8, nib - 16, nib).to(torch.int32).reshape(*packed.shape[:-1], k)


_PACK_DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def pack_weight_cuda(weight: torch.Tensor, layout: str = "row", row_words: int | None = None,
                     rotate: bool | None = None, device: torch.device | str | None = None) -> torch.Tensor:
    """Linear.weight [N, K] -> packed int32 on a CUDA device by the
    ``w4a4_pack_weight`` kernel, in its final layout: ``layout="row"`` gives
    [N, row_words] (default K/8 + 1; K/8 + 8 is the load-time pad), and
    ``"fragment"`` the fragment-major [N, K/8 + 9].  Bit-identical to
    ``pack_linear_weight`` (and its padding / preshuffle)."""
    from .. import _native as nat

    if weight.dim() != 2:
        raise ValueError(f"expected 2D weight, got {tuple(weight.shape)}")
    n, k = weight.shape
    dev = torch.device(device) if device is not None else weight.device
    if dev.type != "cuda":
        raise ValueError("pack_weight_cuda packs on a CUDA device")
    w = weight.detach()
    if w.dtype not in _PACK_DTYPES:
        w = w.float()
    w = w.to(dev)
    if w.stride(1) != 1:
        w = w.contiguous()
    if layout == "row":
        words = k // 8 + 1 if row_words is None else row_words
        lay = nat.LAYOUT_ROW_MAJOR
    elif layout == "fragment":
        words = k // 8 + WMMA_PRESHUFFLE_PAD_WORDS
        lay = nat.LAYOUT_FRAGMENT_MAJOR
    else:
        raise ValueError(f"unknown layout {layout!r}")
    out = torch.empty((n, words), dtype=torch.int32, device=dev)
    rot = nat.ROTATE_BY_K if rotate is None else int(bool(rotate))
    with torch.cuda.device(dev):
        nat.check(nat.lib().w4a4_pack_weight(w.data_ptr(), _PACK_DTYPES[w.dtype], w.stride(0), n, k, rot, lay,
                                             out.data_ptr(), words, torch.cuda.current_stream(dev).cuda_stream))
    return out


def pack_linear_weight(weight: torch.Tensor, rotate: bool | None = None,
                       device: torch.device | str = "cpu") -> torch.Tensor:
    """Linear.weight [N, K] -> int32 [N, K/8 + 1], computed in fp32 on ``device``
    (CPU by default, as the reference packs; a CUDA device runs the
    ``w4a4_pack_weight`` kernel)."""
    if weight.dim() != 2:
        raise ValueError(f"expected 2D weight, got {tuple(weight.shape)}")
    n, k = weight.shape
    if k % 64 != 0:
        raise ValueError(f"K must be a multiple of 64 for gemm_iu4, got {k}")
    if torch.device(device).type == "cuda":
        return pack_weight_cuda(weight, rotate=rotate, device=device)
    w = weight.detach().to(device=device, dtype=torch.float32)
    if should_rotate(k, rotate):
        w = fwht_unnormalized(w) * (1.0 / math.sqrt(k))
    amax = w.abs().amax(dim=-1).clamp_min(1e-12)
    scale = amax / torch.full_like(amax, 7.0)
    q = torch.round(w / scale[:, None]).clamp_(-7, 7)
    return torch.cat([pack_nibbles(q), scale.contiguous().view(torch.int32)[:, None]], dim=1)


def unpack_linear_weight(packed: torch.Tensor, k: int | None = None):
    """(codes int32 [N, K], scale fp32 [N], K) of a row-major packed weight."""
    n, row = packed.shape
    k = (row - 1) * 8 if k is None else k
    q = unpack_nibbles(packed[:, : k // 8], k)
    scale = packed[:, k // 8].contiguous().view(torch.float32)
    return q, scale, k


def pad_row_words(packed: torch.Tensor, row_words: int) -> torch.Tensor:
    """Append zero words so each row has ``row_words`` words."""
    extra = row_words - packed.shape[1]
    if extra < 0:
        raise ValueError("cannot shrink packed rows")
    if extra == 0:
        return packed
    return torch.nn.functional.pad(packed, (0, extra))


def preshuffle_wmma_weight(packed: torch.Tensor, k: int) -> torch.Tensor:
    """Row-major [N, >=K/8+1] -> fragment-major [N, K/8+9]."""
    if packed.dim() != 2:
        raise ValueError(f"expected 2D packed weight, got {tuple(packed.shape)}")
    n = packed.shape[0]
    words = k // 8
    if k % 16 != 0 or packed.shape[1] < words + 1:
        raise ValueError(f"invalid packed weight shape {tuple(packed.shape)} for K={k}")
    out = torch.zeros((n, words + WMMA_PRESHUFFLE_PAD_WORDS), dtype=packed.dtype,
                      device=packed.device)
    flat = out.view(-1)
    body = packed[:, :words].reshape(n, words // 2, 2).transpose(0, 1).reshape(-1)
    flat[: n * words] = body
    flat[n * words: n * words + n] = packed[:, words]
    return out


def layer_meta(name: str, packed: torch.Tensor, rotate: bool, has_bias: bool) -> dict[str, Any]:
    """meta.json entry of one packed layer (pack_w4a4_prefix.py:61-66 keys)."""
    n, row = packed.shape
    return {"name": name, "in_features": (row - 1) * 8, "out_features": n,
            "rotate": rotate, "has_bias": has_bias}
