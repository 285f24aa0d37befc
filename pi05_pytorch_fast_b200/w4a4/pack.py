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

Weight packing runs on the CPU in fp32, as the reference's does, so packed
checkpoints are bit-identical to the reference's.  None of this is on the
inference path; the GEMM reads these layouts directly on the GPU.
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


def pack_linear_weight(weight: torch.Tensor, rotate: bool | None = None,
                       device: torch.device | str = "cpu") -> torch.Tensor:
    """Linear.weight [N, K] -> int32 [N, K/8 + 1], computed in fp32 on ``device``
    (CPU by default, as the reference packs).  Divisions are tensor/tensor so
    that a CUDA pack is bit-identical to the CPU pack."""
    if weight.dim() != 2:
        raise ValueError(f"expected 2D weight, got {tuple(weight.shape)}")
    n, k = weight.shape
    if k % 64 != 0:
        raise ValueError(f"K must be a multiple of 64 for gemm_iu4, got {k}")
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
