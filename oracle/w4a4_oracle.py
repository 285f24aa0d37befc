"""CPU oracle for the W4A4 prefix-LM GEMM path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it.
The shipped path (``pi05_pytorch_fast_b200``) never calls into it and fails
loudly when its CUDA library is missing.

It restates, in numpy, the arithmetic of the reference project
(harrysocool/pi05-pytorch-fast; paths below are relative to that project):

* ``pi05_fast/w4a4/pack.py``        -- offline weight pack and the CPU emulation
  ``int4_gemm_ref`` (fp32 FWHT, per-token INT4 codes, exact integer GEMM).
* ``pi05_fast/w4a4/csrc/int4_gemm.cu`` -- the HIP kernel ``quant_rot_rb<K,R>``,
  whose FWHT keeps the first log2(R) butterfly stages in fp32 and rounds to
  fp16 after that stage and after every later stage ("fp16 staging").

Parity status
-------------
* ``staging="fp32"`` (the reference's ``quant_activation_cpu`` /
  ``int4_gemm_ref``) is PINNED: ``tests/test_oracle.py`` checks it bit-for-bit
  against golden vectors produced by running the unmodified reference code
  (``tests/golden/make_golden.py``).
* ``staging="fp16"`` (the reference's HIP ``quant_rot_rb``) is restated from
  ``int4_gemm.cu:396-449`` and PINNED to that kernel's own source:
  ``oracle/ref_quant`` compiles it from the reference checkout for host
  threads, and ``tests/test_oracle_ref_quant.py`` requires equal codes and
  row scales (where the checkout is present; the library lands in
  ``oracle/_ref``).  A second, loop-level restatement of the kernel's thread
  structure (``quant_rot_rb_loops``) cross-checks it too.
"""

from __future__ import annotations

import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

# Rotated K values: pack.py:14 (ROTATE_K); kernel dispatch int4_gemm.cu:520-527.
ROTATE_K = frozenset({1024, 2048, 16384})
# Fragment-major marker: pack.py:15 (WMMA_PRESHUFFLE_PAD_WORDS).
FRAGMENT_MAJOR_PAD_WORDS = 9
# Number of threads of the HIP quant kernel (int4_gemm.cu:35); R = K / 256.
_HIP_QUANT_THREADS = 256

F32 = np.float32
F16 = np.float16


def should_rotate(k: int, rotate: bool | None = None) -> bool:
    """pack.py:79-82."""
    if rotate is not None:
        return bool(rotate)
    return k in ROTATE_K


def inv_sqrt_k(k: int) -> np.float32:
    """fp32 constant 1/sqrt(K) as the reference's torch code forms it
    (a Python double rounded to fp32: pack.py:94, :122)."""
    return F32(1.0 / math.sqrt(k))


# ----------------------------------------------------------------------------
# Fast Walsh-Hadamard transforms
# ----------------------------------------------------------------------------
def fwht_fp32(x: np.ndarray) -> np.ndarray:
    """Unnormalised FWHT along the last axis, all butterflies in fp32, stages
    in ascending stride order h = 1, 2, 4, ... (pack.py:18-31)."""
    x = np.asarray(x, dtype=F32)
    n = x.shape[-1]
    if n <= 0 or n & (n - 1):
        raise ValueError(f"FWHT length must be a power of 2, got {n}")
    lead = x.shape[:-1]
    src = x.reshape(-1, n).copy()
    dst = np.empty_like(src)
    rows = src.shape[0]
    h = 1
    while h < n:
        v = src.reshape(rows, n // (2 * h), 2, h)
        o = dst.reshape(rows, n // (2 * h), 2, h)
        np.add(v[:, :, 0, :], v[:, :, 1, :], out=o[:, :, 0, :])
        np.subtract(v[:, :, 0, :], v[:, :, 1, :], out=o[:, :, 1, :])
        src, dst = dst, src
        h *= 2
    return src.reshape(*lead, n)


def fwht_fp16_staged(x: np.ndarray) -> np.ndarray:
    """FWHT as the HIP kernel computes it (int4_gemm.cu:396-426).

    With R = K/256 values per thread, the stages of stride 1 .. R/2 run in
    fp32 (:404-413); the result is rounded to fp16 (:415); every later stage
    adds/subtracts the fp16 values in fp32 and rounds the result to fp16
    (:417-426).  Returns fp32 arrays holding fp16-representable values."""
    x = np.asarray(x, dtype=F32)
    n = x.shape[-1]
    if n not in ROTATE_K:
        raise ValueError(f"fp16 staging is defined for K in {sorted(ROTATE_K)}, got {n}")
    r = n // _HIP_QUANT_THREADS
    lead = x.shape[:-1]
    y = x.reshape(-1, n).copy()
    rows = y.shape[0]
    h = 1
    while h < n:
        v = y.reshape(rows, n // (2 * h), 2, h)
        a = v[:, :, 0, :].copy()
        b = v[:, :, 1, :].copy()
        s, d = a + b, a - b
        if h >= r:
            s = s.astype(F16).astype(F32)
            d = d.astype(F16).astype(F32)
        v[:, :, 0, :] = s
        v[:, :, 1, :] = d
        h *= 2
        if h == r:
            y = y.astype(F16).astype(F32)
    return y.reshape(*lead, n)


# ----------------------------------------------------------------------------
# Activation quantisation
# ----------------------------------------------------------------------------
def _quant_rows(xf: np.ndarray, rot: bool, staging: str, k: int):
    if rot:
        if staging == "fp16":
            xf = fwht_fp16_staged(xf)
        elif staging == "fp32":
            xf = fwht_fp32(xf)
        else:
            raise ValueError(f"unknown staging {staging!r}")
    # The HIP kernels reduce with fmaxf (a NaN operand is ignored:
    # int4_gemm.cu:426-436), the torch CPU code with amax (NaN propagates);
    # they differ only for a row whose FWHT overflowed fp16.
    amax = np.fmax.reduce(np.abs(xf), axis=-1) if staging == "fp16" else np.abs(xf).max(axis=-1)
    sdiv = (amax / F32(7.0)).astype(F32) + F32(1e-12)
    scale = (sdiv * inv_sqrt_k(k)).astype(F32) if rot else sdiv.astype(F32)
    with np.errstate(invalid="ignore"):
        q = np.clip(np.rint(xf / sdiv[:, None]), -7, 7)
    return q.astype(np.int8), scale


def _row_chunks(m: int, k: int):
    """Row blocks for thread-parallel evaluation (numpy releases the GIL on
    large array operations); rows are independent, so results are identical
    to a single pass."""
    if m * k < (1 << 20) or m < 16:
        return [(0, m)]
    nchunks = min(m, 4 * (os.cpu_count() or 1))
    step = -(-m // nchunks)
    return [(i, min(m, i + step)) for i in range(0, m, step)]


def quant_activation(
    x: np.ndarray, rotate: bool | None = None, staging: str = "fp32"
) -> tuple[np.ndarray, np.ndarray]:
    """Per-token symmetric INT4 quantisation of x [M, K] (fp16 values).

    Returns (codes int8 [M, K] in [-7, 7], row scales fp32 [M]).

    * rotated K: FWHT (fp32: pack.py:118-119; fp16 staging: int4_gemm.cu:404-426),
      amax over the transformed values, sdiv = fl(amax/7) + 1e-12
      (pack.py:120-121, int4_gemm.cu:438), codes = clamp(rint(v/sdiv), -7, 7)
      with round-half-even (pack.py:123, int4_gemm.cu:443-444),
      scale = sdiv * fl32(1/sqrt(K)) (pack.py:122).
    * other K: no rotation, scale = sdiv (pack.py:124-130, int4_gemm.cu:451-477).
    """
    x = np.asarray(x)
    if x.ndim != 2:
        raise ValueError("quant_activation expects [M, K]")
    m, k = x.shape
    if staging not in ("fp16", "fp32"):
        raise ValueError(f"unknown staging {staging!r}")
    if m == 0:
        return np.zeros((0, k), np.int8), np.zeros((0,), F32)
    rot = should_rotate(k, rotate)
    chunks = _row_chunks(m, k)
    if len(chunks) == 1:
        return _quant_rows(x.astype(F32), rot, staging, k)
    codes = np.empty((m, k), np.int8)
    scale = np.empty((m,), F32)

    def work(span):
        a, b = span
        codes[a:b], scale[a:b] = _quant_rows(x[a:b].astype(F32), rot, staging, k)

    with ThreadPoolExecutor(max_workers=len(chunks)) as pool:
        list(pool.map(work, chunks))
    return codes, scale


def quant_rot_rb_loops(x_row: np.ndarray) -> tuple[np.ndarray, np.float32]:
    """Second, loop-level restatement of the HIP kernel ``quant_rot_rb<K,R>``
    (int4_gemm.cu:396-449) for ONE row: 256 virtual threads, each holding R
    consecutive values in fp32 registers, then an fp16 scratch array with one
    butterfly per (idx) slot per stage.  Slow; used only to cross-check
    ``fwht_fp16_staged`` on small inputs.  Returns (codes int8 [K], sdiv)."""
    k = x_row.shape[-1]
    r = k // _HIP_QUANT_THREADS
    lds = np.zeros(k, dtype=F16)
    for tid in range(_HIP_QUANT_THREADS):
        reg = [F32(x_row[tid * r + j]) for j in range(r)]
        length = 1
        while length < r:
            for i in range(0, r, 2 * length):
                for j in range(i, i + length):
                    a, b = reg[j], reg[j + length]
                    reg[j] = F32(a + b)
                    reg[j + length] = F32(a - b)
            length <<= 1
        for j in range(r):
            lds[tid * r + j] = F16(reg[j])
    length = r
    while length < k:
        for idx in range(k // 2):
            group, off = divmod(idx, length)
            p = group * 2 * length + off
            a, b = F32(lds[p]), F32(lds[p + length])
            lds[p] = F16(F32(a + b))
            lds[p + length] = F16(F32(a - b))
        length <<= 1
    vals = lds.astype(F32)
    m = F32(0.0)
    for v in vals:
        m = max(m, F32(abs(v)))
    sdiv = F32(F32(m / F32(7.0)) + F32(1e-12))
    codes = np.empty(k, dtype=np.int8)
    for i, v in enumerate(vals):
        q = int(np.rint(F32(v / sdiv)))
        codes[i] = max(-7, min(7, q))
    return codes, sdiv


# ----------------------------------------------------------------------------
# Packed formats
# ----------------------------------------------------------------------------
def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """q[..., K] (values in [-8, 7]) -> int32 [..., K/8]; element j of each
    group of 8 sits at bits 4j..4j+3 (pack.py:34-42)."""
    q = np.asarray(q)
    if q.shape[-1] % 8:
        raise ValueError("K must be a multiple of 8")
    g = (q.astype(np.int64) & 0xF).reshape(*q.shape[:-1], q.shape[-1] // 8, 8)
    shifts = (4 * np.arange(8, dtype=np.int64))
    words = (g << shifts).sum(axis=-1)
    return words.astype(np.uint32).view(np.int32)


def unpack_nibbles(packed: np.ndarray, k: int) -> np.ndarray:
    """int32 [..., K/8] -> int8 [..., K], two's-complement nibbles (pack.py:71-76).
    Little-endian bytes: byte b of a word holds elements 2b (low nibble) and
    2b+1 (high nibble)."""
    w = np.ascontiguousarray(packed, dtype=np.int32)
    b = w.view(np.uint8).reshape(*w.shape[:-1], w.shape[-1] * 4)
    out = np.empty((*w.shape[:-1], k), dtype=np.uint8)
    np.bitwise_and(b, 0xF, out=out[..., 0::2])
    np.right_shift(b, 4, out=out[..., 1::2])
    out ^= 8
    return (out.view(np.int8) - np.int8(8)).astype(np.int8)


def pack_linear_weight(weight: np.ndarray, rotate: bool | None = None) -> np.ndarray:
    """Linear.weight [N, K] -> int32 [N, K/8 + 1] (pack.py:85-101): optional
    FWHT scaled by fl32(1/sqrt(K)), per-row scale = max(amax, 1e-12)/7,
    codes = clamp(round(w/scale), -7, 7), scale bits in the last word."""
    w = np.asarray(weight, dtype=F32)
    if w.ndim != 2:
        raise ValueError("expected 2D weight")
    n, k = w.shape
    if k % 64:
        raise ValueError(f"K must be a multiple of 64 for gemm_iu4, got {k}")
    if should_rotate(k, rotate):
        w = (fwht_fp32(w) * inv_sqrt_k(k)).astype(F32)
    amax = np.maximum(np.abs(w).max(axis=-1), F32(1e-12)).astype(F32)
    scale = (amax / F32(7.0)).astype(F32)
    q = np.clip(np.rint(w / scale[:, None]), -7, 7).astype(np.int32)
    return np.concatenate([pack_nibbles(q), scale.view(np.int32)[:, None]], axis=1)


def pad_rows(packed: np.ndarray, row_words: int) -> np.ndarray:
    """Row-major padding to a longer row stride with zero words
    (apply.py:68-69 pads [N, K/8+1] to [N, K/8+8])."""
    n, w = packed.shape
    out = np.zeros((n, row_words), dtype=np.int32)
    out[:, :w] = packed
    return out


def preshuffle_wmma_weight(packed: np.ndarray, k: int) -> np.ndarray:
    """Fragment-major layout (pack.py:45-68): payload flat as [K/16][N][2
    words], then the N scales, inside a tensor declared [N, K/8 + 9]."""
    n = packed.shape[0]
    words = k // 8
    if k % 16 or packed.shape[1] < words + 1:
        raise ValueError("invalid packed weight shape")
    out = np.zeros((n, words + FRAGMENT_MAJOR_PAD_WORDS), dtype=np.int32)
    flat = out.reshape(-1)
    payload = packed[:, :words].reshape(n, words // 2, 2).transpose(1, 0, 2)
    flat[: n * words] = payload.reshape(-1)
    flat[n * words: n * words + n] = packed[:, words]
    return out


def weight_codes_scales(
    packed: np.ndarray, k: int, layout: str = "row"
) -> tuple[np.ndarray, np.ndarray]:
    """Read codes int8 [N, K] and scales fp32 [N] from any reference layout:
    row-major with row stride = packed.shape[1] (>= K/8+1), or fragment-major
    (int4_gemm.cu:44-61 addressing)."""
    packed = np.ascontiguousarray(packed, dtype=np.int32)
    n, row = packed.shape
    words = k // 8
    if layout == "row":
        if row < words + 1:
            raise ValueError("row too short")
        codes = unpack_nibbles(packed[:, :words], k)
        scales = packed[:, words].copy().view(F32)
    elif layout == "fragment":
        flat = packed.reshape(-1)
        payload = flat[: n * words].reshape(words // 2, n, 2).transpose(1, 0, 2)
        codes = unpack_nibbles(payload.reshape(n, words), k)
        scales = flat[n * words: n * words + n].copy().view(F32)
    else:
        raise ValueError(layout)
    return codes, scales


# ----------------------------------------------------------------------------
# GEMM
# ----------------------------------------------------------------------------
def int_accumulate(qa: np.ndarray, qw: np.ndarray) -> np.ndarray:
    """acc[m, n] = sum_k qa[m, k] * qw[n, k] as int32.  fp32 BLAS is exact
    here because every partial sum is an integer below 2**24 (|acc| <= 56K),
    which is also why the reference's ``q_a.float() @ q_w.float().T``
    (pack.py:143) is exact."""
    k = qa.shape[-1]
    if 56 * k >= 1 << 24:
        raise ValueError("K too large for an exact fp32 accumulation")
    acc = qa.astype(F32) @ qw.astype(F32).T
    return acc.astype(np.int32)


def dequant(acc: np.ndarray, sa: np.ndarray, sw: np.ndarray) -> np.ndarray:
    """y = fp16((fp32(acc) * sa[m]) * sw[n]), left to right, round to nearest
    even (int4_gemm.cu:199-200, pack.py:144-145)."""
    y = (acc.astype(F32) * sa.astype(F32)[:, None]).astype(F32)
    y = (y * sw.astype(F32)[None, :]).astype(F32)
    return y.astype(F16)


def int4_gemm_ref(
    x: np.ndarray,
    packed_w: np.ndarray,
    rotate: bool | None = None,
    staging: str = "fp32",
    layout: str = "row",
) -> np.ndarray:
    """W4A4 GEMM of x [..., K] fp16 with a packed weight (pack.py:134-145)."""
    x = np.asarray(x)
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    qa, sa = quant_activation(x2, rotate=rotate, staging=staging)
    qw, sw = weight_codes_scales(packed_w, k, layout)
    acc = int_accumulate(qa, qw)
    y = dequant(acc, sa, sw)
    return y.reshape(*x.shape[:-1], qw.shape[0])


# ----------------------------------------------------------------------------
# Seeded inputs (the synthetic stand-ins for the reference's workloads)
# ----------------------------------------------------------------------------
def make_activations(m: int, k: int, seed: int, outlier_frac: float = 0.01,
                     outlier_gain: float = 20.0) -> np.ndarray:
    """x ~ N(0, 1) [m, k] with ``outlier_frac`` of the channels scaled by
    ``outlier_gain``, cast to fp16."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=F32)
    n_out = max(1, int(k * outlier_frac))
    ch = rng.permutation(k)[:n_out]
    x[:, ch] *= F32(outlier_gain)
    return x.astype(F16)


def make_weight(n: int, k: int, seed: int, std: float = 0.02) -> np.ndarray:
    """W ~ N(0, std) [n, k] fp32."""
    rng = np.random.default_rng(seed + 7919)
    return (rng.standard_normal((n, k), dtype=F32) * F32(std)).astype(F32)


def random_packed_weight(n: int, k: int, seed: int) -> np.ndarray:
    """Random int32 payload (every nibble value, -8 included) with scales in
    U[0.01, 0.06): the reference test fixture's construction
    (tests/test_w4a4.py:12-21)."""
    rng = np.random.default_rng(seed + 104729)
    payload = rng.integers(-(2**31), 2**31 - 1, size=(n, k // 8), dtype=np.int64).astype(np.int32)
    scales = (rng.random(n, dtype=F32) * F32(0.05) + F32(0.01)).astype(F32)
    return np.concatenate([payload, scales.view(np.int32)[:, None]], axis=1)
