"""Pins the oracle's fp16-staging quant to the reference's own kernel.

The reference's HIP kernel ``quant_rot_rb<K, R>`` (pi05_fast/w4a4/csrc/
int4_gemm.cu:396-449) is compiled from the reference checkout and run on host
threads (``oracle/ref_quant``; the library lands in ``oracle/_ref``).  Its
codes must equal the oracle's ``staging="fp16"`` restatement bit for bit, and
its row scales too (the kernel multiplies by ``rsqrtf(K)``, taken here as
the IEEE 1/sqrt(K); the oracle and this repository's kernels use the fp32
constant 1/sqrt(K), which is the same number for these K).
Skips where the reference checkout (and so the library) is absent.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

from oracle import w4a4_oracle as orc

HERE = os.path.dirname(os.path.abspath(__file__))


def _ref_lib():
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle", "ref_quant"))
    try:
        import build_ref
    finally:
        sys.path.pop(0)
    path = build_ref.build()
    if path is None:
        pytest.skip("reference checkout absent: the reference quant kernel cannot be built here")
    lib = ctypes.CDLL(path)
    lib.quant_rot_rb_ref.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                     ctypes.c_void_p]
    lib.quant_rot_rb_ref.restype = ctypes.c_int
    return lib


def ref_quant(lib, x: np.ndarray):
    m, k = x.shape
    xb = np.ascontiguousarray(x.astype(np.float16)).view(np.uint16)
    q = np.zeros((m, k // 8), dtype=np.int32)
    sc = np.zeros(m, dtype=np.float32)
    assert lib.quant_rot_rb_ref(xb.ctypes.data, m, k, q.ctypes.data, sc.ctypes.data) == 0
    nib = (q[:, :, None] >> (4 * np.arange(8))[None, None, :]) & 0xF
    codes = np.where(nib >= 8, nib - 16, nib).astype(np.int8).reshape(m, k)
    return codes, sc


def _inputs(k: int, seed: int) -> np.ndarray:
    x = orc.make_activations(6, k, seed=seed)
    x[1] = 0.0                                      # an all-zero row
    x[2] = np.float16(0.25)                         # constant row: one non-zero FWHT output
    x[3, ::3] = np.float16(-60000.0)                # near the fp16 range
    x[4] = (np.arange(k) % 7 - 3).astype(np.float16)  # small integers: ties in q = v / sdiv
    return x.astype(np.float16)


@pytest.mark.filterwarnings("ignore::RuntimeWarning")  # the fp16-overflowing row
@pytest.mark.parametrize("k", [1024, 2048, 16384])
@pytest.mark.parametrize("seed", [0, 1])
def test_fp16_staging_oracle_equals_reference_kernel(k, seed):
    lib = _ref_lib()
    x = _inputs(k, seed)
    codes, sc = ref_quant(lib, x)
    qa, sa = orc.quant_activation(x, rotate=True, staging="fp16")
    np.testing.assert_array_equal(qa, codes)
    # row scales bit for bit (rsqrtf(K) here is the IEEE 1/sqrt(K), equal to
    # the fp32 constant for these K); the overflowing row's scale is inf
    np.testing.assert_array_equal(sa.view(np.int32), sc.view(np.int32))
    assert np.isinf(sc[3])
