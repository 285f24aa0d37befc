"""Generate golden vectors by running the UNMODIFIED reference CPU code.

Run once in a container that holds the reference checkout (its path is taken
from ``--reference`` or the ``W4A4_REFERENCE`` environment variable):

    python tests/golden/make_golden.py --reference <checkout> \
        --out tests/golden/w4a4_golden.npz

The reference functions called are ``pi05_fast.w4a4.pack``'s
``quant_activation_cpu`` (pack.py:113-131), ``pack_linear_weight``
(pack.py:85-101), ``preshuffle_wmma_weight`` (pack.py:45-68) and
``int4_gemm_ref`` (pack.py:134-145).  Inputs are drawn from torch generators
with fixed seeds; every input and output is stored so the tests never need
the reference at run time.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np


def _ref_modules(path: str):
    sys.path.insert(0, path)
    import torch  # noqa: F401
    from pi05_fast.w4a4 import pack  # type: ignore

    return pack


def _activations(torch, m, k, seed, outliers=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    if outliers:
        idx = torch.randperm(k, generator=g)[: max(1, k // 100)]
        x[:, idx] *= 20
    return x.half()


def _packed_random(torch, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    payload = torch.randint(-(2**31), 2**31 - 1, (n, k // 8), dtype=torch.int32, generator=g)
    scales = torch.rand(n, dtype=torch.float32, generator=g) * 0.05 + 0.01
    return torch.cat((payload, scales.view(torch.int32).unsqueeze(1)), dim=1)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("W4A4_REFERENCE", ""))
    ap.add_argument("--out", default=os.path.join(os.path.dirname(__file__), "w4a4_golden.npz"))
    args = ap.parse_args()
    if not args.reference:
        sys.exit("pass --reference <path to the reference checkout>")
    pack = _ref_modules(args.reference)
    import torch

    out: dict[str, np.ndarray] = {}

    # 1. activation quant (fp32 emulation), rotated and non-rotated K.
    for name, (m, k, seed) in {
        "q2048": (13, 2048, 1),
        "q1024": (7, 1024, 2),
        "q16384": (3, 16384, 3),
        "q192": (5, 192, 4),      # not rotated
        "q4096": (2, 4096, 5),    # power of two but not in ROTATE_K
    }.items():
        x = _activations(torch, m, k, seed)
        q, s = pack.quant_activation_cpu(x)
        out[f"{name}_x"] = x.numpy()
        out[f"{name}_codes"] = q.numpy().astype(np.int8)
        out[f"{name}_scale"] = s.numpy()
    # explicit rotate override on a rotated K
    x = _activations(torch, 4, 2048, 6)
    q, s = pack.quant_activation_cpu(x, rotate=False)
    out["q2048norot_x"], out["q2048norot_codes"], out["q2048norot_scale"] = (
        x.numpy(), q.numpy().astype(np.int8), s.numpy())

    # 2. weight pack.
    for name, (n, k, seed, std) in {
        "w2048": (40, 2048, 11, 0.02),
        "w1024": (16, 1024, 12, 0.02),
        "w16384": (8, 16384, 13, 0.02),
        "w128": (9, 128, 14, 0.5),
    }.items():
        g = torch.Generator().manual_seed(seed)
        w = torch.randn(n, k, generator=g) * std
        out[f"{name}_w"] = w.numpy()
        out[f"{name}_packed"] = pack.pack_linear_weight(w).numpy()
    # a zero row exercises the amax clamp (pack.py:96)
    wz = torch.zeros(2, 64)
    out["wzero_w"] = wz.numpy()
    out["wzero_packed"] = pack.pack_linear_weight(wz).numpy()

    # 3. fragment-major preshuffle of the random-payload fixture.
    for name, (n, k, seed) in {"pre64": (7, 64, 21), "pre2048": (32, 2048, 22)}.items():
        p = _packed_random(torch, n, k, seed)
        out[f"{name}_packed"] = p.numpy()
        out[f"{name}_tiled"] = pack.preshuffle_wmma_weight(p, k).numpy()

    # 4. end-to-end CPU GEMM emulation.
    cases = {
        # config-0-like QKV block, scaled down: M=17 tokens, N=160 rows
        "g2048": (17, 2048, 160, 31, "packed_from_w"),
        # down-projection width with the random-payload fixture (has -8 nibbles)
        "g16384": (3, 16384, 24, 32, "random"),
        "g1024": (9, 1024, 48, 33, "packed_from_w"),
        "g128": (6, 128, 20, 34, "packed_from_w"),   # not rotated
    }
    for name, (m, k, n, seed, kind) in cases.items():
        x = _activations(torch, m, k, seed)
        if kind == "random":
            p = _packed_random(torch, n, k, seed + 1)
        else:
            g = torch.Generator().manual_seed(seed + 1)
            p = pack.pack_linear_weight(torch.randn(n, k, generator=g) * 0.02)
        y = pack.int4_gemm_ref(x, p)
        out[f"{name}_x"] = x.numpy()
        out[f"{name}_packed"] = p.numpy()
        out[f"{name}_y"] = y.numpy()

    np.savez_compressed(args.out, **out)
    total = sum(v.nbytes for v in out.values())
    print(f"wrote {len(out)} arrays ({total / 1e6:.2f} MB raw) to {args.out}")


if __name__ == "__main__":
    main()
