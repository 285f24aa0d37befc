"""Build oracle/_ref/libquant_rot_rb_ref.so from the reference checkout.

TEST INFRASTRUCTURE ONLY.  The reference's HIP quant kernel
(pi05_fast/w4a4/csrc/int4_gemm.cu, ``quant_rot_rb`` and ``QUANT_TPB``) is read
from the reference tree at build time and handed to g++ unchanged, on its
standard input, between ``gpu_shim.h`` and ``driver.cpp``, which run it on
host threads; only the compiled library is written (``oracle/_ref``, not
committed).  Without the reference tree (the GPU box) the library built
earlier is used, else the tests that need it skip.
"""

from __future__ import annotations

import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(os.path.dirname(HERE), "_ref")
LIB = os.path.join(OUT_DIR, "libquant_rot_rb_ref.so")
DEFAULT_SRC = os.path.join(os.sep, "root", "reference", "pi05_fast", "w4a4", "csrc", "int4_gemm.cu")


def _extract(text: str) -> str:
    tpb = re.search(r"^#define QUANT_TPB\s+\d+\s*$", text, re.M)
    start = text.index("template <int K, int R>\n__global__ void quant_rot_rb(")
    depth, i, opened = 0, text.index("{", start), False
    while True:
        c = text[i]
        if c == "{":
            depth += 1
            opened = True
        elif c == "}":
            depth -= 1
            if opened and depth == 0:
                break
        i += 1
    if not tpb:
        raise RuntimeError("QUANT_TPB not found in the reference source")
    return tpb.group(0) + "\n\n" + text[start:i + 1] + "\n"


def build(src: str = DEFAULT_SRC, force: bool = False) -> str | None:
    """Path of the library, built here when the reference checkout is
    present; without it, the library built earlier (it travels with the
    repository's built files), else None."""
    if not os.path.exists(src):
        return LIB if os.path.exists(LIB) else None
    inputs = [__file__, os.path.join(HERE, "driver.cpp"), os.path.join(HERE, "gpu_shim.h"), src]
    if os.path.exists(LIB) and not force and os.path.getmtime(LIB) >= max(map(os.path.getmtime, inputs)):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    with open(src) as f:
        kernel = _extract(f.read())
    unit = '#include "gpu_shim.h"\n' + kernel + '#include "driver.cpp"\n'
    cmd = ["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-pthread", "-I", HERE, "-x", "c++", "-",
           "-o", LIB]
    subprocess.run(cmd, input=unit, text=True, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
