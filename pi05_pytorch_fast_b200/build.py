"""Build libw4a4_sm100.so in-tree with nvcc for sm_100a.

    python -m pi05_pytorch_fast_b200.build [--force] [--verbose]

The library is self-contained (static CUDA runtime; the TMA descriptor
encoder is fetched from the driver at run time), so the built file travels
with the source tree to any B200 host with a CUDA 12.8+ driver.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT = os.path.join(PKG_DIR, "libw4a4_sm100.so")
MAIN_SOURCE = os.path.join(CSRC, "w4a4_sm100.cu")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "-shared",
]


def _sources() -> list[str]:
    files = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))
             if f.endswith((".cu", ".cuh", ".h"))]
    files += [os.path.join(INCLUDE, f) for f in sorted(os.listdir(INCLUDE)) if f.endswith(".h")]
    return files


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.isfile(cand):
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not os.path.isfile(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(f) <= t for f in _sources())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library unless it is newer than every source; returns its path."""
    if not force and up_to_date():
        return OUT
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-o", OUT + ".tmp", MAIN_SOURCE]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
