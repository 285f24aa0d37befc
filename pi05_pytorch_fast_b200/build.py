"""Build the two in-tree libraries of the package.

    python -m pi05_pytorch_fast_b200.build [--force] [--verbose]

libw4a4_sm100.so: the kernels and the C ABI (nvcc, sm_100a).  Self-contained
(static CUDA runtime; the TMA descriptor encoder is fetched from the driver
at run time), so it travels with the source tree to any B200 host with a
CUDA 12.8+ driver.

_w4a4_ops.so: the pi05_w4a4 torch ops (g++ against the installed torch's
headers), calling libw4a4_sm100.so through its C ABI; found next to it
through an $ORIGIN run path.  It must be rebuilt when torch changes.
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
OPS_SOURCE = os.path.join(CSRC, "torch_ops.cpp")
OPS_OUT = os.path.join(PKG_DIR, "_w4a4_ops.so")

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


def _ops_sources() -> list[str]:
    import torch

    return [OPS_SOURCE, OUT, torch.__file__,
            *[os.path.join(INCLUDE, f) for f in sorted(os.listdir(INCLUDE)) if f.endswith(".h")]]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.isfile(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _cxx() -> str:
    """The host C++ compiler for the op library: W4A4_CXX, else the system
    g++.  CXX is not used on purpose: a compiler whose own libstdc++ gets
    linked statically puts a second C++ runtime into the library, and an
    exception torch throws through the op body (any TORCH_CHECK whose message
    needs a temporary string) then unwinds with a foreign personality routine
    and crashes the process."""
    for cand in (os.environ.get("W4A4_CXX"), "/usr/bin/g++", shutil.which("g++")):
        if cand and os.path.isfile(cand):
            return cand
    raise RuntimeError("g++ not found")


def _newer(out: str, sources: list[str]) -> bool:
    if not os.path.isfile(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(f) <= t for f in sources)


def up_to_date() -> bool:
    return _newer(OUT, _sources()) and _newer(OPS_OUT, _ops_sources())


def _run(cmd: list[str], out: str, verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"{cmd[0]} failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    os.replace(out + ".tmp", out)


def build_ops(force: bool = False, verbose: bool = False) -> str:
    """Compile _w4a4_ops.so (needs libw4a4_sm100.so built first)."""
    if not force and _newer(OPS_OUT, _ops_sources()):
        return OPS_OUT
    import torch
    from torch.utils import cpp_extension

    abi = int(torch.compiled_with_cxx11_abi())
    cmd = [_cxx(), "-O2", "-std=c++17", "-shared", "-fPIC",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-I", INCLUDE]
    for inc in cpp_extension.include_paths():
        cmd += ["-I", inc]
    cmd += ["-I", os.path.join(os.path.dirname(os.path.dirname(_nvcc())), "include"),
            "-o", OPS_OUT + ".tmp", OPS_SOURCE]
    for libdir in cpp_extension.library_paths():
        cmd += ["-L", libdir]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch_cpu", "-L", PKG_DIR, "-lw4a4_sm100",
            "-Wl,-rpath,$ORIGIN"]
    _run(cmd, OPS_OUT, verbose)
    return OPS_OUT


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile both libraries unless each is newer than its sources; returns
    the kernel library's path."""
    if force or not _newer(OUT, _sources()):
        _build_kernels(verbose)
    build_ops(force=force, verbose=verbose)
    return OUT


def _build_kernels(verbose: bool) -> None:
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-o", OUT + ".tmp", MAIN_SOURCE]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    _run(cmd, OUT, verbose)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
