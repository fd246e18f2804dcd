"""Builds the cnnue CUDA library in-tree (chineseai_b200/libcnnue.so) for sm_100a.

Usage: python -m chineseai_b200.build [--force] [--ptxas-info]
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libcnnue.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-shared",
    "-Xcompiler",
    "-fPIC,-O3,-ffp-contract=off",  # host float code rounds every operation (restated reference arithmetic)
    "--expt-relaxed-constexpr",
    "-I" + INCLUDE,
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the cnnue library needs CUDA 12.9+ to build")
    return cand


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, ptxas_info: bool = False) -> str:
    """Compiles every CUDA/C++ source of the package into libcnnue.so."""
    if not force and not ptxas_info and not _stale():
        return LIB
    cmd = [_nvcc()] + ARCH_FLAGS + NVCC_FLAGS
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    tmp = LIB + ".tmp"
    cmd += ["-o", tmp] + sources()
    proc = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("nvcc failed building libcnnue.so")
    if ptxas_info:
        sys.stdout.write(proc.stderr)
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, ptxas_info=args.ptxas_info))


if __name__ == "__main__":
    main()
