"""Build libs2s.so (sm_100a) in-tree with nvcc.

    python swin2sr-rs_b200/build.py [--force]

The library is one unity translation unit (csrc/s2s.cu) compiled for
sm_100a only, with the C ABI of include/s2s.h; it depends on the CUDA runtime
(linked statically) and zlib (the PNG codec).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB = PKG / "libs2s.so"
SOURCES = sorted((PKG / "csrc").glob("*.cu")) + sorted((PKG / "csrc").glob("*.cuh")) + \
    [ROOT / "include" / "s2s.h"]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr"]


def build(force: bool = False, verbose: bool = False) -> Path:
    if LIB.exists() and not force:
        newest = max(p.stat().st_mtime for p in SOURCES)
        if LIB.stat().st_mtime >= newest:
            return LIB
    cmd = [NVCC, *FLAGS, "-I", str(ROOT / "include"), "-o", str(LIB) + ".tmp",
           str(PKG / "csrc" / "s2s.cu"), "-lz"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
