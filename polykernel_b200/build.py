"""Build libpkb200.so in-tree for sm_100a (nvcc cross-compiles without a GPU)."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_lib", "libpkb200.so")


def build(verbose: bool = False) -> str:
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
           "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-shared",
           "-o", OUT, os.path.join(CSRC, "pkb200.cu"), "-lcudart"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=CSRC)
    # the .npy launcher harness (reference cuda_run command line) over the library
    harness = ["nvcc", "-Wno-deprecated-gpu-targets", "-O2", "-std=c++17", "-o", os.path.join(os.path.dirname(OUT), "cuda_run"),
               os.path.join(CSRC, "cuda_run.cpp"), "-L" + os.path.dirname(OUT), "-lpkb200",
               "-lcudart", "-Xlinker", "-rpath=$ORIGIN"]
    if verbose:
        print(" ".join(harness))
    subprocess.run(harness, check=True, cwd=CSRC)
    return OUT


if __name__ == "__main__":
    print(build(verbose=True))
