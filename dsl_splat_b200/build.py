"""Builds libsplat200.so in place for sm_100a (nvcc, no JIT cache).

-fmad=false keeps every multiply-add two IEEE roundings unless the source
asks for __fmaf_rn, which is what makes radii, tile counts and sort keys
reproducible on the CPU.  Division and square root stay IEEE-rounded (the
nvcc defaults -prec-div=true -prec-sqrt=true, no --use_fast_math).
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libsplat200.so")
SOURCES = ["splat200.cu"]
HEADERS = ["splat_common.cuh", "cameras.cuh", "project.cuh", "binning.cuh", "render.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17", "-fmad=false",
    "-Xcompiler", "-fPIC", "-shared",
]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    built = os.path.getmtime(LIB)
    inputs = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    inputs.append(os.path.join(ROOT, "include", "splat200.h"))
    return any(os.path.exists(f) and os.path.getmtime(f) > built for f in inputs)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    cmd = [nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp",
           *[os.path.join(CSRC, f) for f in SOURCES]]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
