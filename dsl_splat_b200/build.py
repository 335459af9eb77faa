"""Builds libsplat200.so in place for sm_100a (nvcc, no JIT cache).

Three translation units, compiled in parallel and linked into one library:

* splat200.cu (entry points, forward kernels, binning, blending) with
  -fmad=false: every multiply-add stays two IEEE roundings unless the source
  asks for __fmaf_rn, which is what makes radii, tile counts, sort keys and
  the blended image reproducible on the CPU;
* project_backward.cu (the projection + SH backward) and aaa_backward.cu
  (the AAA blend's record backward) with -fmad=true -prec-div=false
  -prec-sqrt=false: their outputs are gradients, compared within a relative
  tolerance, and contraction plus the approximate divide and square root (a
  few ulp) remove a large part of their arithmetic.

splat200.cu keeps IEEE-rounded division and square root (the nvcc defaults
-prec-div=true -prec-sqrt=true); nothing is built with --use_fast_math.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libsplat200.so")
BUILD_DIR = os.path.join(HERE, "_build")
# source -> its contraction flag
SOURCES = {"splat200.cu": ["-fmad=false"],
           "project_backward.cu": ["-fmad=true", "-prec-div=false", "-prec-sqrt=false"],
           "aaa_backward.cu": ["-fmad=true", "-prec-div=false", "-prec-sqrt=false"]}
HEADERS = ["splat_common.cuh", "cameras.cuh", "project.cuh", "binning.cuh", "render.cuh",
           "footprint.cuh", "tile_modes.cuh", "host_runtime.h", "rade.cuh", "rade_project.cuh",
           "aaa.cuh", "aaa_render.cuh", "aaa_api.cuh", "aaa_blend_params.cuh",
           "aaa_backward.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    built = os.path.getmtime(LIB)
    inputs = [os.path.join(CSRC, f) for f in [*SOURCES, *HEADERS]]
    inputs.append(os.path.join(ROOT, "include", "splat200.h"))
    return any(os.path.exists(f) and os.path.getmtime(f) > built for f in inputs)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    os.makedirs(BUILD_DIR, exist_ok=True)
    objects, jobs = [], []
    for src, flags in SOURCES.items():
        obj = os.path.join(BUILD_DIR, os.path.splitext(src)[0] + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, *flags, "-I", os.path.join(ROOT, "include"), "-c",
               os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        jobs.append((cmd, subprocess.Popen(cmd)))
        objects.append(obj)
    failed = [cmd for cmd, job in jobs if job.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, failed[0])
    link = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LIB + ".tmp",
            *objects]
    if verbose:
        print(" ".join(link), file=sys.stderr)
    subprocess.run(link, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
