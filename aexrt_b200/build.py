"""Builds the in-tree CUDA library ``aexrt_b200/libaexrt_b200.so`` for sm_100a.

The library is a plain C-ABI shared object (see include/aexrt_b200.h) built by
nvcc directly; the CUDA runtime is linked statically and the driver is reached
through cudaGetDriverEntryPoint, so the .so loads on machines without a GPU.

    python -m aexrt_b200.build [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libaexrt_b200.so")
SOURCES = ["capi.cu"]
HEADERS = ["conv_halo.cuh", "conv_tc.cuh", "ptx.cuh", "quant.cuh", "stem.cuh", "yolo_ops.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-shared",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _host_compiler_flags() -> list:
    # Prefer the system gcc (the image's PATH gcc wrapper lacks some runtime specs).
    gxx = "/usr/bin/g++"
    return ["-ccbin", gxx] if os.path.exists(gxx) else []


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(ROOT, "include", "aexrt_b200.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    cmd = [_nvcc()] + _host_compiler_flags() + NVCC_FLAGS
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, f) for f in SOURCES] + ["-o", LIB + ".tmp"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libaexrt_b200.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
