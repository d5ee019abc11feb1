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
# capi.cu holds the C ABI and the memory-bound kernels; the conv kernel instances are split over
# translation units that compile in parallel
SOURCES = ["capi.cu", "engine_file.cu", "yolo_runtime.cu", "kernels_slot.cu", "kernels_halo_i8_silu.cu", "kernels_halo_i8_linear.cu",
           "kernels_halo_f16.cu", "kernels_halo_mb.cu", "kernels_halo_pg.cu", "kernels_halo_ql.cu",
           "kernels_halo_ql_mb.cu",
           "kernels_stem16.cu", "kernels_stem32.cu", "kernels_stem48.cu", "kernels_stem64.cu"]
HEADERS = ["codes.cuh", "conv_halo.cuh", "conv_tc.cuh", "engine_file.h", "graph_ops.cuh", "kernels.cuh", "launch.cuh", "nms.cuh",
           "psa.cuh", "ptx.cuh",
           "quant.cuh", "quant_cluster.cuh", "stem.cuh", "yolo_ops.cuh"]
OBJ_DIR = os.path.join(HERE, "_build")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
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
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [
        os.path.join(ROOT, "include", h) for h in ("aexrt_b200.h", "aexrt_yolo.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list, what: str, verbose: bool) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed: {what}")
    if verbose:
        sys.stderr.write(res.stderr)


def _includes(path: str, seen: set) -> set:
    """The quoted #include files a source reaches (transitively), as absolute paths."""
    import re

    if path in seen or not os.path.exists(path):
        return seen
    seen.add(path)
    for inc in re.findall(r'^#include "([^"]+)"', open(path, encoding="utf-8").read(), re.M):
        _includes(os.path.normpath(os.path.join(os.path.dirname(path), inc)), seen)
    return seen


def _stale(src: str, obj: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in _includes(os.path.join(CSRC, src), set()))


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    from concurrent.futures import ThreadPoolExecutor

    os.makedirs(OBJ_DIR, exist_ok=True)
    base = [_nvcc()] + _host_compiler_flags() + NVCC_FLAGS
    objs = [os.path.join(OBJ_DIR, os.path.splitext(f)[0] + ".o") for f in SOURCES]
    jobs = []
    for src, obj in zip(SOURCES, objs):
        if not (force or verbose) and not _stale(src, obj):
            continue  # object newer than its source and every header it includes
        cmd = base + (["-Xptxas", "-v"] if verbose else []) + ["-c", os.path.join(CSRC, src), "-o", obj]
        jobs.append((cmd, src))
    with ThreadPoolExecutor(max_workers=max(1, len(jobs))) as ex:
        for f in [ex.submit(_run, cmd, src, verbose) for cmd, src in jobs]:
            f.result()
    _run(base + ["-shared"] + objs + ["-o", LIB + ".tmp"], "link", verbose)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
