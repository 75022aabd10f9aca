"""Build librsort_b200.so in-tree with nvcc for sm_100a.

    python -m rccl_b200.build_ext [--force]

Each translation unit is compiled to an object file in parallel, then the
objects are linked into one shared library.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_lib", "librsort_b200.so")
SOURCES = ["rsort_kernels.cu", "rsort_dist.cu", "rsort_api.cu", "rsort_static.cu",
           "rsort_exchange.cu", "rsort_records.cu", "rsort_dist_nccl.cu",
           "rsort_multiway.cu"]
HEADERS = ["rsort_device.cuh", "rsort_kernels.cuh", "rsort_dist.cuh", "rsort_records.cuh",
           "rsort_internal.cuh", "rsort_multiway.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _deps():
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(HERE, "..", "include", "rsort_b200.h"))
    deps.append(os.path.abspath(__file__))
    return [d for d in deps if os.path.exists(d)]


def _stale(out: str) -> bool:
    if not os.path.exists(out):
        return True
    built = os.path.getmtime(out)
    return any(os.path.getmtime(d) > built for d in _deps())


def build(force: bool = False, verbose: bool = False, out: str = OUT,
          extra_flags: list[str] | None = None) -> str:
    """Compile the library (only when a source, header or this script is
    newer than `out`, unless `force`).  `extra_flags` are passed to every
    nvcc compile (tile-shape macros of the kernels, for example)."""
    if not force and not _stale(out):
        return out
    os.makedirs(os.path.dirname(out), exist_ok=True)
    objdir = out + ".objs"
    os.makedirs(objdir, exist_ok=True)
    extra = list(extra_flags or [])

    def compile_one(src: str) -> str:
        obj = os.path.join(objdir, os.path.splitext(src)[0] + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", "-o", obj, os.path.join(CSRC, src)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        return obj

    workers = max(1, min(len(SOURCES), os.cpu_count() or 1))
    with ThreadPoolExecutor(workers) as pool:
        objs = list(pool.map(compile_one, SOURCES))
    tmp = out + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
