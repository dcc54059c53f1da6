"""In-tree build of libmegamoe.so for sm_100a (nvcc cross-compiles without a GPU)."""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
SOURCES = ["mm_api.cu", "mm_route.cu", "mm_experts.cu", "mm_finalize.cu", "mm_comm.cu"]
HEADERS = ["mm_kernels.cuh", "mm_layout.cuh", "mm_numerics.cuh", "mm_ptx.cuh"]
OUTPUT = os.path.join(HERE, "libmegamoe.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-shared",
    "-cudart",
    "static",
]


def _stale() -> bool:
    if not os.path.exists(OUTPUT):
        return True
    built = os.path.getmtime(OUTPUT)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(REPO, "include", "megamoe.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(p) > built for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; returns its path."""
    if not force and not _stale():
        return OUTPUT
    cmd = [NVCC, *FLAGS, "-I", os.path.join(REPO, "include"), "-I", CSRC, "-o", OUTPUT]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode}) building {OUTPUT}")
    if verbose:
        sys.stderr.write(res.stderr)
    return OUTPUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
