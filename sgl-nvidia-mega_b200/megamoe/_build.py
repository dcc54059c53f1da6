"""In-tree build of libmegamoe.so for sm_100a (nvcc cross-compiles without a GPU).

Each translation unit compiles to its own object (in parallel), then one link:
mm_gate_dsv41.cu takes the DeepSeek-V4.1 gate's floating-point flags
(flush-to-zero, approximate square root and division, the reference's NVRTC
options for that gate), every other file the default IEEE ones.
"""

from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
SOURCES = ["mm_api.cu", "mm_route.cu", "mm_gate_dsv41.cu", "mm_experts.cu", "mm_finalize.cu", "mm_comm.cu"]
HEADERS = ["mm_gate.cuh", "mm_kernels.cuh", "mm_layout.cuh", "mm_numerics.cuh", "mm_ptx.cuh"]
OUTPUT = os.path.join(HERE, "libmegamoe.so")
OBJDIR = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMPILE = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC"]
# per-file floating-point flags (the DeepSeek-V4.1 gate's, routed_expert_gemm.py:213-220)
FILE_FLAGS = {"mm_gate_dsv41.cu": ["-ftz=true", "-prec-sqrt=false", "-prec-div=false"]}


def compile_flags(source: str) -> list:
    """nvcc flags of one translation unit (without -c / -o)."""
    return [*COMPILE, *FILE_FLAGS.get(source, []), "-I", os.path.join(REPO, "include"), "-I", CSRC]


def _stale() -> bool:
    if not os.path.exists(OUTPUT):
        return True
    built = os.path.getmtime(OUTPUT)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(REPO, "include", "megamoe.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(p) > built for p in deps)


def _run(cmd, verbose):
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose:
        sys.stderr.write(res.stderr)
    return res


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; returns its path."""
    if not force and not _stale():
        return OUTPUT
    os.makedirs(OBJDIR, exist_ok=True)
    objs = [os.path.join(OBJDIR, s.replace(".cu", ".o")) for s in SOURCES]
    cmds = [[NVCC, *compile_flags(s), *(["-Xptxas", "-v"] if verbose else []), "-c", os.path.join(CSRC, s), "-o", o]
            for s, o in zip(SOURCES, objs)]
    with ThreadPoolExecutor(max_workers=len(cmds)) as pool:
        results = list(pool.map(lambda c: _run(c, verbose), cmds))
    for cmd, res in zip(cmds, results):
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError(f"nvcc failed ({res.returncode}): {' '.join(cmd)}")
    link = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", OUTPUT, *objs]
    res = _run(link, verbose)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc link failed ({res.returncode}) building {OUTPUT}")
    return OUTPUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
