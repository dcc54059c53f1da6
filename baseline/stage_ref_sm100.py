#!/usr/bin/env python
"""Stage the reference's own SM100 routed-expert pair into baseline/_ref/.

The same-box comparison (baseline/ref_sm100.py, bench.py --impl ref-sm100 and
tests/test_gpu_ref_sm100.py) runs sgl-nvidia-mega's RoutedExpertGemm
(deepseek_v41/sm103/moe/routed_expert_gemm.py: gate_topk.cu, route.cu,
route_wide.cu, gemm1.cu, gemm2.cu, compiled by NVRTC on the GPU) unmodified.
Only the files that module imports are copied, byte for byte, from a checkout
of the reference given on the command line (or in MM_REFERENCE_ROOT):

    sgl_nvidia_mega/__init__.py
    sgl_nvidia_mega/common/__init__.py, common/jit.py
    sgl_nvidia_mega/deepseek_v41/__init__.py, deepseek_v41/sm103/__init__.py
    sgl_nvidia_mega/deepseek_v41/sm103/moe/ (Python files and src/)

baseline/_ref/ is git-ignored (nothing of the reference enters the history) and
travels to the GPU box with the working tree. The rest of the reference stays
out on purpose: the staged tree must name no TMA load with cluster multicast,
because runs on two or more GPUs carry it too; a file that does is refused.

Usage: python baseline/stage_ref_sm100.py --reference <checkout of sgl-nvidia-mega>
"""

from __future__ import annotations

import argparse
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
DEST = os.path.join(HERE, "_ref")
FILES = [
    "sgl_nvidia_mega/__init__.py",
    "sgl_nvidia_mega/common/__init__.py",
    "sgl_nvidia_mega/common/jit.py",
    "sgl_nvidia_mega/deepseek_v41/__init__.py",
    "sgl_nvidia_mega/deepseek_v41/sm103/__init__.py",
]
TREES = ["sgl_nvidia_mega/deepseek_v41/sm103/moe"]
SUFFIXES = (".py", ".cu", ".cuh", ".json")


def _listing(reference: str):
    out = list(FILES)
    for tree in TREES:
        for root, dirs, names in os.walk(os.path.join(reference, tree)):
            dirs[:] = sorted(d for d in dirs if d != "__pycache__")
            for name in sorted(names):
                if name.endswith(SUFFIXES):
                    out.append(os.path.relpath(os.path.join(root, name), reference))
    return out


def stage(reference: str) -> int:
    if not os.path.isfile(os.path.join(reference, "sgl_nvidia_mega", "__init__.py")):
        raise SystemExit(f"{reference}: not a checkout of sgl-nvidia-mega (no sgl_nvidia_mega/__init__.py)")
    files = _listing(reference)
    for rel in files:
        with open(os.path.join(reference, rel), "rb") as f:
            if b"multicast" in f.read().lower():
                raise SystemExit(f"refusing to stage {rel}: it names a multicast load")
    if os.path.isdir(DEST):
        shutil.rmtree(DEST)
    for rel in files:
        dst = os.path.join(DEST, rel)
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        shutil.copyfile(os.path.join(reference, rel), dst)
    return len(files)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MM_REFERENCE_ROOT"),
                    help="checkout of sgl-nvidia-mega (default: $MM_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or MM_REFERENCE_ROOT) is required")
    n = stage(os.path.abspath(args.reference))
    print(f"staged {n} files of the reference into {DEST}")


if __name__ == "__main__":
    sys.exit(main())
