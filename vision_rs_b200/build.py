"""Build ``libvisionattn.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m vision_rs_b200.build          # or: python vision_rs_b200/build.py

Every ``csrc/*.cu`` is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` into ``_build/`` and
linked into ``vision_rs_b200/libvisionattn.so`` (static cudart, no torch
dependency).  Rebuilds only what changed.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libvisionattn.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                  "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps(src: str) -> list[str]:
    return [src] + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def build(verbose: bool = False, extra: list[str] | None = None) -> str:
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in _deps(src)):
            continue
        cmd = [nvcc, *NVFLAGS, *(extra or []), "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
