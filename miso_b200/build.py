"""Builds the sm_100a CUDA library in-tree: miso_b200/lib/libmiso_b200.so.

One nvcc invocation over csrc/capi.cu (which includes every kernel header), compiled for
sm_100a only. The library is written next to the sources so it travels with the repository
snapshot; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(os.path.dirname(ROOT), "include")
LIB_DIR = os.path.join(ROOT, "lib")
LIB = os.path.join(LIB_DIR, "libmiso_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2", "-shared",
    "-Xptxas", "-warn-spills",
]


def _sources() -> list[str]:
    out = []
    for base, _dirs, files in os.walk(CSRC):
        for f in files:
            if f.endswith((".cu", ".cuh", ".hpp", ".h")):
                out.append(os.path.join(base, f))
    out.append(os.path.join(INCLUDE, "miso_cuda.h"))
    return out


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(s) > t for s in _sources())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles the library if any source is newer than it; returns its path."""
    if not force and not stale():
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    nvcc = os.environ.get("NVCC", "nvcc")
    tmp = LIB + ".tmp"
    cmd = [nvcc, *NVCC_FLAGS, f"-I{CSRC}", f"-I{INCLUDE}", "-o", tmp,
           os.path.join(CSRC, "capi.cu")]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
