"""In-tree build of libbfp200.so for sm_100a (B200).

nvcc cross-compiles without a GPU.  The library lands in bfp200/lib/ so it
travels with the source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

from ._lib import LIB_DIR, LIB_PATH

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))   # tinyllm-fpga_b200/
CSRC = os.path.join(PKG_ROOT, "csrc")
SOURCES = ["kernels.cu", "gemv.cu", "layer1.cu", "tc.cu", "sample.cu", "rtl.cu", "engine.cu", "noalloc.cu"]
HEADERS = ["bfp_device.cuh", "kernels.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC", "-shared"]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale():
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    inc = os.path.join(os.path.dirname(PKG_ROOT), "include", "bfp200.h")
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [inc]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False):
    """Compiles csrc/*.cu into bfp200/lib/libbfp200.so (sm_100a)."""
    if not force and not _stale():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc()] + ARCH + FLAGS + ["-o", tmp] + [os.path.join(CSRC, s) for s in SOURCES]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
