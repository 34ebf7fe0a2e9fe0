"""Builds libvmps_kernels.so in-tree with nvcc for sm_100a.

``python -m vllm_mps_b200.build`` (or ``build_kernels()``) compiles every
``csrc/*.cu`` into ``vllm_mps_b200/libvmps_kernels.so``.  The library is a
plain C-ABI shared object (see ``include/vmps.h``); it statically links the
CUDA runtime and resolves driver entry points at run time, so it needs no
libcuda at link time and builds on a machine without a GPU.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libvmps_kernels.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
    "-shared",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put it on PATH)")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(PKG_DIR, "csrc", "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = sources() + glob.glob(os.path.join(PKG_DIR, "csrc", "*.cuh")) + \
        glob.glob(os.path.join(PKG_DIR, "csrc", "*.h")) + \
        glob.glob(os.path.join(PKG_DIR, "..", "include", "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build_kernels(force: bool = False, verbose: bool = False) -> str:
    """Compile the CUDA sources into the in-tree shared library; return its path."""
    if not force and not _stale():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", tmp, *sources()]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build_kernels(force="--force" in sys.argv, verbose=True))
