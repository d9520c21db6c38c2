"""Build the sm_100a shared library ``libmomentum_scan_b200.so`` in-tree with nvcc.

    python -m momentummamba_b200.build [--force]

The library is a plain C-ABI .so (include/momentum_scan_b200.h); Python reaches
it through ctypes (momentummamba_b200/_lib.py).  nvcc cross-compiles for
sm_100a on machines without a GPU.
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
LIB_NAME = "libmomentum_scan_b200.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
]
OBJ_DIR = os.path.join(PKG, "_build")


def _nvcc() -> str:
    cand = [os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"),
            shutil.which("nvcc") or ""]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found (set CUDA_HOME)")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def deps():
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def is_stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(d) > t for d in deps())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every .cu unit (in parallel) and link the shared library."""
    if not force and not is_stale():
        return LIB_PATH
    nvcc = _nvcc()
    os.makedirs(OBJ_DIR, exist_ok=True)
    inc = ["-I", os.path.join(ROOT, "include")]
    jobs = []
    for src in sources():
        obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc, *NVCC_FLAGS, *inc, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        jobs.append((obj, subprocess.Popen(cmd)))
    failed = [obj for obj, proc in jobs if proc.wait() != 0]
    if failed:
        raise RuntimeError("nvcc failed for " + ", ".join(os.path.basename(f) for f in failed))
    tmp = LIB_PATH + ".tmp"
    link = [nvcc, *NVCC_FLAGS, "--shared", "-o", tmp, *[obj for obj, _ in jobs]]
    if verbose:
        print(" ".join(link))
    subprocess.run(link, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
