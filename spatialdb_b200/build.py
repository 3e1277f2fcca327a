"""Builds libslx.so (the sm_100a kernels and the C ABI) in-tree under spatialdb_b200/_build/.

nvcc compiles each source for sm_100a only (-gencode arch=compute_100a,code=sm_100a); the host
compiler runs without floating-point contraction so the fp32 stages keep the reference's
sequential multiply-then-add rounding.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT_DIR = os.path.join(PKG, "_build")
LIB = os.path.join(OUT_DIR, "libslx.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: libslx needs the CUDA toolkit to build")


def _flags() -> list[str]:
    return ARCH + [
        "-O3", "-lineinfo", "-std=c++17", "--fmad=false", "-ccbin", "g++",
        "-Xcompiler", "-fPIC,-ffp-contract=off,-fno-fast-math",
        "-I", INCLUDE, "-I", CSRC,
    ]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _deps() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(CSRC, "*.hpp")) + glob.glob(os.path.join(INCLUDE, "*.h")) + [__file__]


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in _deps())


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> str:
    """Compile every source to an object and link libslx.so. Returns the library path."""
    if not force and not stale():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    nvcc = _nvcc()
    flags = _flags()

    def compile_one(src: str) -> str:
        obj = os.path.join(OUT_DIR, os.path.basename(src) + ".o")
        cmd = [nvcc] + flags + ["-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stderr[-6000:]}")
        if verbose and r.stderr:
            print(r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB + ".tmp"
    cmd = [nvcc] + ARCH + ["-shared", "-ccbin", "g++", "-o", tmp] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr[-4000:]}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import sys

    print(build(force="-f" in sys.argv, verbose="-v" in sys.argv))
