"""Builds the sm_100a kernel library ``bloth_b200/libbloth_b200.so`` in-tree.

Each ``csrc/*.cu`` file is compiled to an object under ``_build/`` (in
parallel, skipped when newer than every source and header), then linked
with the static CUDA runtime into one shared library that exports the
C ABI of ``include/bloth_b200.h``.

Run ``python -m bloth_b200.build`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
BUILD_DIR = os.path.join(REPO_DIR, "_build")
LIB_NAME = "libbloth_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-I" + INCLUDE,
] + ARCH


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build bloth_b200")


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, jobs: int | None = None, extra_flags: list[str] | None = None) -> str:
    """Compiles and links the library if anything changed; returns its path."""
    nvcc = nvcc_path()
    os.makedirs(BUILD_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = _headers()
    flags = NVCC_FLAGS + list(extra_flags or [])

    def compile_one(src: str) -> str:
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        if _stale(obj, [src, __file__] + headers):
            cmd = [nvcc, *flags, "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
            if verbose and (res.stdout or res.stderr):
                print(res.stdout + res.stderr, flush=True)
        return obj

    workers = jobs or max(1, min(len(sources), os.cpu_count() or 1))
    with ThreadPoolExecutor(max_workers=workers) as ex:
        objs = list(ex.map(compile_one, sources))

    if _stale(LIB_PATH, objs):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc, "-shared", *ARCH, "-Xcompiler", "-fPIC", "-o", tmp, *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv)
    print(path)
