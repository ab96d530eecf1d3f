"""Builds ``libnwd.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

Each ``csrc/*.cu`` file is compiled to an object under ``_build/`` (only when
it or a header changed) and the objects are linked into
``<package>/libnwd.so``.  The CUDA runtime is linked statically; the driver
API (TMA descriptor encoding) is reached through cudaGetDriverEntryPoint, so
the library needs no libcuda at link time and loads on machines without a GPU.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
BUILD_DIR = os.path.join(PKG_DIR, "_build")
LIB_PATH = os.path.join(PKG_DIR, "libnwd.so")
HOST_SRC = os.path.join(PKG_DIR, "host", "nwd_host.cc")
HOST_PATH = os.path.join(PKG_DIR, "nwd_host")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3,-Wall", "-I", INCLUDE, "-I", CSRC,
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile changed sources and relink libnwd.so; returns its path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = _headers()
    objects = []
    for src in sources:
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objects.append(obj)
        if ptxas_info or _stale(obj, [src] + headers):
            cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_info else []) + \
                ["-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if _stale(LIB_PATH, objects):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc()] + ARCH_FLAGS + ["-shared", "-Xcompiler", "-fPIC", "-o", tmp] + objects + \
            ["-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB_PATH)
    build_host(verbose)
    return LIB_PATH


def build_host(verbose: bool = False) -> str:
    """The C++ engine host (host/nwd_host.cc): links only libnwd.so, found next to it."""
    if _stale(HOST_PATH, [HOST_SRC, LIB_PATH, os.path.join(INCLUDE, "nwd.h")]):
        cxx = os.environ.get("CXX_HOST", "g++")
        tmp = HOST_PATH + ".tmp"
        cmd = [cxx, "-O2", "-std=c++17", "-Wall", "-Wextra", "-I", INCLUDE, HOST_SRC, "-o", tmp,
               "-L", PKG_DIR, "-lnwd", "-Wl,-rpath,$ORIGIN"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, HOST_PATH)
    return HOST_PATH


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="--ptxas" in sys.argv))
