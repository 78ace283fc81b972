"""Builds the C-ABI library ``aegaeon_b200/libaegaeon_b200.so`` for sm_100a with nvcc.

Every ``csrc/*.cu`` file is compiled to an object under ``aegaeon_b200/_build`` and linked with
the static CUDA runtime into one shared library whose exported symbols are the ``aeg_*``
functions declared in ``include/aegaeon_b200.h``. The library is built in-tree so that it
travels with the source tree; nothing is installed into site-packages.

Usage: ``python -m aegaeon_b200.build [--force]``.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD_DIR = os.path.join(PKG, "_build")
LIB_PATH = os.path.join(PKG, "libaegaeon_b200.so")
HEADER = os.path.join(ROOT, "include", "aegaeon_b200.h")

NVCC = os.environ.get("NVCC", os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"))
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                             "-I" + os.path.join(ROOT, "include")]


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return _sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [HEADER]


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _deps())


def _compile(src: str) -> str:
    obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
    cmd = [NVCC] + COMMON_FLAGS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(_compile, srcs))
    tmp = LIB_PATH + ".tmp"
    cmd = [NVCC] + ARCH_FLAGS + ["-shared", "-cudart", "static", "-o", tmp] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    if verbose:
        print(f"built {LIB_PATH}")
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
