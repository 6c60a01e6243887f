"""Builds libswiftlet_cuda.so in-tree with nvcc for sm_100a.

Each translation unit is compiled to an object in parallel, then linked.
Usage: python -m swiftlet_b200.build [--verbose]
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libswiftlet_cuda.so")
OBJ = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")) + glob.glob(os.path.join(HERE, "csrc", "*.cpp")))


def headers() -> list[str]:
    return (glob.glob(os.path.join(HERE, "csrc", "*.h")) + glob.glob(os.path.join(HERE, "csrc", "*.cuh"))
            + [os.path.join(ROOT, "include", "swiftlet_cuda.h")])


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in sources() + headers())


def _nvcc() -> str:
    return os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def _compile(src: str, verbose: bool, force: bool = True) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if not force and os.path.exists(obj):
        t = os.path.getmtime(obj)
        if all(os.path.getmtime(p) <= t for p in [src] + headers()):
            return obj
    cmd = [_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O3",
           "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    os.makedirs(OBJ, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, force), sources()))
    subprocess.run([_nvcc(), *ARCH, "-shared", "-o", LIB + ".tmp", *objs], check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force=True)
