"""Build libnovamlx_cuda.so in-tree with nvcc for sm_100a (no PyTorch involved).

Usage: python -m novamlx_b200.build  (or import and call build()).
Each .cu/.cpp under csrc/ is compiled to an object in parallel, then linked
into novamlx_b200/libnovamlx_cuda.so. Rebuilds only what changed.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libnovamlx_cuda.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-diag-suppress", "191", "-I", str(INCLUDE)]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall", "-I", str(INCLUDE)]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _deps(src: Path) -> list[Path]:
    return [p for p in CSRC.glob("*.h")] + [p for p in CSRC.glob("*.cuh")] + [INCLUDE / "nmx.h", src]


def _compile(src: Path) -> Path:
    obj = BUILD / (src.name + ".o")
    if obj.exists() and all(obj.stat().st_mtime >= d.stat().st_mtime for d in _deps(src)):
        return obj
    if src.suffix == ".cu":
        cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++", *CXX_FLAGS, "-I", "/usr/local/cuda/include", "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return obj


def build(verbose: bool = True) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(_compile, srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if LIB.exists() and LIB.stat().st_mtime >= newest:
        return LIB
    cmd = [_nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static", "-lrt",
           "-lpthread", "-ldl"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build()
    sys.exit(0)
