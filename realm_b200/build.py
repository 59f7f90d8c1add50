"""Builds realm_b200/librealm_b200.so (sm_100a) in-tree with nvcc.

Usage: python realm_b200/build.py [--force]   (run by path: the package import needs the library)
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "librealm_b200.so")
SOURCES = ["gemv.cu", "attention.cu", "engine.cu", "sample.cu", "scheduler.cpp", "gguf.cpp"]
HEADERS = ["common.cuh", "quant.cuh", "gemv.cuh", "attention.cuh", "xfrag.cuh", "sample.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
         "-Xcompiler", "-fPIC"]


def _mtime(p: str) -> float:
    return os.path.getmtime(p) if os.path.exists(p) else 0.0


def _deps_mtime() -> float:
    files = [os.path.join(CSRC, h) for h in HEADERS]
    files.append(os.path.join(HERE, "..", "include", "realm_b200.h"))
    return max(_mtime(f) for f in files)


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    if force or _mtime(obj) < max(_mtime(path), _deps_mtime()):
        cmd = [NVCC, *FLAGS, "-c", path, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    if force or _mtime(LIB) < max(_mtime(o) for o in objs):
        # the exported C ABI keeps default visibility through the header's extern "C" block
        cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LIB, *objs,
               "-Xcompiler", "-fPIC", "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
