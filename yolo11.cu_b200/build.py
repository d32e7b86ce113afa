"""Build the native engine in-tree for sm_100a.

    lib/libyolob200.so   engine + kernels behind include/yolo.h and include/yk.h
    bin/yolocuda         CLI (detect / pipeline / bench / profile / dump), links the library

Rebuilds only when a source under csrc/ or include/ is newer than the target.
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "lib", "libyolob200.so")
CLI = os.path.join(PKG, "bin", "yolocuda")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC"]


def _sources():
    out = []
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in sorted(os.listdir(d)):
            if f.endswith((".cu", ".cuh", ".h", ".cpp")):
                out.append(os.path.join(d, f))
    return out


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)


def build(force: bool = False, verbose: bool = False) -> str:
    deps = _sources()
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    os.makedirs(os.path.dirname(CLI), exist_ok=True)
    if force or _stale(LIB, deps):
        if verbose:
            print("nvcc ->", LIB, flush=True)
        tmp = LIB + ".tmp"
        _run([NVCC, *ARCH, *FLAGS, "-shared", os.path.join(CSRC, "libyolob200.cu"), "-o", tmp,
              "-lnvjpeg"])
        os.replace(tmp, LIB)
    if force or _stale(CLI, deps + [LIB]):
        if verbose:
            print("nvcc ->", CLI, flush=True)
        _run([NVCC, *ARCH, "-O2", "-std=c++17", os.path.join(CSRC, "yolocuda.cpp"),
              "-L" + os.path.dirname(LIB), "-lyolob200", "-Xlinker",
              "-rpath=$ORIGIN/../lib", "-o", CLI])
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
