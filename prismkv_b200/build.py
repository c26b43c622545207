"""Builds libprismkv_b200.so (sm_100a) in-tree with nvcc.

    python -m prismkv_b200.build [--verbose]

The library is the C ABI declared in include/prismkv_b200.h.  Flags:
sm_100a only; no fast-math, and --fmad=false so that every fused
multiply-add in the kernels is an explicit fmaf (the exact-parity kernels
depend on the written rounding steps).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libprismkv_b200.so"
SOURCES = ["capi.cu", "route.cu", "union.cu", "sparse_av.cu", "build.cu", "layout.cu", "p2p.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--fmad=false", "-Xcompiler", "-fPIC", "--extended-lambda"]


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every source in parallel and link the shared library."""
    if not force and not _stale():
        return LIB
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    procs, objs = [], []
    for src in SOURCES:
        obj = objdir / (Path(src).stem + ".o")
        objs.append(obj)
        cmd = [NVCC, *ARCH, *FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode:
            sys.stderr.write(out)
        if p.returncode:
            failed.append(src)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose="--verbose" in sys.argv)
    print(LIB)
