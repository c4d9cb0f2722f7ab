"""Builds the in-tree CUDA library elips_b200/libelips_b200.so for sm_100a.

Usage: python elips_b200/build.py [--verbose] [--ptxas-info]
(run as a file: importing the package itself loads the library this builds)

nvcc cross-compiles without a GPU. The library is written next to this file so
it ships with the source tree; the C runtime is linked statically.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libelips_b200.so"

SOURCES = ["engine.cu", "capi.cu", "noalloc.cu", "quant.cu", "ivfpq.cu", "train.cu", "batcher.cu"]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def needs_build() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + [INCLUDE / "elips_b200.h", Path(__file__)]
    return any(p.stat().st_mtime > mtime for p in deps if p.exists())


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
           "-o", str(tmp), *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, ptxas_info="--ptxas-info" in sys.argv)
    print(LIB)
