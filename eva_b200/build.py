"""Build libeva_moe.so (all CUDA translation units) in-tree for sm_100a with nvcc.

The library has no torch dependency: it links only the CUDA runtime. The output lands next to
this file (eva_b200/libeva_moe.so) so that it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libeva_moe.so"
SOURCES = ["capi.cu", "routing.cu", "router_tc.cu", "experts.cu", "prefill.cu", "noalloc.cu", "ep.cu", "stack.cu",
           "decode_bench.cu", "residency.cu"]
HEADERS = ["common.cuh", "internal.h", "tc.cuh", "decode_tc.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [PKG.parent / "include" / "eva_moe.h"]
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    flags = ["-O3", "-std=c++17", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC", "-shared",
             "--expt-relaxed-constexpr", "-I", str(PKG.parent / "include")]
    if verbose:
        flags += ["-Xptxas", "-v"]
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *flags, *[str(CSRC / s) for s in SOURCES], "-o", str(tmp), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libeva_moe.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
