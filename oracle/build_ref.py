"""Build oracle/_ref/libref_coop.so from the reference checkout — test infrastructure only.

Compiles oracle/ref_harness.cu (this repository's launcher) with the reference's vendored EXL3 /
MoE coop headers included in place from <reference>/runtime/ds41/csrc/moe_coop2048 (nothing is
copied). The headers use torch's c10 headers for TORCH_CHECK and cuBLAS headers, so torch's include
directories are added; nothing from torch is linked. Output goes only to oracle/_ref/ (git-ignored,
travels to the GPU box with the tree).

Usage: python oracle/build_ref.py [/path/to/reference]   (default: $EVA_REFERENCE, else ../reference)
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "libref_coop.so"


def reference_root() -> Path | None:
    """The reference checkout: $EVA_REFERENCE, else a folder named `reference` beside this repository."""
    env = os.environ.get("EVA_REFERENCE")
    if env:
        return Path(env)
    sibling = HERE.parent.parent / "reference"
    return sibling if sibling.is_dir() else None


def main():
    ref = Path(sys.argv[1]) if len(sys.argv) > 1 else reference_root()
    if ref is None:
        print("no reference checkout (argument, EVA_REFERENCE, or a 'reference' folder beside this repository); "
              "oracle/_ref not built")
        return 1
    src = ref / "runtime" / "ds41" / "csrc" / "moe_coop2048"
    if not (src / "vendor" / "quant" / "exl3_moe_coop_kernel.cuh").exists():
        print(f"reference sources not found under {src}; oracle/_ref not built")
        return 1
    import torch.utils.cpp_extension as ce
    incs = ce.include_paths()
    OUT.parent.mkdir(exist_ok=True)
    cmd = ["/usr/local/cuda/bin/nvcc", "-O3", "-std=c++20", "--expt-relaxed-constexpr", "-lineinfo",
           "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC", "-shared",
           "-I", str(src), *[f"-I{p}" for p in incs], str(HERE / "ref_harness.cu"), "-o", str(OUT)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode:
        sys.stderr.write(res.stdout + res.stderr)
        print("oracle/_ref build failed")
        return 2
    print(OUT)
    return 0


if __name__ == "__main__":
    sys.exit(main())
