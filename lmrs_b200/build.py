"""Build the sm_100a C-ABI library ``lmrs_b200/liblmrs_quant.so`` in-tree.

One nvcc invocation over the unity translation unit ``csrc/lmrs_capi.cu``
(kernels + host dispatch), static CUDA runtime, no link-time libcuda (the TMA
descriptor encoder is fetched through the runtime's driver entry point), so
the library loads on a machine without a GPU and travels with the repository.
"""
from __future__ import annotations

import os
import pathlib
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
LIB = PKG / "liblmrs_quant.so"
SRC = PKG / "csrc" / "lmrs_capi.cu"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    return sorted((PKG / "csrc").glob("*.cu*")) + sorted((ROOT / "include").glob("*.h"))


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources())


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if pathlib.Path(cand).exists() else "nvcc"


def build_library(force: bool = False, verbose: bool = False) -> pathlib.Path:
    if not force and not stale():
        return LIB
    cmd = [nvcc(), "-std=c++17", *ARCH, "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-shared", "-cudart", "static",
           "-I", str(ROOT / "include"), "-o", str(LIB), str(SRC)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed building {LIB.name}")
    if verbose:
        sys.stderr.write(res.stderr)
    return LIB


if __name__ == "__main__":
    build_library(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
