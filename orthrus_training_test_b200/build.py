"""Build the sm_100a shared library ``libklgemm.so`` in-tree with nvcc.

    python -m orthrus_training_test_b200.build

The library is one translation unit (``csrc/klg_capi.cu`` includes the kernel
and PTX headers) linked against the static CUDA runtime; at run time it needs
only the CUDA driver.  ``KLG_NVCC_FLAGS`` appends extra nvcc flags.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
SRC = PKG / "csrc" / "klg_capi.cu"
LIB = PKG / "libklgemm.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC=/path/to/nvcc)")


def sources():
    return [SRC] + sorted((PKG / "csrc").glob("*.cuh")) + [ROOT / "include" / "klgemm.h"]


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-I", str(ROOT / "include"), "-o", str(LIB) + ".tmp", str(SRC)]
    cmd += os.environ.get("KLG_NVCC_FLAGS", "").split()
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
