"""In-tree build of libcheetah_cuda.so for sm_100a (nvcc cross-compiles
without a GPU). The built library sits next to this file and travels with the
repository snapshot to the GPU box."""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libcheetah_cuda.so"

SOURCES = ["cheetah_cuda.cu", "store.cpp"]
HEADERS = ["common.cuh", "gemv.cuh", "attention.cuh", "kernels_misc.cuh", "store.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [INCLUDE / "cheetah_cuda.h", Path(__file__)]
    deps += list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")) + list(CSRC.glob("*.h"))
    return any(d.exists() and d.stat().st_mtime > built for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the CUDA backend if any source is newer than the library."""
    if not force and not _stale():
        return LIB
    sources = [str(CSRC / s) for s in SOURCES]
    cmd = [nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
           "-I", str(INCLUDE), "-I", str(CSRC),
           "--expt-relaxed-constexpr",
           "-o", str(LIB) + ".tmp", *sources]
    if os.environ.get("CHEETAH_PTXAS_VERBOSE"):
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + (res.stderr or "") + (res.stdout or ""))
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
