"""In-tree build of libcheetah_cuda.so for sm_100a (nvcc cross-compiles
without a GPU). The built library sits next to this file and travels with the
repository snapshot to the GPU box.

Profiling builds add defines and write another library, which
CHEETAH_CUDA_LIB then selects, e.g.

    python -m cheetah_b200.build --define CHEETAH_ATTN_TRACE \
        --out cheetah_b200/libcheetah_cuda_attn_trace.so
"""

from __future__ import annotations

import argparse
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


def build(force: bool = False, verbose: bool = False, defines=(), out: Path | None = None) -> Path:
    """Compile the CUDA backend if any source is newer than the library
    (always when `defines` or `out` are given: a profiling build)."""
    target = Path(out) if out is not None else LIB
    if not force and not defines and out is None and not _stale():
        return LIB
    sources = [str(CSRC / s) for s in SOURCES]
    cmd = [nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
           "-I", str(INCLUDE), "-I", str(CSRC),
           "--expt-relaxed-constexpr",
           *[f"-D{d}" for d in defines],
           "-o", str(target) + ".tmp", *sources]
    if os.environ.get("CHEETAH_PTXAS_VERBOSE"):
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + (res.stderr or "") + (res.stdout or ""))
    os.replace(str(target) + ".tmp", target)
    return target


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--define", action="append", default=[], help="preprocessor define (repeatable)")
    ap.add_argument("--out", default=None, help="library path (default: the in-tree libcheetah_cuda.so)")
    a = ap.parse_args()
    print(build(force=True, verbose=True, defines=a.define, out=a.out))
