"""Build libsiphon_cuda.so in-tree with nvcc for sm_100a.

    python -m siphon_b200.build            # builds siphon_b200/libsiphon_cuda.so

The library links the CUDA runtime statically, so it only needs the driver at
run time and shares the device's primary context with anything else in the
process (torch included).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
ROOT = PKG.parent
LIB = PKG / "libsiphon_cuda.so"

SOURCES = ["abi.cu", "gemv.cu", "gemv_batch.cu", "gemv_f16.cu", "quantize.cu", "noalloc.cu", "prefill.cu", "allreduce.cu", "prologue.cu", "softmax.cu", "tcpeak.cu"]
HEADERS = ["common.cuh", "gemv.cuh", "quantize.cuh", "launch.h", "tc.cuh", "allreduce.cuh", "prologue.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / "include" / "siphon_cuda.h"]
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every source to an object (in parallel), then link the shared
    library; rebuilds only when a source or header is newer than it."""
    if not force and not stale():
        return LIB
    from concurrent.futures import ThreadPoolExecutor
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    flags = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
             "-I", str(ROOT / "include")]
    if os.environ.get("SICU_PTXAS_VERBOSE"):
        flags.insert(0, "-Xptxas=-v")

    def compile_one(src: str) -> Path:
        obj = objdir / (Path(src).stem + ".o")
        cmd = [nvcc(), *flags, "-c", "-o", str(obj), str(CSRC / src)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB) + ".tmp", *map(str, objs)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
