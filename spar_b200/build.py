"""Builds libspar_b200.so (all CUDA sources, sm_100a) in-tree.

Run as ``python -m spar_b200.build``. nvcc cross-compiles without a GPU, so this also works on
CPU-only machines. Objects go to ``_build/`` at the repository root; the shared library is
written next to this file so it travels with the package.
"""
from __future__ import annotations

import concurrent.futures
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIBRARY = PKG / "libspar_b200.so"

SOURCES = [
    "layernorm.cu",
    "elementwise.cu",
    "softmax.cu",
    "cross_entropy.cu",
    "adamw.cu",
    "embedding.cu",
    "gemm.cu",
    "matmul.cu",
    "attention.cu",
    "compat.cu",
    "trainer.cu",
    "comm.cpp",
    "checkpoint.cpp",
    "batches.cu",
    "qknorm.cu",
]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC",
          f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))


def _compile(src: Path, obj: Path, newest_header: float, verbose: bool) -> None:
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
        return
    if src.suffix == ".cu":
        cmd = [NVCC, *ARCH, "-lineinfo", *COMMON, "-c", str(src), "-o", str(obj)]
    else:
        # host-only C++: no device code, so no target architecture to name
        cmd = [NVCC, *COMMON, "-Wno-deprecated-gpu-targets", "-x", "c++", "-c", str(src), "-o",
               str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    newest = max((h.stat().st_mtime for h in _headers()), default=0.0)
    srcs = [CSRC / s for s in SOURCES if (CSRC / s).exists()]
    objs = [BUILD / (s.name + ".o") for s in srcs]
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        list(pool.map(lambda so: _compile(so[0], so[1], newest, verbose), zip(srcs, objs)))
    if not LIBRARY.exists() or LIBRARY.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objs), "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIBRARY


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIBRARY)
