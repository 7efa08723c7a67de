"""Builds librevk.so (the C-ABI kernel library) in-tree with nvcc for sm_100a.

Usage: ``python -m reversability_b200.build`` (or ``build()`` from Python).
Each ``csrc/*.cu`` compiles to an object in ``_build/`` in parallel, then the
objects link into ``reversability_b200/librevk.so`` with the CUDA runtime
linked statically, so the library loads without a matching libcudart. A
rebuild happens only when a source or header is newer than the library.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "librevk.so"
INCLUDE = ROOT / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-diag-suppress", "20044"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build librevk")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    newest = max(p.stat().st_mtime for p in [*CSRC.glob("*.cu"), *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")])
    return newest > LIB.stat().st_mtime


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{result.stdout}\n{result.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every kernel for sm_100a and links librevk.so; returns its path."""
    if not force and not _stale():
        return LIB
    BUILD.mkdir(exist_ok=True)
    sources = _sources()
    workers = min(len(sources), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=workers) as pool:
        objects = list(pool.map(lambda s: _compile(s, verbose), sources))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "--cudart", "static", "-o", str(tmp), *map(str, objects)]
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
