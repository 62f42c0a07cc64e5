"""Builds the native library of the paged-KV path: ``vllm_b200/_lib/libtvp_paged.so``.

Every CUDA translation unit is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) with the CUDA runtime linked
statically, so the library has no dependency on torch or on a particular
libcudart; nvcc cross-compiles without a GPU.  Objects go to
``vllm_b200/_build/`` and are rebuilt when a source or header is newer.

Usage: ``python -m vllm_b200.build [--force]``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libtvp_paged.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["tvp_append.cu", "tvp_decode.cu", "tvp_decode_heads.cu", "tvp_compat.cu", "tvp_capi.cu", "tvp_host.cpp",
           "tvp_noalloc.cu", "tvp_gather.cu", "tvp_prefill.cu", "tvp_argmax.cu",
           "tvp_project.cu"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build vllm_b200")
    return cand


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h")) + sorted(INCLUDE.glob("*.hpp"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    headers = _headers()
    objs = []
    for src in SOURCES:
        path = CSRC / src
        obj = BUILD / (src + ".o")
        objs.append(obj)
        if not force and not _stale(obj, [path, *headers]):
            continue
        cmd = [nvcc(), "-std=c++17", *ARCH, "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
               "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(path), "-o", str(obj)]
        if src.endswith(".cpp"):
            cmd[1:1] = ["-x", "cu"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
