"""Builds ``libmote_cuda.so`` (the C ABI in ``include/mote_cuda.h``) in-tree.

The library is one CUDA translation unit compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); it cross-compiles on hosts
without a GPU.  ``MOTE_CUDA_ARCH`` overrides the architecture string and
``NVCC`` the compiler, mirroring ``MOTE_HIP_ARCH`` / ``HIPCC`` of the HIP
backend's build script (crates/mote-backend-hip/build.rs:7-9,36-92).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_PATH = PKG / "libmote_cuda.so"
ENTRY = CSRC / "libmote_cuda.cu"


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def command(out: Path = LIB_PATH, extra: list[str] | None = None) -> list[str]:
    arch = os.environ.get("MOTE_CUDA_ARCH", "100a")
    return [
        nvcc_path(),
        "-gencode", f"arch=compute_{arch},code=sm_{arch}",
        "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-shared",
        "-I", str(PKG.parent / "include"),
        "-o", str(out), str(ENTRY),
        *(extra or []),
    ]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + \
        [PKG.parent / "include" / "mote_cuda.h"]


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > built for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not is_stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = command(tmp)
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    tmp.replace(LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB_PATH)
