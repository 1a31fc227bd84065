"""Build libpraxis_b200_moe.so in-tree with nvcc for sm_100a.

The library is one CUDA translation unit (csrc/praxis_b200_moe.cu) with a C
ABI (include/praxis_b200_moe.h); it links the CUDA runtime statically and
has no torch dependency. ``python -m`` style entry: ``python build.py``.
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
LIB_NAME = "libpraxis_b200_moe.so"
LIB_PATH = PKG / LIB_NAME
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA 12.9 toolkit is required to build the library")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [
        INCLUDE / "praxis_b200_moe.h"
    ]


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    built = LIB_PATH.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if any source is newer than the .so."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        nvcc(),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-shared",
        "-I",
        str(INCLUDE),
        "-o",
        str(tmp),
        str(CSRC / "praxis_b200_moe.cu"),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr[-4000:]}")
    if verbose:
        print(proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
