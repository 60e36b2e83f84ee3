"""Builds libtechjam_b200.so (sm_100a) in-tree with nvcc.

The library is one translation unit (csrc/api.cu includes the kernel files)
with the CUDA runtime linked statically, so it loads on a machine without a
GPU (the C-ABI symbol test) and on the B200 box without a JIT cache.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
REPO = PKG_DIR.parent
INCLUDE = REPO / "include"
LIB_NAME = "libtechjam_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build the library")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [
        INCLUDE / "techjam_b200.h"
    ]


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    lib_mtime = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > lib_mtime for p in sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "--shared",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        "-cudart",
        "static",
        "-I",
        str(INCLUDE),
        "-o",
        str(tmp),
        str(CSRC / "api.cu"),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    if extra:
        cmd[1:1] = extra
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(
            "nvcc failed (%d):\n%s\n%s" % (proc.returncode, " ".join(cmd), proc.stderr[-8000:])
        )
    if verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
