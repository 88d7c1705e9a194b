"""Builds librldx_b200.so (all sm_100a kernels + the C ABI) in this package directory.

The library is one nvcc translation unit (csrc/rldx_b200.cu) compiled for sm_100a only:
no PTX for other architectures is embedded, so it loads only on B200-class GPUs.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
LIB_NAME = "librldx_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-shared",
]


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))) + [
        PKG_DIR.parent / "include" / "rldx_b200.h"
    ]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    lib_mtime = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > lib_mtime for p in _sources() if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the library if a source is newer than the .so (or when forced)."""
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, str(CSRC / "rldx_b200.cu"), "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, cwd=str(CSRC), capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB_PATH)
