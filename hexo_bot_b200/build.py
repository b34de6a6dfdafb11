"""Build recipe for the native library (sm_100a only).

    python -m hexo_bot_b200.build          # -> hexo_bot_b200/_native/libshrimp_b200.so

nvcc cross-compiles for sm_100a without a GPU. The library is written in-tree
so it travels with the repository snapshot to the GPU machine.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_native"
LIB_NAME = "libshrimp_b200.so"
SOURCES = ["api.cu"]
HEADERS = ["ptx.cuh", "gemm.cuh", "conv_ts.cuh", "conv_grid.cuh", "mlp.cuh", "attention.cuh", "attention_geo.cuh", "aux.cuh"]
INCLUDE = PKG.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build shrimp_b200")
    return cand


def lib_path() -> Path:
    return OUT_DIR / LIB_NAME


def _inputs() -> list[Path]:
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [INCLUDE / "shrimp_b200.h"]


def is_stale() -> bool:
    out = lib_path()
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    out = lib_path()
    if not force and not is_stale():
        return out
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True)
    print(p)
