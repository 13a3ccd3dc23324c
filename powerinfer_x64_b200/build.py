"""Builds the sm_100a C-ABI library ``libpi_moe.so`` in-tree.

Each ``csrc/*.cu`` file is compiled with nvcc for ``sm_100a`` only and the
objects are linked into ``powerinfer_x64_b200/_lib/libpi_moe.so``. Objects are
rebuilt when their source or any header changed. Run ``python -m
powerinfer_x64_b200.build`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libpi_moe.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}"]


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def build(verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    hm = _headers_mtime()
    objs = []
    for src in sorted(CSRC.glob("*.cu")):
        obj = OBJ / (src.stem + ".o")
        objs.append(obj)
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hm):
            continue
        cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
    print(LIB)
