"""Build the sm_100a library in-tree: stratametal_b200/libsmoe.so (nvcc, one translation unit).

The kernels compile for sm_100a only (-gencode arch=compute_100a,code=sm_100a); nvcc cross-compiles them
on a machine without a GPU.  Floating-point flags stay at nvcc's IEEE defaults (no fast math: the q8_1 rule
needs the correctly rounded division, and the reference's sums are reproduced operation by operation).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
SRC = PKG / "csrc" / "smoe_lib.cu"
OUT = PKG / "libsmoe.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17", "-shared",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-O2"]


def sources() -> list[Path]:
    return sorted((PKG / "csrc").glob("*.cu")) + sorted((PKG / "csrc").glob("*.cuh")) + \
        sorted((PKG / "csrc").glob("*.inc")) + [PKG.parent / "include" / "smoe.h"]


def needs_build() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and not needs_build():
        return OUT
    cmd = [NVCC, *FLAGS, *(extra or []), "-o", str(OUT), str(SRC)]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
    if verbose and r.stderr:
        print(r.stderr)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, extra=["-Xptxas", "-v"] if "-v" in sys.argv else None)
    print(OUT)
