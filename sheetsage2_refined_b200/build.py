"""Build ``libs2r.so`` (the CUDA engine behind ``include/s2r.h``) in-tree.

    python -m sheetsage2_refined_b200.build        # or build() from Python

nvcc compiles for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``);
no GPU is needed to build.  The library links the CUDA runtime statically and
has no torch dependency.
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
LIB = PKG / "libs2r.so"
SOURCES = [CSRC / "engine.cu", CSRC / "noalloc.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "s2r.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the B200 engine needs the CUDA toolkit to build")


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    return any(p.stat().st_mtime > built for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    cmd = [
        nvcc(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
        "-Xptxas", "-v" if verbose else "-O3",
        "-I", str(ROOT / "include"), *map(str, SOURCES), "-o", str(LIB) + ".tmp",
    ]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
