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
SOURCES = [CSRC / "engine.cu", CSRC / "noalloc.cu", CSRC / "kernels_select.cu", CSRC / "kernels_tc.cu",
           CSRC / "kernels_proj_ln.cu", CSRC / "kernels_proj_rows.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [ROOT / "include" / "s2r.h"]
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
    """Compile every translation unit in parallel, then link the shared library."""

    if not force and not stale():
        return LIB
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    flags = [*ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include")]
    procs = []
    for src in SOURCES:
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc(), *flags, "-Xptxas", "-v" if verbose else "-O3", "-c", str(src), "-o", str(obj)]
        procs.append((src, obj, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
    failed = []
    for src, obj, proc in procs:
        out, err = proc.communicate()
        if proc.returncode != 0:
            failed.append(f"{src.name} ({proc.returncode}):\n{out}\n{err}")
        elif verbose:
            sys.stderr.write(err)
    if failed:
        raise RuntimeError("nvcc failed: " + "\n".join(failed))
    link = [nvcc(), *ARCH, "-shared", *[str(obj) for _, obj, _ in procs], "-o", str(LIB) + ".tmp"]
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
