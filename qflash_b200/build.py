"""Build the C-ABI CUDA library ``libqflash_b200.so`` in-tree for sm_100a.

    python -m qflash_b200.build [--force]

nvcc compiles each ``csrc/*.cu`` to an object under ``_build/`` and links
the shared library (cudart linked statically); nothing else is needed at run
time besides the driver.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libqflash_b200.so"
SOURCES = [CSRC / "qflash_fwd.cu", CSRC / "qflash_quant.cu", CSRC / "qflash_noalloc.cu", CSRC / "qflash_peak.cu",
           CSRC / "qflash_peer.cu"]
HEADERS = [CSRC / "sm100_ptx.cuh", CSRC / "qfb_internal.h", PKG.parent / "include" / "qflash_b200.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


OBJDIR = PKG / "_build"


def _obj(src: Path) -> Path:
    return OBJDIR / (src.stem + ".o")


def _newer(a: Path, deps) -> bool:
    return not a.exists() or any(p.exists() and p.stat().st_mtime > a.stat().st_mtime for p in deps)


def stale() -> bool:
    return any(_newer(_obj(s), [s, *HEADERS]) for s in SOURCES) or _newer(LIB, [_obj(s) for s in SOURCES])


def _run(cmd, verbose):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile each source to an object (when it or a header changed), then
    link the shared library."""
    OBJDIR.mkdir(exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = _obj(src)
        if force or _newer(obj, [src, *HEADERS]):
            _run([nvcc(), *ARCH, *FLAGS, "-c", "-o", str(obj), str(src)], verbose)
        objs.append(obj)
    if force or _newer(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        _run([nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs)], verbose)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
