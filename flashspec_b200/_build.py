"""Compile the native library ``libflashspec_b200.so`` in-tree with nvcc for sm_100a.

The library is plain C ABI (``include/flashspec_b200.h``); no torch headers are
involved, so the build is a direct nvcc invocation per source file plus a link.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libflashspec_b200.so"
SOURCES = ["decode.cu", "decode_generic.cu", "quant.cu", "noalloc.cu", "exchange.cu", "probe.cu", "tree.cu"]
HEADERS = ["ptx.cuh", "common.h", "generic.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", f"-I{ROOT / 'include'}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / "include" / "flashspec_b200.h", Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Build (if stale) and return the path of the shared library."""
    if not force and not _stale():
        return LIB
    BUILD.mkdir(exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = BUILD / (Path(src).stem + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
