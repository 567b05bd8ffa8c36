"""Build libabx (the sm_100a kernels behind include/abx.h) in-tree with nvcc.

    python -m adambridge_b200._build [--force] [--verbose]

The library lands in ``adambridge_b200/_lib/libabx.so`` (next to this package, so a
copy of the repository carries it).  It links the CUDA runtime statically, so it
needs no libcudart on the loader path; the CUDA driver of the machine it runs on
provides the rest.

Compiler flags that matter for results: ``-fmad=false -ftz=false -prec-div=true
-prec-sqrt=true`` keep every floating-point operation IEEE round-to-nearest with
subnormals, so the only fused multiply-adds are the ones the source spells out.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIBDIR = PKG / "_lib"
LIB = LIBDIR / "libabx.so"
SOURCES = [CSRC / "abx_kernels.cu", CSRC / "abx_clip.cu", CSRC / "abx_convert.cu"]
DEPENDS = SOURCES + [CSRC / "abx_device.cuh", INCLUDE / "abx.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
         "-Xcompiler", "-fPIC,-fvisibility=hidden,-O2", "--cudart", "static", "-shared"]


def nvcc() -> str:
    cand = os.environ.get("ABX_NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: set ABX_NVCC or put the CUDA toolkit's bin on PATH")
    return cand


def _digest() -> str:
    h = hashlib.sha256()
    for f in DEPENDS:
        h.update(f.read_bytes())
    h.update(" ".join(ARCH + FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile libabx unless an up-to-date copy exists; returns its path."""
    stamp = LIBDIR / "libabx.sha256"
    digest = _digest()
    if not force and LIB.exists() and stamp.exists() and stamp.read_text().strip() == digest:
        return LIB
    LIBDIR.mkdir(exist_ok=True)
    tmp = LIBDIR / f".libabx.{os.getpid()}.so"
    cmd = [nvcc(), *ARCH, *FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-I", str(INCLUDE),
           *map(str, SOURCES), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        tmp.unlink(missing_ok=True)
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr}")
    if verbose and proc.stderr:
        print(proc.stderr, file=sys.stderr)
    os.replace(tmp, LIB)
    stamp.write_text(digest + "\n")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(LIB)
