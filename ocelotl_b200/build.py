"""Build the sm_100a CUDA library (libocelotl_cuda.so) in-tree with nvcc.

The library holds every kernel of the quantized-linear path and the C ABI
declared in include/ocelotl_cuda.h.  It is built in place (next to this file) so
that it travels with the source tree; nothing is installed elsewhere.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libocelotl_cuda.so"

SOURCES = ["api.cu", "repack.cu", "gemv.cu", "noalloc.cu", "gemm.cu", "argmax.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + [ROOT / "include" / "ocelotl_cuda.h"]
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if _stale(o, [s] + headers) or ptxas_verbose:
            cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-c", str(s), "-o", str(o)]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
    if _stale(LIB, objs):
        cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *map(str, objs),
               "-o", str(LIB), "-lcudart"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_verbose="-v" in sys.argv)
