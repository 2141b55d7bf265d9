"""Build libgafime_cuda.so in-tree for sm_100a (B200).

    python -m gafime_b200.build          # or gafime_b200.build.build()

nvcc compiles every .cu under csrc/ with ``-gencode arch=compute_100a,code=sm_100a``
and links them into gafime_b200/libgafime_cuda.so (cudart linked statically, so the
library loads with ctypes without a CUDA toolkit on the library path).  The build is
incremental on source mtimes.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OBJ_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libgafime_cuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -fno-tree-loop-vectorize: g++ 13.3's loop vectorizer miscompiles a short loop that fills
# per-operator arrays from a two-entry table (a wrong element read, reproduced standalone at
# -O3); host code here is not throughput-bound, so the host side is built without it.
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fno-tree-loop-vectorize",
              "--expt-relaxed-constexpr",
              "-ccbin", "/usr/bin/g++"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA 12.9 toolkit is required to build libgafime_cuda.so")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers_mtime() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    nvcc = _nvcc()
    os.makedirs(OBJ_DIR, exist_ok=True)
    hdr = _headers_mtime()
    objs = []
    for src in sources():
        obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
        objs.append(obj)
        if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr) \
                and not ptxas_info:
            continue
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-c", src, "-o", obj]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [nvcc, *ARCH, "-shared", "-ccbin", "/usr/bin/g++", "-o", LIB, *objs]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="-v" in sys.argv))
