"""Build libhier_b200.so (all CUDA sources of the package) for sm_100a.

The library is built in-tree next to this file so that it travels with the
repository to the GPU machine.  ``python -m multics_b200.build`` rebuilds it;
``build(verbose=True)`` also prints ptxas register/shared-memory usage.
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
LIB = PKG / "libhier_b200.so"
SOURCES = ["hier_capi.cu", "hier_meta.cu", "hier_prep.cu", "hier_attn.cu", "hier_selftest.cu",
           "hier_cached.cu", "hier_tiled.cu", "hier_shard.cu", "hier_bwd.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def build(verbose: bool = False, force: bool = False) -> Path:
    srcs = [CSRC / s for s in SOURCES if (CSRC / s).exists()]
    deps = srcs + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [ROOT / "include" / "hier_b200.h"]
    if LIB.exists() and not force:
        newest = max(p.stat().st_mtime for p in deps)
        if LIB.stat().st_mtime >= newest:
            return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-I", str(ROOT / "include"), "-o", str(tmp), *map(str, srcs), "-lcudart"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libhier_b200.so")
    if verbose:
        sys.stdout.write(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force=True)
    print(LIB)
