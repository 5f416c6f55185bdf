"""Builds the sm_100a shared library of the hot path (lib/libt8b.so) with nvcc.

Every .cu under csrc/ becomes one object; the engine translation unit is compiled with
--fmad=false (a fused multiply-add would round once where the reference CPU engine rounds
twice). Objects go to _build/ and are rebuilt when a source or header is newer.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "lib" / "libt8b.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
          f"-I{ROOT / 'include'}", f"-I{CSRC}"]
# Per-source extra flags.
EXTRA = {"sim.cu": ["--fmad=false"]}


def _newest_header() -> float:
    headers = list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in headers), default=0.0)


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    newest_header = _newest_header()
    objects = []
    for source in sorted(CSRC.glob("*.cu")):
        obj = BUILD / (source.stem + ".o")
        objects.append(obj)
        if obj.exists() and obj.stat().st_mtime >= max(source.stat().st_mtime, newest_header):
            continue
        cmd = [NVCC, *ARCH, *COMMON, *EXTRA.get(source.name, []), "-c", str(source), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objects):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objects), "-lcudart", "-lcuda", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
