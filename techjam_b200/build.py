"""Build ``libtj.so`` (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m techjam_b200.build          # or: from techjam_b200.build import build; build()

The library is written next to this file so it travels with the source tree;
nothing is installed into site-packages or a JIT cache.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libtj.so"
SOURCES = ["tj_api.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build libtj.so")


def _inputs():
    return [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "tj.h"]


def is_stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _inputs())


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> Path:
    """Compile ``libtj.so`` if any source is newer than it (or ``force``)."""
    if not force and not is_stale():
        return LIB
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr", "-I", str(PKG.parent / "include"),
           *(extra_flags or []), "-o", str(LIB) + ".tmp", *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr}\n{res.stdout}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(LIB)
