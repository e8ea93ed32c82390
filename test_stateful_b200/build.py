"""Build ``libqtts_b200.so`` (all sm_100a kernels + the C ABI) in-tree with nvcc.

The library is a single translation unit (``csrc/qtts.cu``) compiled for
``sm_100a`` only; the CUDA runtime is linked statically, so the .so depends on
the driver alone and travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libqtts_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "qtts_b200.h"]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources())


def build(force: bool = False, verbose: bool = False, extra=None) -> Path:
    if not force and up_to_date():
        return LIB
    cmd = [nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
           "-I", str(PKG.parent / "include"),
           "-o", str(LIB) + ".tmp", str(CSRC / "qtts.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    if extra:
        cmd[1:1] = list(extra)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed for libqtts_b200.so")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
