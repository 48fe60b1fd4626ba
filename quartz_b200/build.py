"""Build the sm_100a shared library ``quartz_b200/libquartz_b200.so`` in-tree.

    python -m quartz_b200.build

nvcc cross-compiles for sm_100a on a host without a GPU. The library exports
the C ABI declared in include/quartz_b200.h.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
SRC = PKG / "csrc"
OUT = PKG / "libquartz_b200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def sources() -> list[Path]:
    return sorted(SRC.glob("*.cu")) + sorted(SRC.glob("*.cuh")) + [REPO / "include" / "quartz_b200.h"]


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    cmd = [nvcc(), *NVCC_FLAGS, f"-I{REPO / 'include'}", f"-I{SRC}",
           "-o", str(OUT), str(SRC / "qz_api.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
