"""Build the sm_100a shared library ``quartz_b200/libquartz_b200.so`` in-tree.

    python -m quartz_b200.build

nvcc cross-compiles for sm_100a on a host without a GPU. The library exports
the C ABI declared in include/quartz_b200.h.
"""

from __future__ import annotations

import os
import re
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


RESOURCES = PKG / "libquartz_b200.resources.txt"


def parse_ptxas(log: str) -> dict[str, dict]:
    """Per kernel: registers, static shared memory bytes, spill bytes (from
    ptxas -v)."""
    out: dict[str, dict] = {}
    cur = None
    for line in log.splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            cur = m.group(1)
            out[cur] = {"registers": 0, "smem": 0, "spill": 0}
            continue
        if cur is None:
            continue
        m = re.search(r"(\d+) bytes spill stores", line)
        if m:
            out[cur]["spill"] = int(m.group(1))
        m = re.search(r"Used (\d+) registers", line)
        if m:
            out[cur]["registers"] = int(m.group(1))
            m2 = re.search(r"(\d+) bytes smem", line)
            out[cur]["smem"] = int(m2.group(1)) if m2 else 0
    return out


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    cmd = [nvcc(), "-Xptxas=-v", *NVCC_FLAGS, f"-I{REPO / 'include'}", f"-I{SRC}",
           "-o", str(OUT), str(SRC / "qz_api.cu")]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise subprocess.CalledProcessError(r.returncode, cmd)
    if verbose:
        sys.stderr.write(r.stderr)
    res = parse_ptxas(r.stderr)
    RESOURCES.write_text("".join(f"{k} registers={v['registers']} smem={v['smem']} "
                                 f"spill={v['spill']}\n" for k, v in sorted(res.items())))
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
