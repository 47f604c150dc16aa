"""Build libspectral_b200.so (sm_100a) in-tree.

    python spectral-ai_b200/build.py [--force] [-v]

Compiles csrc/lib.cu (one translation unit: kernels + C ABI) with nvcc for
``arch=compute_100a,code=sm_100a`` into sb200/libspectral_b200.so.  The build
is skipped when the library is newer than every source file.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT = PKG / "sb200" / "libspectral_b200.so"

NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(s.stat().st_mtime <= t for s in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-o", str(tmp), str(CSRC / "lib.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=not verbose, text=True)
    if r.returncode != 0:
        msg = (r.stderr or "") + (r.stdout or "")
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{msg}")
    os.replace(tmp, OUT)
    return OUT


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    p = build(a.force, a.v)
    print(p)
    return 0


if __name__ == "__main__":
    sys.exit(main())
