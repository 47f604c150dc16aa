"""Build the reference's own kernels into oracle/_ref/ (checker only): the
ternary torch extension and the legacy ray-sphere tree router library.

Compiles cuda/v5/ternary_torch_ext.cu from the reference tree, where it lies,
with torch.utils.cpp_extension for sm_100a.  The resulting module
(``oracle/_ref/ternary_expert_ext_ref*.so``) is used only by tests as a second
pin for the packing restatement (its ``pack_ternary`` is host code and runs
without a GPU) and, on a GPU box, as the timed reference-GPU kernel.  Nothing
in the product loads it.  Sources are never copied into this repository.

Usage: python oracle/build_ref.py --reference /path/to/reference   (or SB_REFERENCE_ROOT)
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"


def build(reference: Path, verbose: bool = False) -> bool:
    src = reference / "cuda" / "v5" / "ternary_torch_ext.cu"
    if not src.is_file():
        print(f"[oracle/_ref] reference source not found: {src}")
        return False
    OUT.mkdir(exist_ok=True)
    from torch.utils.cpp_extension import load
    load(
        name="ternary_expert_ext_ref",
        sources=[str(src)],
        build_directory=str(OUT),
        extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
        verbose=verbose,
        is_python_module=True,
    )
    return True


def build_tree_kernel(reference: Path, verbose: bool = False) -> bool:
    """cuda/v5/bvh_router_kernel.cu -> oracle/_ref/libbvh_router_ref.so with the
    reference's own compile line (its file header), for sm_100a."""
    import shutil
    import subprocess
    src = reference / "cuda" / "v5" / "bvh_router_kernel.cu"
    if not src.is_file():
        print(f"[oracle/_ref] reference source not found: {src}")
        return False
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    OUT.mkdir(exist_ok=True)
    out = OUT / "libbvh_router_ref.so"
    cmd = [nvcc, "-O3", "--use_fast_math", "-shared", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
           "--maxrregcount=64", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(out), str(src)]
    r = subprocess.run(cmd, capture_output=not verbose, text=True)
    if r.returncode != 0:
        print(f"[oracle/_ref] nvcc failed:\n{r.stderr if not verbose else ''}")
        return False
    return True


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SB_REFERENCE_ROOT"),
                    help="root of the reference checkout (default: $SB_REFERENCE_ROOT)")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    if not a.reference:
        ap.error("pass --reference or set SB_REFERENCE_ROOT")
    ok = build(Path(a.reference), a.v)
    ok = build_tree_kernel(Path(a.reference), a.v) and ok
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
