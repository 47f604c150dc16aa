"""Golden outputs of the reference's legacy tree router kernel, run on a GPU.

Loads oracle/_ref/libbvh_router_ref.so (built from the reference's
cuda/v5/bvh_router_kernel.cu by oracle/build_ref.py) through its own ctypes
API (bvh_upload_tree, bvh_alloc_buffers, bvh_route_batch; :378-717) and stores
its outputs for seeded trees and rays (sb200.synth.legacy_tree / rays; only
checksums of the inputs are kept).  Needs a CUDA device:

    python tests/golden/make_tree_golden.py --out tests/golden/tree_ref.npz
"""

from __future__ import annotations

import argparse
import ctypes as C
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO / "spectral-ai_b200"))
from sb200 import synth  # noqa: E402

CASES = [("t0", 0, 1000, 11), ("t1", 1, 256, 12), ("t2", 2, 1024, 13)]


def checksum(a):
    a = np.asarray(a, np.float64)
    return np.array([a.sum(), (a * a).sum(), a.ravel()[:: max(1, a.size // 4099)].sum()])


def run_reference(lib, tree, o, d):
    f = lambda a: np.ascontiguousarray(a, np.float32)
    P = lambda a: a.ctypes.data_as(C.c_void_p)
    arrs = [f(tree[k]) for k in ("centers", "radii", "portals", "snell_w", "snell_b")]
    assert lib.bvh_upload_tree(*[P(a) for a in arrs]) == 0
    B = o.shape[0]
    assert lib.bvh_alloc_buffers(B) == 0
    spec = np.zeros((B, 64), np.float32)
    ex = np.zeros(B, np.int32)
    sc = np.zeros((B, 64), np.float32)
    pa = np.zeros((B, 3), np.int32)
    cf = np.zeros(B, np.float32)
    o, d = f(o), f(d)
    assert lib.bvh_route_batch(P(o), P(d), P(spec), P(ex), P(sc), P(pa), P(cf), B, 0) == 0
    return ex, sc, pa, cf


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--lib", default=str(REPO / "oracle" / "_ref" / "libbvh_router_ref.so"))
    ap.add_argument("--out", default=str(REPO / "tests" / "golden" / "tree_ref.npz"))
    a = ap.parse_args()
    lib = C.CDLL(a.lib)
    for fn in ("bvh_upload_tree", "bvh_alloc_buffers", "bvh_route_batch"):
        getattr(lib, fn).restype = C.c_int
    out = {}
    for name, seed, B, rseed in CASES:
        tree = synth.legacy_tree(seed)
        o, d = synth.rays(B, rseed)
        ex, sc, pa, cf = run_reference(lib, tree, o, d)
        out[f"{name}/meta"] = np.array([seed, B, rseed])
        out[f"{name}/in_checksum"] = np.concatenate([checksum(tree["centers"]), checksum(o), checksum(d)])
        out[f"{name}/expert"], out[f"{name}/scores"] = ex, sc
        out[f"{name}/path"], out[f"{name}/confidence"] = pa, cf
    np.savez_compressed(a.out, **out)
    print(f"wrote {a.out}")


if __name__ == "__main__":
    main()
