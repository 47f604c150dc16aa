"""Legacy ray-sphere tree router on the GPU (needs a B200).

The B200 kernel (sb_tree_route, the bvh_router_ext drop-in and the reference
ctypes ABI exported by libspectral_b200.so) against the oracle
(oracle/tree.py) and, when oracle/_ref/libbvh_router_ref.so was built from the
reference source, against the reference kernel itself on the same inputs:
paths and experts identical except where two children's distances lie within
1e-5 (relative) of each other; scores and confidence within 1e-5 relative
(both kernels use the fast exp; the oracle is float64).
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import tree as otree

pytestmark = pytest.mark.gpu
REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libbvh_router_ref.so"


def _P(a):
    return a.ctypes.data_as(C.c_void_p)


def tie_rows(margins, path_ref, path_got, scale=1.0):
    """Rows whose paths differ only after a level whose best two children tie."""
    bad = np.zeros(len(path_ref), bool)
    excused = np.zeros(len(path_ref), bool)
    for l in range(3):
        diff = (path_ref[:, l] != path_got[:, l]) & ~excused & ~bad
        tie = margins[:, l] <= 1e-5 * scale
        excused |= diff & tie
        bad |= diff & ~tie
    return bad, excused


def upload(tree):
    import bvh_router_ext as ext
    ext.upload_tree(*[torch.from_numpy(np.ascontiguousarray(tree[k], np.float32))
                      for k in ("centers", "radii", "portals", "snell_w", "snell_b")])
    return ext


@pytest.mark.parametrize("seed,B", [(0, 1), (0, 1000), (1, 129), (2, 70000)])
def test_tree_route_against_oracle(cuda_device, seed, B):
    from sb200 import synth
    tree = synth.legacy_tree(seed)
    o, d = synth.rays(B, 100 + seed)
    ext = upload(tree)
    s = torch.zeros(B, 64, device=cuda_device)
    ex, sc, cf, pa = ext.route(torch.from_numpy(o).to(cuda_device), torch.from_numpy(d).to(cuda_device), s)
    rex, rsc, rpa, rcf, margins = otree.route(tree["centers"], tree["radii"], tree["portals"], o, d)
    bad, excused = tie_rows(margins, rpa, pa.cpu().numpy())
    assert bad.sum() == 0
    ok = ~excused
    assert np.array_equal(ex.cpu().numpy()[ok], rex[ok])
    np.testing.assert_allclose(sc.cpu().numpy(), rsc, rtol=1e-5, atol=1e-30)
    np.testing.assert_allclose(cf.cpu().numpy()[ok], rcf[ok], rtol=1e-5, atol=1e-30)
    assert ex.dtype == torch.int32 and pa.dtype == torch.int32 and sc.shape == (B, 64)


def test_ctypes_abi_graph_replay(cuda_device):
    """The reference's ctypes entry points exported by libspectral_b200.so:
    graph capture on first use, replay with other host buffers, errors as -1."""
    from sb200 import _lib, synth
    lib = _lib.load()
    tree = synth.legacy_tree(3)
    arrs = [np.ascontiguousarray(tree[k], np.float32) for k in ("centers", "radii", "portals", "snell_w", "snell_b")]
    assert lib.bvh_upload_tree(*[_P(a) for a in arrs]) == 0
    assert lib.bvh_alloc_buffers(512) == 0 and lib.bvh_get_batch_capacity() == 512
    assert (lib.bvh_get_num_nodes(), lib.bvh_get_num_experts(), lib.bvh_get_spec_dim()) == (85, 64, 64)
    for it, (B, g) in enumerate([(300, 1), (300, 1), (300, 0), (200, 1), (300, 1)]):
        o, d = synth.rays(B, 300 + it)
        spec = np.zeros((B, 64), np.float32)
        ex, sc = np.zeros(B, np.int32), np.zeros((B, 64), np.float32)
        pa, cf = np.zeros((B, 3), np.int32), np.zeros(B, np.float32)
        assert lib.bvh_route_batch(_P(o), _P(d), _P(spec), _P(ex), _P(sc), _P(pa), _P(cf), B, g) == 0
        rex, rsc, rpa, rcf, margins = otree.route(tree["centers"], tree["radii"], tree["portals"], o, d)
        bad, excused = tie_rows(margins, rpa, pa)
        assert bad.sum() == 0, it
        np.testing.assert_allclose(sc, rsc, rtol=1e-5, atol=1e-30)
    o, d = synth.rays(600, 9)
    z = np.zeros((600, 64), np.float32)
    assert lib.bvh_route_batch(_P(o), _P(d), _P(z), None, None, None, None, 600, 1) == -1  # over capacity
    lib.bvh_free_buffers()
    assert lib.bvh_get_batch_capacity() == 0


@pytest.mark.skipif(not REF.is_file(), reason="reference tree library not built (oracle/build_ref.py)")
@pytest.mark.parametrize("seed,B", [(0, 1000), (4, 1024), (5, 7)])
def test_tree_route_against_reference_kernel(cuda_device, seed, B):
    """Same inputs through the reference's own kernel: identical decisions."""
    from sb200 import synth
    tree = synth.legacy_tree(seed)
    o, d = synth.rays(B, 200 + seed)
    ref = C.CDLL(str(REF))
    for fn in ("bvh_upload_tree", "bvh_alloc_buffers", "bvh_route_batch"):
        getattr(ref, fn).restype = C.c_int
    arrs = [np.ascontiguousarray(tree[k], np.float32) for k in ("centers", "radii", "portals", "snell_w", "snell_b")]
    assert ref.bvh_upload_tree(*[_P(a) for a in arrs]) == 0
    assert ref.bvh_alloc_buffers(B) == 0
    spec = np.ascontiguousarray(np.random.default_rng(seed).standard_normal((B, 64)), np.float32)
    rex, rsc = np.zeros(B, np.int32), np.zeros((B, 64), np.float32)
    rpa, rcf = np.zeros((B, 3), np.int32), np.zeros(B, np.float32)
    assert ref.bvh_route_batch(_P(o), _P(d), _P(spec), _P(rex), _P(rsc), _P(rpa), _P(rcf), B, 0) == 0
    ext = upload(tree)
    ex, sc, cf, pa = ext.route(torch.from_numpy(o).to(cuda_device), torch.from_numpy(d).to(cuda_device),
                               torch.from_numpy(spec).to(cuda_device))
    _, _, _, _, margins = otree.route(tree["centers"], tree["radii"], tree["portals"], o, d)
    bad, excused = tie_rows(margins, rpa, pa.cpu().numpy())
    assert bad.sum() == 0
    ok = ~excused
    assert np.array_equal(ex.cpu().numpy()[ok], rex[ok])
    np.testing.assert_allclose(sc.cpu().numpy(), rsc, rtol=1e-6, atol=1e-30)
    np.testing.assert_allclose(cf.cpu().numpy()[ok], rcf[ok], rtol=1e-6, atol=1e-30)
