"""Legacy ray-sphere tree router: the oracle against the reference kernel's
own outputs (no GPU).

tests/golden/tree_ref.npz holds outputs of the reference's
cuda/v5/bvh_router_kernel.cu, built from its source into oracle/_ref/ and run
through its ctypes API on a GPU by tests/golden/make_tree_golden.py; inputs
regenerate from sb200.synth.legacy_tree / rays and are checked by checksum.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import tree as otree

GOLD = Path(__file__).resolve().parent / "golden" / "tree_ref.npz"


def _cs(a):
    a = np.asarray(a, np.float64)
    return np.array([a.sum(), (a * a).sum(), a.ravel()[:: max(1, a.size // 4099)].sum()])


@pytest.mark.skipif(not GOLD.is_file(), reason="tree_ref.npz not generated")
@pytest.mark.parametrize("name", ["t0", "t1", "t2"])
def test_oracle_matches_reference_kernel(name):
    from sb200 import synth
    g = dict(np.load(GOLD))
    seed, B, rseed = (int(v) for v in g[f"{name}/meta"])
    tree = synth.legacy_tree(seed)
    o, d = synth.rays(B, rseed)
    np.testing.assert_allclose(np.concatenate([_cs(tree["centers"]), _cs(o), _cs(d)]), g[f"{name}/in_checksum"],
                               rtol=1e-9)
    ex, sc, pa, cf, margins = otree.route(tree["centers"], tree["radii"], tree["portals"], o, d)
    rpa = g[f"{name}/path"]
    diff = (pa != rpa).any(axis=1)
    # a differing path must start at a level whose best two children tie
    for b in np.nonzero(diff)[0]:
        l = int(np.argmax(pa[b] != rpa[b]))
        assert margins[b, l] <= 1e-5, (b, l, margins[b, l])
    ok = ~diff
    assert np.array_equal(ex[ok], g[f"{name}/expert"][ok])
    # the reference kernel's fast exp: its error grows with the argument
    # (|d|^2 up to ~10 here), 6.4e-6 relative at most on these cases
    np.testing.assert_allclose(sc, g[f"{name}/scores"], rtol=1e-5, atol=1e-30)
    np.testing.assert_allclose(cf[ok], g[f"{name}/confidence"][ok], rtol=1e-5, atol=1e-30)


def test_oracle_tree_structure():
    from sb200 import synth
    tree = synth.legacy_tree(7)
    o, d = synth.rays(500, 7)
    ex, sc, pa, cf, _ = otree.route(tree["centers"], tree["radii"], tree["portals"], o, d)
    assert ((pa[:, 0] >= 1) & (pa[:, 0] <= 4)).all()
    assert ((pa[:, 1] - 1) // 4 == pa[:, 0]).all() and ((pa[:, 2] - 1) // 4 == pa[:, 1]).all()
    assert np.array_equal(ex, pa[:, 2] - 21)
    assert ((cf > 0) & np.isfinite(cf)).all() and ((sc > 0) & (sc <= 1)).all()


def test_dropin_argument_checks():
    import bvh_router_ext as ext
    with pytest.raises(RuntimeError):
        ext.upload_tree(torch.zeros(84, 3), torch.zeros(85), torch.zeros(85, 12), torch.zeros(85, 64),
                        torch.zeros(85))
    with pytest.raises(RuntimeError):
        ext.route(torch.zeros(4, 3), torch.zeros(4, 3), torch.zeros(4, 64))   # CPU tensors
