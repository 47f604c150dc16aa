"""The OptiX router's routing restated on the CPU (oracle/gas.py): cases with
known answers, and the drop-in extension's host-side checks (no GPU).

Parity is unpinned by the reference (its programs need OptiX); these cases fix
the geometry the restatement follows."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gas


def test_octahedron_and_box_hits():
    centers = np.array([[0.0, 0.0, 5.0], [0.0, 0.0, 10.0], [3.0, 0.0, 5.0]])
    radii = np.array([1.0, 1.0, 0.5])
    o, d = np.zeros(3), np.array([0.0, 0.0, 1.0])
    # the octahedron's near vertex is at z = 4; the box's near face too
    assert gas.trace(o, d, centers, radii, True) == (0, pytest.approx(4.0))
    assert gas.trace(o, d, centers, radii, False) == (0, pytest.approx(4.0))
    # a ray between the spheres misses
    assert gas.trace(o, np.array([0.0, 1.0, 0.0]), centers, radii, True) == (-1, 1e30)
    # off-axis: the octahedron's face is farther than the box's corner region
    o2 = np.array([0.6, 0.6, 0.0])
    e_t, t_t = gas.trace(o2, d, centers, radii, True)
    e_b, t_b = gas.trace(o2, d, centers, radii, False)
    assert e_t == -1 or t_t > 4.0          # |x|+|y|+|z-5| <= 1 is not met at x=y=0.6 for z near 5
    assert (e_b, t_b) == (0, pytest.approx(4.0))
    # a ray starting inside a box hits it at tmin
    assert gas.trace(np.array([0.0, 0.0, 5.0]), d, centers, radii, False) == (0, pytest.approx(gas.TMIN))


def test_fan_directions():
    d = np.array([0.0, 0.0, 1.0])
    dirs = gas.fan(d, 8)
    assert len(dirs) == 8
    np.testing.assert_allclose(dirs[0], d)
    for di in dirs:
        assert abs(np.linalg.norm(di) - 1.0) < 1e-12
        assert np.arccos(np.clip(di @ d, -1, 1)) <= 0.5 + 1e-9   # inside the 0.5-rad cone


def test_dropin_checks():
    import optix_training_ext as ext
    ext.shutdown()
    with pytest.raises(RuntimeError):
        ext.build_gas(torch.zeros(4, 3), torch.ones(4))        # not initialised
    ext.initialize("raygen.ptx", "hitgroup.ptx")
    with pytest.raises(RuntimeError):
        ext.build_gas(torch.zeros(4, 2), torch.ones(4))        # wrong shape
    with pytest.raises(RuntimeError):
        ext.route(torch.zeros(2, 3), torch.zeros(2, 3))        # no geometry yet
    assert not ext.is_ready() and not ext.is_coopvec_supported()
    assert ext.upload_calibration_affine(torch.ones(4), torch.zeros(4)) and ext.has_calibration()
    assert ext.disable_calibration() and not ext.has_calibration()
    ext.shutdown()
