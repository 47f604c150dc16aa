"""The OptiX router's route / route_topk on the CUDA kernel (needs a B200),
against the CPU restatement (oracle/gas.py): expert ids identical except where
the two closest hits lie within 1e-4 of each other in t; distances within 1e-4
(relative to max(1, t)) on agreeing hits."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gas

pytestmark = pytest.mark.gpu


def scene(n, seed):
    g = np.random.default_rng(seed)
    centers = (g.standard_normal((n, 3)) * 3.0).astype(np.float32)
    radii = (0.4 + 0.6 * g.random(n)).astype(np.float32)
    return centers, radii


def queries(B, seed):
    g = np.random.default_rng(seed)
    p = (g.standard_normal((B, 3)) * 2.0).astype(np.float32)
    d = g.standard_normal((B, 3))
    d = (d / np.linalg.norm(d, axis=1, keepdims=True)).astype(np.float32)
    return p, d


def second_best(o, d, centers, radii, tris, first):
    keep = np.arange(len(centers)) != first
    e, t = gas.trace(o, d, centers[keep], radii[keep], tris)
    return t


@pytest.mark.parametrize("tris", [True, False])
@pytest.mark.parametrize("k", [1, 8])
def test_route_matches_oracle(cuda_device, tris, k):
    import optix_training_ext as ext
    centers, radii = scene(64, 3 + k)
    p, d = queries(200, 7 + k)
    ext.initialize("", "")
    ext.build_gas(torch.from_numpy(centers), torch.from_numpy(radii), use_triangles=tris)
    assert ext.is_ready() and ext.num_experts() == 64
    P, D = torch.from_numpy(p).to(cuda_device), torch.from_numpy(d).to(cuda_device)
    if k == 1:
        ids, ts = ext.route(P, D)
        ids, ts = ids.cpu().numpy()[:, None], ts.cpu().numpy()[:, None]
        rids, rts = gas.route(p, d, centers, radii, tris, 1)
        rids, rts = rids[:, None], rts[:, None]
        dirs = [[di] for di in d]
    else:
        ids, ts = ext.route_topk(P, D, k)
        assert ids.shape == (200, k) and ids.dtype == torch.int32
        ids, ts = ids.cpu().numpy(), ts.cpu().numpy()
        rids, rts = gas.route(p, d, centers, radii, tris, k)
        dirs = [gas.fan(di, k) for di in d]
    assert (rids >= 0).mean() > 0.2   # the scene is hit often enough to mean something
    bad = 0
    for b in range(len(p)):
        for i in range(k):
            if ids[b, i] == rids[b, i]:
                if rids[b, i] >= 0:
                    assert abs(ts[b, i] - rts[b, i]) <= 1e-4 * max(1.0, rts[b, i])
                continue
            # excused: two hits (or a hit and a miss at the range edge) within 1e-4 in t
            alt = second_best(p[b], dirs[b][i], centers, radii, tris, rids[b, i]) if rids[b, i] >= 0 else np.inf
            if not (abs(alt - rts[b, i]) <= 1e-4 * max(1.0, rts[b, i])):
                bad += 1
    assert bad == 0
    ext.shutdown()
