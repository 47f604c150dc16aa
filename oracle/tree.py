"""CPU restatement of the legacy ray-sphere tree router (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU leg use
this module; the product path never does.

Follows cuda/v5/bvh_router_kernel.cu:244-371 (bvh_router_fused_kernel_v2), the
kernel behind the reference's ctypes library and its torch extension
(cuda/v5/bvh_torch_ext.cu:270-371), in float64:
  * 85 nodes: root 0, children of n are 4n+1 .. 4n+4, leaves 21..84 = experts;
  * per level: d_k = |o + t d - c_k|^2 - r_k^2, t = (c_k - o).d, for the four
    children; the first minimum wins (``<=`` tournament, :108-118);
  * the chosen child's 3x4 portal maps the origin (affine) and the direction
    (linear, renormalised with rsqrt(|d|^2 + 1e-12), :131-178);
  * confidence = prod exp(-d_min); scores[leaf] = exp(-|o + t d - c_leaf|^2)
    with the original ray (:349-370);
  * the Snell dispersion (:180-229) only rewrites the ray's spectral vector,
    which no output reads, so it is not restated.
Pinned against the reference kernel itself, built from its source into
oracle/_ref/ (oracle/build_ref.py) and run on a GPU box, through the fixture
tests/golden/tree_ref.npz (tests/golden/make_tree_golden.py).
"""

from __future__ import annotations

import numpy as np

NODES, LEAVES, LEAF0, LEVELS = 85, 64, 21, 3


def ray_dist2(o, d, c):
    """|o + t d - c|^2 with t = (c - o).d; o, d [B,3], c [...,3] broadcast."""
    t = ((c - o) * d).sum(axis=-1, keepdims=True)
    p = o + t * d - c
    return (p * p).sum(axis=-1)


def route(centers, radii, portals, origins, directions):
    """(expert [B] int32, scores [B,64] f32, path [B,3] int32, confidence [B] f32,
    margins [B,3] gap between the best and second-best child per level)."""
    C = np.asarray(centers, np.float64).reshape(NODES, 3)
    R = np.asarray(radii, np.float64).reshape(NODES)
    P = np.asarray(portals, np.float64).reshape(NODES, 3, 4)
    o = np.asarray(origins, np.float64).reshape(-1, 3).copy()
    d = np.asarray(directions, np.float64).reshape(-1, 3).copy()
    B = o.shape[0]
    o0, d0 = o.copy(), d.copy()
    node = np.zeros(B, np.int64)
    conf = np.ones(B)
    path = np.zeros((B, LEVELS), np.int32)
    margins = np.zeros((B, LEVELS))
    rows = np.arange(B)
    for lvl in range(LEVELS):
        kids = node[:, None] * 4 + 1 + np.arange(4)[None, :]          # [B,4]
        dist = ray_dist2(o[:, None, :], d[:, None, :], C[kids]) - R[kids] ** 2
        k = np.argmin(dist, axis=1)                                     # first minimum
        srt = np.sort(dist, axis=1)
        margins[:, lvl] = srt[:, 1] - srt[:, 0]
        best = dist[rows, k]
        child = kids[rows, k]
        path[:, lvl] = child
        A = P[child]                                                    # [B,3,4]
        o = np.einsum("bij,bj->bi", A[:, :, :3], o) + A[:, :, 3]
        d = np.einsum("bij,bj->bi", A[:, :, :3], d)
        d = d / np.sqrt((d * d).sum(axis=1, keepdims=True) + 1e-12)
        conf *= np.exp(-best)
        node = child
    scores = np.exp(-ray_dist2(o0[:, None, :], d0[:, None, :], C[LEAF0:][None, :, :]))
    return ((node - LEAF0).astype(np.int32), scores.astype(np.float32), path, conf.astype(np.float32), margins)
