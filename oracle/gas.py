"""CPU restatement of the OptiX router's routing (test infrastructure only).

Only ``tests/`` uses this module; the product path never does.

Follows the reference's device programs and geometry builders, in float64:
  * rays: origin = position, direction as given, t in [0.001, 1000]
    (cuda/optix_router_host.cpp:719-720); closest hit names the expert
    (cuda/optix_router_hitgroup.cu:44-60), a miss gives (-1, 1e30) (:66-71);
  * triangles: per expert the octahedron c +- r e_x, c +- r e_y, c +- r e_z
    with faces {0,2,4},{0,4,3},{0,3,5},{0,5,2},{1,4,2},{1,3,4},{1,5,3},{1,2,5}
    (optix_router_host.cpp:512-560), two-sided;
  * boxes: c +- r, hit at the entry point max(t_entry, tmin) (the reference's
    intersection program reports tmin for every box, leaving the choice to the
    traversal order; the entry point is the semantics its comment describes);
  * top-k: a fan of k rays on a golden-angle spiral in a 0.5-rad cone around
    the direction (cuda/optix_router_raygen.cu:103-170).
Ties between experts go to the lower index.  Parity unpinned by the
reference: its programs need OptiX, which is not part of this build.
"""

from __future__ import annotations

import numpy as np

TMIN, TMAX = 0.001, 1000.0
_FACES = np.array([[0, 2, 4], [0, 4, 3], [0, 3, 5], [0, 5, 2], [1, 4, 2], [1, 3, 4], [1, 5, 3], [1, 2, 5]])
_AXES = np.array([[1, 0, 0], [-1, 0, 0], [0, 1, 0], [0, -1, 0], [0, 0, 1], [0, 0, -1]], np.float64)


def _tri_t(o, d, v0, v1, v2):
    e1, e2 = v1 - v0, v2 - v0
    p = np.cross(d, e2)
    det = e1 @ p
    if abs(det) < 1e-12:
        return np.inf
    inv = 1.0 / det
    s = o - v0
    u = (s @ p) * inv
    if u < 0 or u > 1:
        return np.inf
    q = np.cross(s, e1)
    v = (d @ q) * inv
    if v < 0 or u + v > 1:
        return np.inf
    return (e2 @ q) * inv


def trace(o, d, centers, radii, triangles=True):
    """(expert or -1, t or 1e30) of one ray."""
    o, d = np.asarray(o, np.float64), np.asarray(d, np.float64)
    best, bi = np.inf, -1
    for e, (c, r) in enumerate(zip(np.asarray(centers, np.float64), np.asarray(radii, np.float64))):
        t = np.inf
        if triangles:
            vx = c + r * _AXES
            for f in _FACES:
                tk = _tri_t(o, d, vx[f[0]], vx[f[1]], vx[f[2]])
                if TMIN <= tk <= TMAX and tk < t:
                    t = tk
        else:
            with np.errstate(divide="ignore", invalid="ignore"):
                lo, hi = (c - r - o) / d, (c + r - o) / d
            t0, t1 = -np.inf, np.inf
            for a in range(3):
                if d[a] == 0:
                    if o[a] < c[a] - r or o[a] > c[a] + r:
                        t0 = np.inf
                else:
                    ta, tb = sorted((lo[a], hi[a]))
                    t0, t1 = max(t0, ta), min(t1, tb)
            te = max(t0, TMIN)
            if t0 <= t1 and t1 >= TMIN and te <= TMAX:
                t = te
        if t < best:
            best, bi = t, e
    return bi, (1e30 if bi < 0 else best)


def fan(d, k):
    """The k ray directions of the top-k fan around d."""
    d = np.asarray(d, np.float64)
    tmp = np.array([1.0, 0, 0]) if abs(d[0]) < 0.9 else np.array([0, 1.0, 0])
    u = np.cross(d, tmp)
    n = np.linalg.norm(u)
    if n > 1e-6:
        u = u / n
    v = np.cross(d, u)
    out = []
    for i in range(k):
        t = i / k
        phi = 2.0 * 3.14159265 * t * 1.6180339887
        r = 0.5 * np.sqrt(t)
        di = d + r * (np.cos(phi) * u + np.sin(phi) * v)
        n = np.linalg.norm(di)
        out.append(di / n if n > 1e-6 else di)
    return out


def route(positions, directions, centers, radii, triangles=True, k=1):
    """(ids [B] or [B,k], dists [B] or [B,k])."""
    P, D = np.asarray(positions, np.float64), np.asarray(directions, np.float64)
    if k <= 1:
        res = [trace(o, d, centers, radii, triangles) for o, d in zip(P, D)]
        return np.array([r[0] for r in res], np.int32), np.array([r[1] for r in res])
    ids = np.zeros((len(P), k), np.int32)
    ds = np.zeros((len(P), k))
    for b, (o, d) in enumerate(zip(P, D)):
        for i, di in enumerate(fan(d, k)):
            ids[b, i], ds[b, i] = trace(o, di, centers, radii, triangles)
    return ids, ds
