"""CPU restatement of the MoE pipeline stage kernels and of the reference
pipeline simulator's stages (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU leg import
this module; the product path never does.

  * ``apply_calibration``   cuda/async_pipeline.cu:150-170
        c[t,i] = b[i] + sum_j W[i,j] raw[t,j]
  * ``softmax_topk``        cuda/async_pipeline.cu:177-230
        p = softmax(c) over the experts (max-subtracted exp, sum, divide);
        k passes of a first-maximum scan: largest first, lower index first
        among equal values; the weights are the chosen probabilities.
  * ``scatter_by_expert``   cuda/async_pipeline.cu:79-101
        counts[e] = entries with id e (ids >= E skipped); dispatch lists in
        ascending entry order t*k + j (the stable order the reference's
        Python stage builds, python/async_pipeline_bridge.py:113-126; the
        reference kernel's atomic slots give some order of the same set);
        only slots below the limit are stored.
  * ``weighted_combine``    cuda/async_pipeline.cu:112-132
        out[t,d] = sum_j w[t,j] eo[t,j,d], j ascending.

Sums run in float64 here and are compared with tolerances; the scatter is
integer work and compared exactly.  Pinned against the reference simulator's
own outputs through tests/golden/pipeline_*.npz (tests/golden/make_golden.py).
"""

from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

F32 = np.float32


def apply_calibration(raw: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    return (np.asarray(raw, np.float64) @ np.asarray(w, np.float64).T + np.asarray(b, np.float64)).astype(F32)


def topk_first_max(v: np.ndarray, k: int) -> Tuple[np.ndarray, np.ndarray]:
    """k largest per row, descending; equal values toward the lower index."""
    idx = np.argsort(-np.asarray(v), axis=1, kind="stable")[:, :k]
    return np.take_along_axis(v, idx, axis=1), idx


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float64)
    e = np.exp(x - x.max(axis=1, keepdims=True))
    return (e / e.sum(axis=1, keepdims=True)).astype(F32)


def softmax_topk(logits: np.ndarray, k: int, cal_w: Optional[np.ndarray] = None,
                 cal_b: Optional[np.ndarray] = None, apply_softmax: bool = True):
    """(probs [B,E], ids [B,k], weights [B,k])."""
    v = np.asarray(logits, F32)
    if cal_w is not None:
        v = apply_calibration(v, cal_w, cal_b if cal_b is not None else np.zeros(v.shape[1], F32))
    p = softmax(v) if apply_softmax else v
    w, ids = topk_first_max(p, k)
    return p, ids, w


def scatter_by_expert(ids: np.ndarray, n_experts: int, max_per: int, store_entry: bool = False):
    """(dispatch [E, max] int32 with -1 in unused slots, counts [E] int32)."""
    ids = np.asarray(ids)
    B, k = ids.shape
    flat = ids.reshape(-1)
    disp = np.full((n_experts, max_per), -1, np.int32)
    counts = np.zeros(n_experts, np.int32)
    for e in range(n_experts):
        r = np.nonzero(flat == e)[0]
        counts[e] = len(r)
        vals = r if store_entry else r // k
        disp[e, :min(len(r), max_per)] = vals[:max_per]
    return disp, counts


def weighted_combine(eo: np.ndarray, w: np.ndarray) -> np.ndarray:
    return np.einsum("tjd,tj->td", np.asarray(eo, np.float64), np.asarray(w, np.float64)).astype(F32)
