"""Parity rules shared by the oracle and CUDA tests.

Router:
  * expert ids / route paths identical, except where the deciding scores lie
    within ``TIE`` (1e-6, relative to max(1, |score|)) of each other;
  * routing weights within 1e-5 relative (fp32 engines) or 2e-2 (bf16 engine).
A token whose path legitimately diverges at some level (a tie) is excused for
everything downstream of that level, since its later levels see a different
parent.
"""

from __future__ import annotations

import numpy as np

TIE = 1e-6


def tie_excused(margins: np.ndarray, level: int, scale: np.ndarray | None = None) -> np.ndarray:
    """Tokens whose top-2 logits at ``level`` are within TIE (relative)."""
    m = margins[:, level]
    s = np.ones_like(m) if scale is None else np.maximum(1.0, np.abs(scale))
    return m <= TIE * s


def compare_paths(ref_path: np.ndarray, got_path: np.ndarray, margins: np.ndarray):
    """Returns (n_mismatch_unexcused, excused_mask[B]) for route paths [B, L]."""
    B, L = ref_path.shape
    excused = np.zeros(B, bool)
    bad = np.zeros(B, bool)
    for l in range(L):
        diff = (ref_path[:, l] != got_path[:, l]) & ~excused & ~bad
        tie = tie_excused(margins, l)
        excused |= diff & tie
        bad |= diff & ~tie
    return int(bad.sum()), excused


def rel_err(got, ref, floor=1e-12):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.abs(got - ref) / np.maximum(np.abs(ref), floor)


def topk_ids_match(ref_probs: np.ndarray, ref_ids: np.ndarray, got_ids: np.ndarray, tol: float):
    """Top-k id rows agree position by position, except where the oracle's
    probabilities of the two experts involved are within ``tol`` (relative to
    the larger one), i.e. where their order is a tie.  Returns the number of
    unexcused mismatching positions."""
    B, k = ref_ids.shape
    rows = np.arange(B)[:, None]
    pr = ref_probs[rows, ref_ids].astype(np.float64)
    pg = ref_probs[rows, np.clip(got_ids, 0, ref_probs.shape[1] - 1)].astype(np.float64)
    valid = (got_ids >= 0) & (got_ids < ref_probs.shape[1])
    same = ref_ids == got_ids
    close = np.abs(pr - pg) <= tol * np.maximum(np.abs(pr), np.abs(pg))
    return int((~same & ~(close & valid)).sum())


def ternary_errors(got, ref):
    """(row-normwise relative error max, elementwise error relative to |ref| + row rms max)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    diff = got - ref
    rn = np.sqrt((ref * ref).sum(axis=1)) + 1e-30
    norm = np.sqrt((diff * diff).sum(axis=1)) / rn
    rms = rn / np.sqrt(ref.shape[1])
    elem = np.abs(diff) / (np.abs(ref) + rms[:, None])
    return float(norm.max()), float(elem.max())


def hybrid_ids_mismatch(bvh_probs: np.ndarray, full_probs: np.ndarray, n_cand: int, ref_ids: np.ndarray,
                        got_ids: np.ndarray, tie_bvh: float, tie_full: float) -> int:
    """Hybrid pre-filter ids: rows whose n-th and (n+1)-th BVH probabilities lie
    within ``tie_bvh`` (relative) have an ambiguous candidate set and are
    excused; elsewhere the top-k ids agree position by position up to ties of
    the dense probabilities within ``tie_full``.  Returns unexcused mismatches."""
    s = -np.sort(-np.asarray(bvh_probs, np.float64), axis=1)
    if n_cand < s.shape[1]:
        amb = (s[:, n_cand - 1] - s[:, n_cand]) <= tie_bvh * np.abs(s[:, n_cand - 1])
    else:
        amb = np.zeros(s.shape[0], bool)
    keep = ~amb
    return topk_ids_match(full_probs[keep], ref_ids[keep], got_ids[keep], tie_full)
