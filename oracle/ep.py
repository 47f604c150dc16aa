"""CPU statement of the expert-parallel exchange (test infrastructure only).

Only ``tests/`` use this module; the product path (csrc/ep.cu behind
sb200.ep.ExpertParallelMoE) never does.

It states, in numpy fp32, the two things the device layer relies on:

* the summation tree of a token's expert outputs (csrc/tree_sum.cuh), here in
  its recursive form — split the positions (expert ids, ascending) at the
  first boundary whose highest differing bit is the largest, sum both halves,
  add — and, beside it, a line-by-line port of the device's stack schedule, so
  that tests can check the two agree bit for bit;
* the exchange protocol of csrc/ep.cu with W ranks: a token goes once to each
  rank holding one of its experts, that rank returns the tree sum of the
  token's entries among its experts (its aligned block of E/W ids), and the
  token's rank sums the partials along the tree over the rank index.  With
  E/W a power of two this equals the tree over all k entries bit for bit,
  which is what makes the sharded layer equal the single-GPU layer.

The reference sums a token's slots in slot order (python/olmoe_extract.py:
146-155); any order is the same sum up to fp32 rounding, which the layer
tests bound against the float64 oracle.
"""

from __future__ import annotations

from typing import Callable, List, Sequence

import numpy as np

F32 = np.float32


def level(p: int, q: int) -> int:
    """Tree level of the boundary between positions p and q (-1 when equal)."""
    return -1 if p == q else int(p ^ q).bit_length() - 1


def tree_sum(values: Sequence[np.ndarray], positions: Sequence[int]) -> np.ndarray:
    """Recursive tree sum; values ordered by ascending position."""
    n = len(values)
    if n == 0:
        raise ValueError("empty tree")
    if n == 1:
        return np.asarray(values[0], F32)
    lv = [level(positions[i], positions[i + 1]) for i in range(n - 1)]
    m = lv.index(max(lv)) + 1          # first boundary at the top level
    left = tree_sum(values[:m], positions[:m])
    right = tree_sum(values[m:], positions[m:])
    return (left + right).astype(F32)


def tree_schedule(positions: Sequence[int]):
    """Port of tree_schedule (csrc/tree_sum.cuh): merges (dst, src) in order."""
    st, sd, merges = [], [], []
    prev = 0
    for i, p in enumerate(positions):
        d = 0x7fffffff if i == 0 else level(prev, p)
        while len(st) >= 2 and sd[-1] < d:
            merges.append((st[-2], st[-1]))
            st.pop(); sd.pop()
        st.append(i); sd.append(d)
        prev = p
    while len(st) >= 2:
        merges.append((st[-2], st[-1]))
        st.pop(); sd.pop()
    return merges


def tree_apply(values: Sequence[np.ndarray], merges) -> np.ndarray:
    v = [np.array(x, F32, copy=True) for x in values]
    for dst, src in merges:
        v[dst] = (v[dst] + v[src]).astype(F32)
    return v[0]


def token_entries(ids_row, vals_row):
    """(position, value) of a token's in-range entries, ascending by (id, slot)."""
    order = sorted(range(len(ids_row)), key=lambda j: (int(ids_row[j]), j))
    return [int(ids_row[j]) for j in order], [vals_row[j] for j in order]


def combine_single(ids: np.ndarray, y_slots: np.ndarray) -> np.ndarray:
    """Single-GPU combine: per token, the tree over its k slot outputs.
    y_slots [B, k, H] fp32 (already weighted)."""
    B, k, H = y_slots.shape
    out = np.zeros((B, H), F32)
    for t in range(B):
        pos, vals = token_entries(ids[t], list(y_slots[t]))
        out[t] = tree_sum(vals, pos)
    return out


def plan_destinations(ids: np.ndarray, n_experts: int, world: int):
    """ep_route: per destination rank, the tokens that go there (ascending) and
    each token's row there (-1 if none)."""
    el = n_experts // world
    B = ids.shape[0]
    send_pos = np.full((B, world), -1, np.int64)
    lists: List[List[int]] = [[] for _ in range(world)]
    for t in range(B):
        for g in sorted({int(e) // el for e in ids[t]}):
            send_pos[t, g] = len(lists[g])
            lists[g].append(t)
    return send_pos, lists


def destination_partials(ids_rows: np.ndarray, y_rows: np.ndarray, rank: int, n_experts: int,
                         world: int) -> np.ndarray:
    """ep_return on rank `rank`: for each received row (its k ids and its k
    slot outputs), the tree sum over the entries whose experts live here,
    positions = local expert ids."""
    el = n_experts // world
    out = np.zeros((len(ids_rows), y_rows.shape[-1]), F32)
    for i in range(len(ids_rows)):
        sel = [j for j in range(ids_rows.shape[1]) if int(ids_rows[i, j]) // el == rank]
        pos, vals = token_entries([int(ids_rows[i, j]) - rank * el for j in sel], [y_rows[i, j] for j in sel])
        out[i] = tree_sum(vals, pos)
    return out


def source_combine(send_pos: np.ndarray, partials: Sequence[np.ndarray]) -> np.ndarray:
    """ep_combine: per token, the tree over its destinations' partials, positions = rank."""
    B, W = send_pos.shape
    H = max((p.shape[1] for p in partials if p.ndim == 2), default=0)
    out = np.zeros((B, H), F32)
    for t in range(B):
        gs = [g for g in range(W) if send_pos[t, g] >= 0]
        if gs:
            out[t] = tree_sum([partials[g][send_pos[t, g]] for g in gs], gs)
    return out


def expert_parallel(ids: np.ndarray, y_slots: np.ndarray, n_experts: int, world: int,
                    exchange: Callable = None) -> np.ndarray:
    """The whole protocol in one process (every rank's part in turn); equals
    combine_single bit for bit when n_experts / world is a power of two."""
    send_pos, lists = plan_destinations(ids, n_experts, world)
    partials = []
    for g in range(world):
        rows = lists[g]
        partials.append(destination_partials(ids[rows], y_slots[rows], g, n_experts, world)
                        if rows else np.zeros((0, y_slots.shape[-1]), F32))
    return source_combine(send_pos, partials)
