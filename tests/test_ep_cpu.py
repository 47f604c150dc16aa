"""The summation tree and the exchange protocol of the expert-parallel layer,
on the CPU (oracle/ep.py; no GPU, one process).

The device layer (csrc/ep.cu, csrc/tree_sum.cuh) relies on one property: the
tree sum of a token's expert outputs splits over aligned blocks of experts, so
per-GPU partial sums combined along the tree over the ranks give the single-GPU
sum bit for bit.  These tests check that property in fp32 and that the
device's stack schedule (ported line by line) builds the same tree.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import ep as oep


def _case(seed, B, E, k, H, spread=3.0):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(B)]).astype(np.int32)
    # magnitudes spread over decades so that the grouping changes the rounding
    y = (rng.standard_normal((B, k, H)) * 10 ** rng.uniform(-spread, spread, (B, k, 1))).astype(np.float32)
    return ids, y


def test_grouping_matters_in_fp32():
    """Sanity: slot order and tree order do differ in fp32 on these inputs, so
    the bitwise checks below are not vacuous."""
    ids, y = _case(0, 64, 64, 8, 16)
    tree = oep.combine_single(ids, y)
    slot = np.zeros_like(tree)
    for j in range(8):
        slot = (slot + y[:, j]).astype(np.float32)
    assert not np.array_equal(tree, slot)
    np.testing.assert_allclose(tree, slot, rtol=1e-5, atol=1e-5 * np.abs(y).max())


@pytest.mark.parametrize("seed", range(5))
def test_device_schedule_builds_the_recursive_tree(seed):
    ids, y = _case(seed, 40, 64, 8, 8)
    for t in range(len(ids)):
        pos, vals = oep.token_entries(ids[t], list(y[t]))
        merges = oep.tree_schedule(pos)
        assert len(merges) == len(pos) - 1
        assert np.array_equal(oep.tree_apply(vals, merges), oep.tree_sum(vals, pos))


def test_schedule_with_repeated_positions():
    """Equal ids (not produced by top-k, allowed by the API) merge deepest, right to left."""
    vals = [np.float32(v) for v in (1e8, 1.0, -1e8, 3.0)]
    pos = [5, 5, 5, 9]
    assert oep.tree_apply(vals, oep.tree_schedule(pos)) == oep.tree_sum(vals, pos)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("E,k", [(64, 8), (16, 4), (32, 16)])
def test_sharded_sum_equals_single_gpu_bitwise(world, E, k):
    if E % world:
        pytest.skip("experts do not divide")
    ids, y = _case(10 + world, 200, E, k, 12)
    assert np.array_equal(oep.expert_parallel(ids, y, E, world), oep.combine_single(ids, y))


def test_token_goes_once_per_destination():
    """Dispatch is deduplicated per destination rank: a token is sent once to
    each rank holding any of its experts (at most min(k, W) copies)."""
    ids, _ = _case(3, 500, 64, 8, 1)
    send_pos, lists = oep.plan_destinations(ids, 64, 8)
    for t in range(len(ids)):
        dests = {int(e) // 8 for e in ids[t]}
        assert {g for g in range(8) if send_pos[t, g] >= 0} == dests
    assert sum(len(l) for l in lists) == sum(len({int(e) // 8 for e in r}) for r in ids)
    # rows of each destination are the tokens in ascending order, numbered 0..n-1
    for g in range(8):
        assert lists[g] == sorted(lists[g])
        assert [send_pos[t, g] for t in lists[g]] == list(range(len(lists[g])))
    # about 5.4 distinct ranks per token for 8 distinct experts over 8 blocks of 8
    assert 5.0 < sum(len(l) for l in lists) / len(ids) < 5.8


@pytest.mark.parametrize("group", [1, 4])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_balanced_placement_is_a_permutation_that_evens_the_ranks(world, group):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "spectral-ai_b200"))
    from sb200.ep import balanced_placement, experts_at
    rng = np.random.default_rng(world)
    # skewed loads like the router's (max/mean about 2.6), hot experts clustered
    loads = np.sort(rng.gamma(1.2, 100.0, 64))[::-1].copy()
    perm = balanced_placement(loads, world, group=group)
    assert sorted(perm) == list(range(64))
    for u in range(64 // group):   # a unit of `group` consecutive experts stays together, in order
        ps = [perm[u * group + i] for i in range(group)]
        assert ps == list(range(ps[0], ps[0] + group)) and ps[0] // (64 // world) == ps[-1] // (64 // world)
    el = 64 // world
    held = [experts_at(perm, r, world) for r in range(world)]
    assert sorted(e for h in held for e in h) == list(range(64))
    for r, h in enumerate(held):
        assert len(h) == el and h == sorted(h)                 # position order = ascending id
        assert all(perm[e] // el == r for e in h)
    per = np.array([loads[h].sum() for h in held])
    contiguous = np.array([loads[r * el:(r + 1) * el].sum() for r in range(world)])
    assert per.max() <= contiguous.max() + 1e-9
    if world > 1:
        # LPT bound: the busiest rank exceeds the mean by at most one unit's load
        unit = loads.reshape(-1, group).sum(axis=1)
        assert per.max() <= per.mean() + unit.max() + 1e-9


def test_placement_keeps_the_sharded_sum_bitwise():
    """Relabelling experts by a placement and sharding by position gives the
    single-process tree sum over the relabelled ids (what csrc/ep.cu computes)."""
    ids, y = _case(5, 40, 16, 4, 8)
    perm = np.random.default_rng(3).permutation(16).astype(np.int32)
    pos = perm[ids]
    ref = oep.combine_single(pos, y)
    for world in (2, 4):
        send_pos, lists = oep.plan_destinations(pos, 16, world)
        partials = []
        for g in range(world):
            rows = lists[g]
            partials.append(oep.destination_partials(pos[rows], y[rows], g, 16, world) if len(rows)
                            else np.zeros((0, y.shape[2]), np.float32))
        got = oep.source_combine(send_pos, partials)
        assert np.array_equal(got, ref)


def _model_cost(perm, ids, world, entry_ns=12.0, row_ns=37.0):
    perm = np.asarray(perm)
    el = len(perm) // world
    owner = perm[ids] // el
    ent = np.bincount(owner.ravel(), minlength=world)
    rows = sum(len(set(o)) for o in owner)
    return entry_ns * ent.max() + row_ns * rows / world


@pytest.mark.parametrize("world", [2, 8])
def test_refine_placement_lowers_the_modelled_step_time(world):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "spectral-ai_b200"))
    from sb200.ep import balanced_placement, refine_placement
    rng = np.random.default_rng(world)
    # clustered routing like a tree router's: a token's experts come mostly
    # from one group of 8 neighbouring experts, with skewed group popularity
    T, E, k = 3000, 64, 8
    groups = rng.choice(8, size=T, p=np.array([8, 6, 5, 4, 3, 2, 1, 1]) / 30)
    ids = np.stack([np.concatenate([rng.choice(8, 6, replace=False) + 8 * g,
                                    rng.choice(E, 2, replace=False)]) for g in groups]).astype(np.int32)
    loads = np.bincount(ids.ravel(), minlength=E).astype(float)
    p0 = balanced_placement(loads, world, group=4)
    p1 = refine_placement(p0, ids, world, iters=1500, seed=1)
    assert sorted(p1) == list(range(E))
    el = E // world
    assert all(sum(1 for p in p1 if p // el == r) == el for r in range(world))
    assert _model_cost(p1, ids, world) <= _model_cost(p0, ids, world)
    # the same inputs give the same placement (every rank computes it alone)
    assert refine_placement(p0, ids, world, iters=1500, seed=1) == p1
