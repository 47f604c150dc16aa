"""MoE pipeline stages: the oracle against the reference simulator (no GPU).

tests/golden/pipeline_h256.npz comes from the reference's own
AsyncPipelineSimulator (python/async_pipeline_bridge.py:49-255) run on the CPU
by tests/golden/make_golden.py: an EnhancedBVHRouter, 64 small dense experts
and, in the "cal" variant, a Linear(64,64) calibration.  Weights and inputs
regenerate from sb200.synth and are checked by checksum.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import enhanced as oe
from oracle import pipeline as op
from parity import topk_ids_match


def gelu(x):
    from scipy.special import erf
    return 0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))


def pipeline_case(name="pipeline_h256"):
    from sb200 import synth
    g = load_golden(name)
    H, seed = int(g["H"]), int(g["seed"])
    w = synth.enhanced_router_weights(H, seed=seed)
    w["expert_head.2.weight"] = (w["expert_head.2.weight"] * float(g["head_gain"])).astype(np.float32)
    experts = synth.mlp_experts(64, H, int(g["inner"]), seed=seed)
    cal = synth.calibration_linear(64, seed=seed)
    x = synth.hidden_states(int(g["batch"]), H, seed=int(g["x_seed"])).numpy()
    a = np.asarray(x, np.float64)
    np.testing.assert_allclose([a.sum(), (a * a).sum(), a.ravel()[:: max(1, a.size // 4099)].sum()],
                               g["x_checksum"], rtol=1e-9)
    return w, experts, cal, x, g


def mlp(sd, x):
    h = gelu(np.asarray(x, np.float64) @ sd["0.weight"].T.astype(np.float64) + sd["0.bias"])
    return h @ sd["2.weight"].T.astype(np.float64) + sd["2.bias"]


def oracle_route(w, cal, x, variant):
    probs, _, logits, _ = oe.router_forward(w, x)
    if variant == "cal":
        p, ids, wts = op.softmax_topk(logits, 8, cal["weight"], cal["bias"])
    else:
        p, ids, wts = op.softmax_topk(probs, 8, apply_softmax=False)
    return p, ids, wts


@pytest.mark.parametrize("variant", ["plain", "cal"])
def test_oracle_route_stage_matches_reference(variant):
    w, experts, cal, x, g = pipeline_case()
    p, ids, wts = oracle_route(w, cal, x, variant)
    assert topk_ids_match(p, g[f"{variant}/expert_ids"], ids, 1e-5) == 0
    np.testing.assert_allclose(np.sort(wts, axis=1), np.sort(g[f"{variant}/expert_weights"], axis=1),
                               rtol=1e-4, atol=1e-8)


@pytest.mark.parametrize("variant", ["plain", "cal"])
def test_oracle_scatter_matches_reference(variant):
    """Integer work: exact, on the reference's own routing ids."""
    g = load_golden("pipeline_h256")
    ids = g[f"{variant}/expert_ids"]
    disp, counts = op.scatter_by_expert(ids, 64, ids.shape[0])
    assert np.array_equal(counts, g[f"{variant}/counts"])
    lists = np.concatenate([disp[e, :counts[e]] for e in range(64)])
    assert np.array_equal(lists, g[f"{variant}/lists"])


@pytest.mark.parametrize("variant", ["plain", "cal"])
def test_oracle_expert_stage_matches_reference(variant):
    w, experts, cal, x, g = pipeline_case()
    ids, wts = g[f"{variant}/expert_ids"], g[f"{variant}/expert_weights"]
    B, k = ids.shape
    eo = np.zeros((B, k, x.shape[1]))
    for t in range(B):
        for j in range(k):
            eo[t, j] = mlp(experts[ids[t, j]], x[t:t + 1])[0]
    out = op.weighted_combine(eo, wts)
    np.testing.assert_allclose(out, g[f"{variant}/output"], rtol=1e-4, atol=1e-5)


def test_scatter_limit_and_sentinel():
    ids = np.array([[0, 1], [1, 7], [1, 0], [9, 1]])
    disp, counts = op.scatter_by_expert(ids, 8, 2)
    assert counts.tolist() == [2, 4, 0, 0, 0, 0, 0, 1]   # id 9 >= E is skipped; counts unclamped
    assert disp[1].tolist() == [0, 1] and disp[0].tolist() == [0, 2] and disp[7].tolist() == [1, -1]
    disp2, _ = op.scatter_by_expert(ids, 8, 4, store_entry=True)
    assert disp2[1].tolist() == [1, 2, 4, 7]


def test_dropin_refuses_cpu():
    from async_pipeline_bridge import AsyncPipelineSimulator, DispatchTable, PipelineConfig
    with pytest.raises(RuntimeError):
        AsyncPipelineSimulator(PipelineConfig(), torch.nn.Identity(), torch.nn.ModuleList(), device="cpu")
    t = DispatchTable(torch.tensor([[1, 4, 0], [3, 0, 0]], dtype=torch.int32), torch.tensor([2, 1]), 2)
    assert t.as_dict() == {0: [0, 2], 1: [1]}
