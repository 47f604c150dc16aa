"""replace_gate_with_bvh: the hybrid pre-filter gate and the checkpoint loader
(no GPU).

Fixtures tests/golden/gate_replace_*.npz come from the reference's own
replace_gate_with_bvh (python/olmoe_e2e_eval.py:1177-1404) run on a checkpoint
written with torch.save and a stand-in model holding a dense gate
(tests/golden/make_golden.py); the router and gate weights regenerate from
sb200.synth and are checked by checksum.  Here the oracle's restatement of the
hybrid gate is pinned to them, and the drop-in loader is checked on the host.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import enhanced as oe
from parity import hybrid_ids_mismatch, topk_ids_match

GATE_GOLDENS = ["gate_replace_h256", "gate_replace_h2048"]


def _cs(a):
    a = np.asarray(a, np.float64)
    return np.array([a.sum(), (a * a).sum(), a.ravel()[:: max(1, a.size // 4099)].sum()])


def gate_case(name):
    """(router weights, dense gate weight, fp32 inputs, golden), checksum-checked."""
    from sb200 import synth
    g = load_golden(name)
    H = int(g["H"])
    w = synth.enhanced_router_weights(H, seed=int(g["seed"]))
    w["expert_head.2.weight"] = (w["expert_head.2.weight"] * float(g["head_gain"])).astype(np.float32)
    wg = synth.dense_gate_weight(64, H, seed=int(g["gate_seed"]))
    x = synth.hidden_states(int(g["batch"]), H, seed=int(g["x_seed"])).numpy()
    np.testing.assert_allclose(_cs(x), g["x_checksum"], rtol=1e-9)
    np.testing.assert_allclose(_cs(wg), g["wg_checksum"], rtol=1e-9)
    return w, wg, x, g


def in_dtype(a, dtype):
    """The hidden states / gate weight as the reference holds them (bf16 or fp32), as fp32."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    return (t.bfloat16().float() if dtype == "bf16" else t).numpy()


def oracle_hybrid(w, wg, x, n_cand, norm, dtype):
    xd = in_dtype(x, dtype)
    bvh_probs, _, _, _ = oe.router_forward(w, xd)
    full_logits = oe.dense_gate_logits(xd, in_dtype(wg, dtype), dtype)
    fp, tw, ti = oe.hybrid_gate(bvh_probs, full_logits, n_cand, 8, norm)
    return bvh_probs, fp, tw, ti


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("norm", [0, 1])
@pytest.mark.parametrize("n_cand", [16, 48])
@pytest.mark.parametrize("name", GATE_GOLDENS)
def test_oracle_hybrid_matches_reference(name, n_cand, norm, dtype):
    w, wg, x, g = gate_case(name)
    bvh, fp, tw, ti = oracle_hybrid(w, wg, x, n_cand, bool(norm), dtype)
    pre = f"hybrid/{n_cand}/{norm}/{dtype}/"
    gp, gw, gi = g[pre + "router_probs"], g[pre + "topk_weights"], g[pre + "topk_ids"]
    if dtype == "f32":
        np.testing.assert_allclose(fp, gp, rtol=1e-5, atol=1e-8)
    else:
        # bf16 logits: a product summed in another order may round one ulp
        # (2^-8 relative) the other way; 99.5 % of entries still agree to 1e-5
        np.testing.assert_allclose(fp, gp, rtol=5e-2, atol=1e-8)
        assert (np.abs(fp - gp) <= 1e-5 * np.abs(gp) + 1e-8).mean() > 0.995
    tie_full = 1e-6 if dtype == "f32" else 5e-2
    assert hybrid_ids_mismatch(bvh, fp, n_cand, gi, ti, 1e-6, tie_full) == 0
    np.testing.assert_allclose(np.sort(oe.round_to(tw, dtype), axis=1), np.sort(gw, axis=1),
                               rtol=1e-5 if dtype == "f32" else 5e-2, atol=1e-8)
    # every selected id is a candidate, distinct per row
    cand = np.argsort(-bvh, axis=1, kind="stable")[:, :n_cand]
    assert all(set(r) <= set(c) for r, c in zip(ti, cand))
    assert (np.sort(ti, axis=1)[:, 1:] != np.sort(ti, axis=1)[:, :-1]).all()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("name", GATE_GOLDENS)
def test_oracle_pure_calibrated_matches_reference(name, dtype):
    """Pure replacement: affine calibration, bf16/fp32 rounding, then the
    inverse expert permutation (olmoe_e2e_eval.py:371-387), softmax top-8."""
    w, wg, x, g = gate_case(name)
    xd = in_dtype(x, dtype)
    _, _, logits, _ = oe.router_forward(w, xd)
    cal = (logits * g["cal_scale"] + g["cal_bias"]).astype(np.float32)
    cal = oe.round_to(cal, dtype)[:, np.argsort(g["expert_perm"])]
    rp, tw, ti = oe.gate_topk(cal, 8, "softmax", False, "f32")
    pre = f"pure_cal/{dtype}/"
    tol = 1e-6 if dtype == "f32" else 8e-3
    assert topk_ids_match(oe.softmax(cal), g[pre + "topk_ids"], ti, tol) == 0
    np.testing.assert_allclose(rp, g[pre + "router_probs"], rtol=1e-4 if dtype == "f32" else 2e-2, atol=1e-7)


def test_dropin_loader_builds_the_reference_objects(tmp_path):
    """The drop-in replace_gate_with_bvh reads the reference checkpoint format
    and installs the same gate objects (host side only)."""
    from olmoe_e2e_eval import BVHGateWrapper, HybridGate, find_gate_module, replace_gate_with_bvh
    w, wg, x, g = gate_case("gate_replace_h256")
    sd = {k: torch.from_numpy(np.array(v)) for k, v in w.items()}
    cfg = {"input_dim": 256, "n_level1": 4, "n_level2": 4, "n_level3": 4, "feature_dim": 128}
    ck = tmp_path / "r.pt"
    cal = {"scale": torch.from_numpy(g["cal_scale"]), "bias": torch.from_numpy(g["cal_bias"])}
    torch.save({"config": cfg, "router_state_dict": sd, "calibration_mode": "affine", "calibration_state": cal,
                "expert_perm": g["expert_perm"].tolist()}, ck)

    def host():
        m = torch.nn.Module()
        m.model = torch.nn.Module()
        layer = torch.nn.Module()
        layer.mlp = torch.nn.Module()
        gate = torch.nn.Linear(256, 64, bias=False)
        with torch.no_grad():
            gate.weight.copy_(torch.from_numpy(wg))
        gate.top_k, gate.norm_topk_prob = 8, False
        layer.mlp.gate = gate
        m.model.layers = torch.nn.ModuleList([layer])
        return m

    m = host()
    orig, fwd = replace_gate_with_bvh(m, str(ck), layer_idx=0, hybrid=False)
    mlp, attr = find_gate_module(m, 0)
    wrapper = getattr(mlp, attr)
    assert isinstance(wrapper, BVHGateWrapper) and fwd is None and isinstance(orig, torch.nn.Linear)
    assert wrapper.calibration_mode == "affine" and wrapper.top_k == 8
    assert torch.equal(wrapper._expert_perm.cpu(), torch.from_numpy(g["expert_perm"]).long())
    for k, v in sd.items():
        assert torch.equal(wrapper.router.state_dict()[k].cpu(), v), k
    m2 = host()
    orig2, fwd2 = replace_gate_with_bvh(m2, str(ck), layer_idx=0, hybrid=True, n_candidates=48)
    gate2 = getattr(*find_gate_module(m2, 0))
    # the gate module stays (its state_dict too); its forward is the hybrid gate
    assert gate2 is orig2 and isinstance(gate2, torch.nn.Linear) and callable(fwd2)
    hg = gate2.forward.__self__
    assert isinstance(hg, HybridGate) and hg.n_candidates == 48 and hg.top_k == 8
    assert set(gate2.state_dict().keys()) == {"weight"}
    assert torch.equal(hg.weight.cpu(), torch.from_numpy(wg))
    with pytest.raises(RuntimeError):
        gate2(torch.from_numpy(x))   # CPU input: there is no CPU path
    with pytest.raises(RuntimeError):
        find_gate_module(m2, 3)
