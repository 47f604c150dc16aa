"""EnhancedBVHRouter + BVHGateWrapper: the oracle against the reference goldens,
and the drop-in modules' host-side contract (no GPU).

Fixtures tests/golden/enhanced_*.npz come from the reference modules
(tests/golden/make_golden.py: olmoe_bvh_distill.EnhancedBVHRouter and
olmoe_e2e_eval.BVHGateWrapper); weights regenerate from
sb200.synth.enhanced_router_weights and are checked by checksum.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import enhanced as oe
from parity import topk_ids_match

ENH_GOLDENS = ["enhanced_h256", "enhanced_h256_t05", "enhanced_h256_sharp", "enhanced_cfg0"]
GATE_VARIANTS = {"softmax": ("softmax", False), "topk_softmax": ("topk_softmax", False),
                 "softmax_norm": ("softmax", True)}


def enhanced_case(name):
    """(weights, fp32 inputs, golden) with the weights and inputs checksum-checked."""
    from sb200 import synth
    g = load_golden(name)
    H = int(g["H"])
    w = synth.enhanced_router_weights(H, seed=int(g["seed"]), perturb=bool(g["perturb"]),
                                      temperature=float(g["temperature"]))
    w["expert_head.2.weight"] = (w["expert_head.2.weight"] * float(g["head_gain"])).astype(np.float32)
    x = synth.hidden_states(int(g["batch"]), H, seed=int(g["x_seed"])).numpy()

    def cs(a):
        a = np.asarray(a, np.float64)
        return np.array([a.sum(), (a * a).sum(), a.ravel()[:: max(1, a.size // 4099)].sum()])

    np.testing.assert_allclose(cs(x), g["x_checksum"], rtol=1e-9)
    for k, v in w.items():
        if k != "expert_head.2.weight":
            np.testing.assert_allclose(cs(v), g["wsum/" + k], rtol=1e-9, atol=1e-9)
    return w, x, g


def gate_key(logits, mode, dtype):
    """The values the gate ranks: softmax probabilities or the (rounded) logits."""
    lg = oe.round_to(logits, dtype)
    return oe.softmax(lg) if mode == "softmax" else lg


@pytest.mark.parametrize("name", ENH_GOLDENS)
def test_oracle_router_matches_reference(name):
    w, x, g = enhanced_case(name)
    probs, ids, logits, side = oe.router_forward(w, x)
    # fp32 against fp32: relative 1e-5, absolute 2e-6 of the largest logit
    np.testing.assert_allclose(logits, g["logits"], rtol=1e-5,
                               atol=2e-6 * max(1.0, float(np.abs(g["logits"]).max())))
    # probabilities carry the logits' absolute error as a relative one (exp):
    # 1e-4 relative, as for the BVHRouter level probabilities
    np.testing.assert_allclose(probs, g["expert_probs"], rtol=1e-4, atol=1e-8)
    assert topk_ids_match(g["expert_probs"], g["expert_ids"][:, None], ids[:, None], 1e-6) == 0
    np.testing.assert_allclose(side["geo_dist"], g["geo_dist"], rtol=1e-5, atol=1e-6)
    assert np.array_equal(side["branch_bonus"], g["branch_bonus"])
    np.testing.assert_allclose(side["h"], g["h"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("variant", list(GATE_VARIANTS))
@pytest.mark.parametrize("name", ENH_GOLDENS)
def test_oracle_gate_matches_reference(name, variant, dtype):
    w, x, g = enhanced_case(name)
    if dtype == "bf16":  # the wrapper routes the bf16 hidden states (upcast to fp32)
        x = torch.from_numpy(x).bfloat16().float().numpy()
    _, _, logits, _ = oe.router_forward(w, x)
    mode, norm = GATE_VARIANTS[variant]
    rp, tw, ti = oe.gate_topk(logits, 8, mode, norm, dtype)
    pre = f"gate/{variant}/{dtype}/"
    assert topk_ids_match(gate_key(logits, mode, dtype), g[pre + "topk_ids"], ti, 1e-6) == 0
    tw_out = oe.round_to(tw, dtype)  # the wrapper returns the weights in the hidden dtype
    # 1e-5 relative (fp32) scaled by the logit magnitude: a softmax weight carries
    # its logit's absolute error, and fp32 sums of different order differ by
    # ~1e-6 of the logit (the head_gain=20 case has logits near 8)
    wtol = 1e-5 * max(1.0, float(np.abs(logits).max()) / 4.0)
    np.testing.assert_allclose(tw_out, g[pre + "topk_weights"], rtol=wtol if dtype == "f32" else 1e-2)
    if mode == "softmax":
        # bf16: a logit next to a rounding boundary may round the other way (one bf16 ulp)
        np.testing.assert_allclose(rp, g[pre + "router_probs"], rtol=1e-4 if dtype == "f32" else 2e-2,
                                   atol=1e-7)
    else:  # the k weights land on tied ids in either order: compare each row's values
        np.testing.assert_allclose(np.sort(rp, axis=1), np.sort(g[pre + "router_probs"], axis=1),
                                   rtol=wtol if dtype == "f32" else 1e-2, atol=1e-7)


def test_dropin_state_dict_matches_reference_keys():
    from olmoe_bvh_distill import EnhancedBVHRouter
    from sb200 import synth
    r = EnhancedBVHRouter(input_dim=256, feature_dim=128)
    ref_keys = set(synth.enhanced_router_weights(256).keys())
    assert set(r.state_dict().keys()) == ref_keys
    w = synth.enhanced_router_weights(256, seed=4)
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()}, strict=True)


def test_dropin_refuses_cpu_training_and_unsupported_modes():
    from olmoe_bvh_distill import EnhancedBVHRouter
    from olmoe_e2e_eval import BVHGateWrapper
    r = EnhancedBVHRouter(input_dim=64)
    with pytest.raises(NotImplementedError):
        r(torch.randn(2, 64))          # training mode
    r.eval()
    with pytest.raises(RuntimeError):
        r(torch.randn(2, 64))          # CPU input
    with pytest.raises(NotImplementedError):
        EnhancedBVHRouter(spectral_mode=True)
    gw = BVHGateWrapper(r, weight_mode="relu_norm")
    with pytest.raises(NotImplementedError):
        gw(torch.randn(2, 64))
