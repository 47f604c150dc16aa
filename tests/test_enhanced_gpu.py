"""CUDA EnhancedBVHRouter + BVHGateWrapper against the oracle (needs a B200).

The oracle is pinned to the reference goldens by test_enhanced_cpu.py; here the
sb_enh kernels are compared with it on the same inputs:
  * EXACT engine (fp32 FFMA GEMMs): logits 1e-5 relative, expert ids and gate
    ids identical up to 1e-6 ties, gate weights 1e-5 relative (scaled by the
    logit magnitude, as in the CPU pin);
  * FAST engine (bf16 tcgen05 GEMMs): gate weights 2e-2 relative (scaled by
    the logit magnitude), ids up to ties within that tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import enhanced as oe
from parity import topk_ids_match
from test_enhanced_cpu import ENH_GOLDENS, GATE_VARIANTS, enhanced_case, gate_key

pytestmark = pytest.mark.gpu


def engine_for(w, H, device):
    from sb200.enhanced import EnhancedEngine
    eng = EnhancedEngine(H, 128, (4, 4, 4), device)
    eng.upload(w)
    return eng


def wtol_for(logits):
    return 1e-5 * max(1.0, float(np.abs(logits).max()) / 4.0)


@pytest.mark.parametrize("name", ENH_GOLDENS)
def test_exact_engine_router_outputs(cuda_device, name):
    w, x, g = enhanced_case(name)
    eng = engine_for(w, int(g["H"]), cuda_device)
    out = eng.forward(torch.from_numpy(x).to(cuda_device), precision="exact",
                      want=("logits", "expert_probs", "expert_ids", "geo_dist", "branch_bonus"))
    probs, ids, logits, side = oe.router_forward(w, x)
    got = {k: v.cpu().numpy() for k, v in out.items()}
    np.testing.assert_allclose(got["logits"], logits, rtol=1e-5, atol=2e-6 * max(1.0, float(np.abs(logits).max())))
    np.testing.assert_allclose(got["expert_probs"], probs, rtol=1e-4, atol=1e-8)
    assert topk_ids_match(probs, ids[:, None], got["expert_ids"][:, None], 1e-6) == 0
    np.testing.assert_allclose(got["geo_dist"], side["geo_dist"], rtol=1e-5, atol=1e-6)
    # the bonus follows the level argmaxes; a level whose top-2 probabilities tie
    # within 1e-6 may pick either branch
    p1s, p2s = np.sort(side["p1"], axis=1), np.sort(side["p2"], axis=1)
    tie = ((p1s[:, -1] - p1s[:, -2]) <= 1e-6 * p1s[:, -1]) | ((p2s[:, -1] - p2s[:, -2]) <= 1e-6 * p2s[:, -1])
    assert np.array_equal(got["branch_bonus"][~tie], side["branch_bonus"][~tie])


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("variant", list(GATE_VARIANTS))
@pytest.mark.parametrize("name", ENH_GOLDENS)
def test_exact_engine_gate(cuda_device, name, variant, dtype):
    w, x, g = enhanced_case(name)
    if dtype == "bf16":
        x = torch.from_numpy(x).bfloat16().float().numpy()
    mode, norm = GATE_VARIANTS[variant]
    eng = engine_for(w, int(g["H"]), cuda_device)
    out = eng.forward(torch.from_numpy(x).to(cuda_device), precision="exact", want=(), gate=mode, k=8,
                      norm_topk_prob=norm, round_dtype=torch.bfloat16 if dtype == "bf16" else torch.float32)
    _, _, logits, _ = oe.router_forward(w, x)
    rp, tw, ti = oe.gate_topk(logits, 8, mode, norm, dtype)
    ids, wts = out["topk_ids"].cpu().numpy(), out["topk_weights"].cpu().numpy()
    # bf16: one logit can round the other way (one ulp, 2^-8 relative)
    tie = 1e-6 if dtype == "f32" else 8e-3
    assert topk_ids_match(gate_key(logits, mode, dtype), ti, ids, tie) == 0
    wtol = wtol_for(logits) if dtype == "f32" else 2e-2
    np.testing.assert_allclose(np.sort(wts, axis=1), np.sort(tw, axis=1), rtol=wtol, atol=1e-7)
    np.testing.assert_allclose(np.sort(out["router_probs"].cpu().numpy(), axis=1), np.sort(rp, axis=1),
                               rtol=max(wtol, 1e-4), atol=1e-7)


@pytest.mark.parametrize("name", ["enhanced_h256", "enhanced_h256_sharp", "enhanced_cfg0"])
def test_fast_engine_gate(cuda_device, name):
    """bf16 hidden states through the bf16 tensor-core GEMMs: weights within 2e-2."""
    w, x, g = enhanced_case(name)
    xb = torch.from_numpy(x).bfloat16()
    eng = engine_for(w, int(g["H"]), cuda_device)
    out = eng.forward(xb.to(cuda_device), precision="fast", want=("logits",), gate="softmax", k=8)
    _, _, logits, _ = oe.router_forward(w, xb.float().numpy())
    rp, tw, ti = oe.gate_topk(logits, 8, "softmax", False, "bf16")
    ids, wts = out["topk_ids"].cpu().numpy(), out["topk_weights"].cpu().numpy()
    # 2e-2 relative, scaled by the logit magnitude like the fp32 bound: the bf16
    # GEMMs give the logits ~1e-2 relative error, which a softmax weight carries
    # as an absolute one (the head_gain=20 case has logits near 8)
    btol = 2e-2 * max(1.0, float(np.abs(logits).max()) / 2.0)
    assert topk_ids_match(gate_key(logits, "softmax", "bf16"), ti, ids, btol) == 0
    np.testing.assert_allclose(np.sort(wts, axis=1), np.sort(tw, axis=1), rtol=btol, atol=1e-6)
    lg = out["logits"].cpu().numpy()
    err = np.abs(lg - logits).max() / max(1.0, np.abs(logits).max())
    assert err < 2e-2, err


@pytest.mark.parametrize("B", [1, 31, 33, 1000])
def test_batch_edges_and_invariance(cuda_device, B):
    from sb200 import synth
    w = synth.enhanced_router_weights(512, seed=7)
    eng = engine_for(w, 512, cuda_device)
    x = synth.hidden_states(B, 512, seed=70 + B)
    out = eng.forward(x.to(cuda_device), precision="exact", want=("logits", "expert_ids"), gate="softmax", k=8)
    _, ids, logits, _ = oe.router_forward(w, x.numpy())
    np.testing.assert_allclose(out["logits"].cpu().numpy(), logits, rtol=1e-5, atol=2e-6)
    # each row alone gives the same bits as inside the batch
    rows = np.unique(np.linspace(0, B - 1, num=min(B, 5)).astype(np.int64))
    for r in rows:
        one = eng.forward(x[r:r + 1].to(cuda_device), precision="exact", want=("logits",), gate="softmax", k=8)
        assert torch.equal(one["logits"][0], out["logits"][r])
        assert torch.equal(one["topk_ids"][0], out["topk_ids"][r])


def test_dropin_modules(cuda_device):
    from olmoe_bvh_distill import EnhancedBVHRouter
    from olmoe_e2e_eval import BVHGateWrapper
    from sb200 import synth
    H = 256
    w = synth.enhanced_router_weights(H, seed=8)
    r = EnhancedBVHRouter(input_dim=H)
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()})
    r = r.to(cuda_device).eval()
    x = synth.hidden_states(40, H, seed=80)
    probs, ids = r(x.to(cuda_device))
    oprobs, oids, ologits, side = oe.router_forward(w, x.numpy())
    assert probs.shape == (40, 64) and ids.dtype == torch.int64
    np.testing.assert_allclose(probs.cpu().numpy(), oprobs, rtol=1e-4, atol=1e-8)
    np.testing.assert_allclose(r._last_logits.cpu().numpy(), ologits, rtol=1e-5, atol=2e-6)
    assert r._last_geometric_distances.shape == (40, 64) and r._last_branch_bonus.shape == (40, 64)
    # the gate on bf16 hidden states of a [batch, seq, H] layer input
    hs = x.reshape(2, 20, H).to(torch.bfloat16).to(cuda_device)
    gw = BVHGateWrapper(r, top_k=8)
    rp, tw, ti = gw(hs)
    assert rp.shape == (40, 64) and rp.dtype == torch.float32
    assert tw.shape == (40, 8) and tw.dtype == torch.bfloat16 and ti.dtype == torch.int64
    # affine calibration and an expert permutation fold into the expert head
    scale, bias = torch.rand(64) + 0.5, torch.randn(64) * 0.1
    perm = torch.randperm(64, generator=torch.Generator().manual_seed(3))
    gw2 = BVHGateWrapper(r, top_k=8, calibration_mode="affine",
                         calibration_state={"scale": scale, "bias": bias}, weight_mode="topk_softmax")
    gw2._expert_perm = perm
    _, tw2, ti2 = gw2(x.to(cuda_device))
    cal = (ologits * scale.numpy() + bias.numpy()).astype(np.float32)[:, torch.argsort(perm).numpy()]
    _, otw, oti = oe.gate_topk(cal, 8, "topk_softmax", False, "f32")
    assert topk_ids_match(cal, oti, ti2.cpu().numpy(), 1e-6) == 0
    np.testing.assert_allclose(np.sort(tw2.cpu().numpy(), axis=1), np.sort(otw, axis=1), rtol=1e-5, atol=1e-7)
    # a parameter update is picked up on the next call
    with torch.no_grad():
        r.expert_head[2].bias.add_(1.0)
    r(x.to(cuda_device))  # softmax is shift-invariant: the logits show the update
    np.testing.assert_allclose(r._last_logits.cpu().numpy(), ologits + 1.0, rtol=1e-5, atol=3e-6)


@pytest.mark.parametrize("branching", [(4, 4, 2), (3, 5, 2), (8, 2, 4), (2, 2, 2)])
@pytest.mark.parametrize("gate", ["softmax", "topk_softmax", "hybrid"])
def test_fast_engine_other_tree_shapes(cuda_device, branching, gate):
    """The tensor-core tail at other trees (32, 30, 64 and 8 experts; up to 8
    children per level) against the oracle, on bf16 hidden states."""
    from sb200 import synth
    from sb200.enhanced import EnhancedEngine
    H = 256
    E = int(np.prod(branching))
    w = synth.enhanced_router_weights(H, branching=branching, seed=sum(branching))
    w["expert_head.2.weight"] = (w["expert_head.2.weight"] * 10.0).astype(np.float32)
    eng = EnhancedEngine(H, 128, branching, cuda_device)
    eng.upload(w)
    k = min(4, E)
    xb = synth.hidden_states(300, H, seed=E, dtype=torch.bfloat16)
    kw = {}
    if gate == "hybrid":
        wg = synth.dense_gate_weight(E, H, seed=E)
        eng.set_dense_gate(torch.from_numpy(wg))
        kw["n_candidates"] = max(k, E // 2)
    out = eng.forward(xb.to(cuda_device), precision="fast", want=("logits", "expert_probs", "expert_ids"),
                      gate=gate, k=k, **kw)
    probs, ids, logits, _ = oe.router_forward(w, xb.float().numpy())
    scale = max(1.0, float(np.abs(logits).max()) / 2.0)
    lg = out["logits"].cpu().numpy()
    assert np.abs(lg - logits).max() / max(1.0, np.abs(logits).max()) < 2e-2
    assert topk_ids_match(probs, ids[:, None], out["expert_ids"].cpu().numpy()[:, None], 5e-2 * scale) == 0
    tw = out["topk_weights"].cpu().numpy()
    ti = out["topk_ids"].cpu().numpy()
    assert ((ti >= 0) & (ti < E)).all()
    assert (np.sort(ti, axis=1)[:, 1:] != np.sort(ti, axis=1)[:, :-1]).all()
    if gate == "softmax":
        rp, rw, ri = oe.gate_topk(logits, k, "softmax", False, "bf16")
        assert topk_ids_match(gate_key(logits, "softmax", "bf16"), ri, ti, 2e-2 * scale) == 0
        np.testing.assert_allclose(np.sort(tw, axis=1), np.sort(rw, axis=1), rtol=2e-2 * scale, atol=1e-6)
    elif gate == "topk_softmax":
        np.testing.assert_allclose(tw.sum(axis=1), 1.0, rtol=1e-5)
    else:
        full = out["router_probs"].cpu().numpy()
        np.testing.assert_allclose(full.sum(axis=1), 1.0, rtol=1e-5)
        # every chosen expert is among the BVH candidates of the kernel's own probabilities
        cand = np.argsort(-out["expert_probs"].cpu().numpy(), axis=1, kind="stable")[:, :kw["n_candidates"]]
        assert all(set(r) <= set(c) for r, c in zip(ti, cand))
