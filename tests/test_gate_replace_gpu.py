"""Hybrid pre-filter gate and replace_gate_with_bvh on the GPU (needs a B200).

The CUDA path (sb_enh_forward_hybrid: router kernels + dense gate GEMM + the
selection in the tail kernel) against the oracle pinned in
test_gate_replace_cpu.py, and the drop-in replace_gate_with_bvh against the
reference's own outputs (tests/golden/gate_replace_*.npz):
  * EXACT engine: dense probabilities 1e-5 relative (fp32 hidden states),
    scaled by max(1, max |dense logit| / 2) since a probability carries its
    logit's absolute fp32 summation error as a relative one;
    candidate sets identical except where the n-th and (n+1)-th BVH
    probabilities tie within 1e-4; ids identical up to dense-probability ties;
  * bf16 hidden states: a dense logit may round one bf16 ulp the other way
    (fp32 sums of another order), so probabilities within 5e-2 and 99.5 % of
    them within 1e-5 (95 % for the tensor-core dense gate of the FAST engine);
  * FAST engine (bf16 tensor-core router): the BVH probabilities carry ~1e-2
    relative error, so candidate-boundary ties are excused within 5e-2.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import enhanced as oe
from parity import hybrid_ids_mismatch, topk_ids_match
from test_gate_replace_cpu import GATE_GOLDENS, gate_case, oracle_hybrid

pytestmark = pytest.mark.gpu


def engine_for(w, wg, H, device, gate_dtype):
    from sb200.enhanced import EnhancedEngine
    eng = EnhancedEngine(H, 128, (4, 4, 4), device)
    eng.upload(w)
    eng.set_dense_gate(torch.from_numpy(wg).to(gate_dtype))
    return eng


def logit_scale(x, wg):
    """max(1, max |dense logit| / 2): a probability carries its logit's absolute
    error (fp32 sums over the hidden size, ~1e-6 of the logit) as a relative one."""
    return max(1.0, float(np.abs(np.asarray(x, np.float64) @ np.asarray(wg, np.float64).T).max()) / 2.0)


def check_probs(got, ref, dtype, scale=1.0, agree=0.995):
    if dtype == "f32":
        np.testing.assert_allclose(got, ref, rtol=1e-5 * scale, atol=1e-8)
    else:
        np.testing.assert_allclose(got, ref, rtol=5e-2, atol=1e-8)
        assert (np.abs(got - ref) <= 1e-5 * np.abs(ref) + 1e-8).mean() > agree


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("n_cand", [8, 16, 48, 64])
@pytest.mark.parametrize("name", GATE_GOLDENS)
def test_exact_hybrid_matches_oracle(cuda_device, name, n_cand, norm, dtype):
    w, wg, x, g = gate_case(name)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    eng = engine_for(w, wg, int(g["H"]), cuda_device, tdt)
    xt = torch.from_numpy(x).to(tdt).to(cuda_device)
    out = eng.forward(xt, precision="exact", want=("expert_probs",), gate="hybrid", k=8, norm_topk_prob=norm,
                      n_candidates=n_cand)
    bvh, fp, tw, ti = oracle_hybrid(w, wg, x, n_cand, norm, dtype)
    np.testing.assert_allclose(out["expert_probs"].cpu().numpy(), bvh, rtol=1e-4, atol=1e-8)
    sc = logit_scale(x, wg)
    check_probs(out["router_probs"].cpu().numpy(), fp, dtype, sc)
    ids = out["topk_ids"].cpu().numpy()
    assert hybrid_ids_mismatch(bvh, fp, n_cand, ti, ids, 1e-4, 1e-5 * sc if dtype == "f32" else 5e-2) == 0
    np.testing.assert_allclose(np.sort(out["topk_weights"].cpu().numpy(), axis=1), np.sort(tw, axis=1),
                               rtol=1e-5 * sc if dtype == "f32" else 5e-2, atol=1e-8)
    if n_cand == 64:  # every expert a candidate: the dense gate's own top-k
        _, dw, di = oe.gate_topk(oe.dense_gate_logits(torch.from_numpy(x).to(tdt).float().numpy(),
                                                      torch.from_numpy(wg).to(tdt).float().numpy(), dtype),
                                 8, "softmax", norm, "f32")
        assert topk_ids_match(fp, di, ids, 1e-5 * sc if dtype == "f32" else 5e-2) == 0


@pytest.mark.parametrize("name", GATE_GOLDENS)
def test_fast_hybrid_matches_oracle(cuda_device, name):
    w, wg, x, g = gate_case(name)
    eng = engine_for(w, wg, int(g["H"]), cuda_device, torch.bfloat16)
    xt = torch.from_numpy(x).bfloat16().to(cuda_device)
    out = eng.forward(xt, precision="fast", want=(), gate="hybrid", k=8, n_candidates=16)
    bvh, fp, tw, ti = oracle_hybrid(w, wg, x, 16, False, "bf16")
    # tensor-core fp32 sums are not IEEE-ordered: a bf16 logit rounds the other
    # way more often than with the FFMA engine (1.5 % of entries at H=2048)
    check_probs(out["router_probs"].cpu().numpy(), fp, "bf16", agree=0.95)
    assert hybrid_ids_mismatch(bvh, fp, 16, ti, out["topk_ids"].cpu().numpy(), 5e-2, 5e-2) == 0


@pytest.mark.parametrize("B", [1, 31, 33, 4097])
def test_hybrid_batch_edges(cuda_device, B):
    from sb200 import synth
    H = 512
    w = synth.enhanced_router_weights(H, seed=9)
    wg = synth.dense_gate_weight(64, H, seed=9)
    eng = engine_for(w, wg, H, cuda_device, torch.float32)
    x = synth.hidden_states(B, H, seed=90 + B)
    out = eng.forward(x.to(cuda_device), precision="exact", want=(), gate="hybrid", k=8, n_candidates=16)
    bvh, fp, tw, ti = oracle_hybrid(w, wg, x.numpy(), 16, False, "f32")
    sc = logit_scale(x.numpy(), wg)
    check_probs(out["router_probs"].cpu().numpy(), fp, "f32", sc)
    assert hybrid_ids_mismatch(bvh, fp, 16, ti, out["topk_ids"].cpu().numpy(), 1e-4, 1e-5 * sc) == 0
    one = eng.forward(x[-1:].to(cuda_device), precision="exact", want=(), gate="hybrid", k=8, n_candidates=16)
    assert torch.equal(one["topk_ids"][0], out["topk_ids"][-1])


def test_hybrid_argument_errors(cuda_device):
    from sb200 import synth
    from sb200.enhanced import EnhancedEngine
    H = 256
    eng = EnhancedEngine(H, 128, (4, 4, 4), cuda_device)
    eng.upload(synth.enhanced_router_weights(H, seed=1))
    x = synth.hidden_states(4, H, seed=1).to(cuda_device)
    with pytest.raises(RuntimeError):   # no dense gate uploaded
        eng.forward(x, precision="exact", want=(), gate="hybrid", k=8, n_candidates=16)
    eng.set_dense_gate(torch.from_numpy(synth.dense_gate_weight(64, H)))
    with pytest.raises(RuntimeError):   # fewer candidates than k
        eng.forward(x, precision="exact", want=(), gate="hybrid", k=8, n_candidates=4)
    with pytest.raises(RuntimeError):   # wrong gate shape
        eng.set_dense_gate(torch.zeros(64, H + 8))


def _host(H, wg, dt, device):
    m = torch.nn.Module()
    m.model = torch.nn.Module()
    layer = torch.nn.Module()
    layer.mlp = torch.nn.Module()
    gate = torch.nn.Linear(H, 64, bias=False)
    with torch.no_grad():
        gate.weight.copy_(torch.from_numpy(wg))
    gate.top_k, gate.norm_topk_prob = 8, False
    layer.mlp.gate = gate
    m.model.layers = torch.nn.ModuleList([layer])
    return m.to(dt).to(device)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("name", GATE_GOLDENS)
def test_dropin_replace_gate_against_reference(cuda_device, tmp_path, name, dtype):
    """Our replace_gate_with_bvh on the reference's checkpoint format against
    the reference's replace_gate_with_bvh outputs: hybrid (n = 16, 48) and the
    pure calibrated + permuted gate."""
    from olmoe_e2e_eval import find_gate_module, replace_gate_with_bvh
    w, wg, x, g = gate_case(name)
    H, B = int(g["H"]), int(g["batch"])
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    sd = {k: torch.from_numpy(np.array(v)) for k, v in w.items()}
    cfg = {"input_dim": H, "n_level1": 4, "n_level2": 4, "n_level3": 4, "feature_dim": 128}
    plain, calib = tmp_path / "r.pt", tmp_path / "rc.pt"
    torch.save({"config": cfg, "router_state_dict": sd}, plain)
    torch.save({"config": cfg, "router_state_dict": sd, "calibration_mode": "affine",
                "calibration_state": {"scale": torch.from_numpy(g["cal_scale"]),
                                      "bias": torch.from_numpy(g["cal_bias"])},
                "expert_perm": g["expert_perm"].tolist()}, calib)
    xs = torch.from_numpy(x).to(tdt).to(cuda_device)
    bvh = oe.router_forward(w, xs.float().cpu().numpy())[0]
    sc = logit_scale(x, wg)
    for n_cand in (16, 48):
        m = _host(H, wg, tdt, cuda_device)
        replace_gate_with_bvh(m, str(plain), layer_idx=0, hybrid=True, n_candidates=n_cand)
        gate = getattr(*find_gate_module(m, 0))
        gate.forward.__self__.router.precision = "exact"
        fp, ts, ti = gate(xs.reshape(2, B // 2, H))
        pre = f"hybrid/{n_cand}/0/{dtype}/"
        assert fp.dtype == torch.float32 and ts.dtype == tdt and ti.dtype == torch.int64
        check_probs(fp.cpu().numpy(), g[pre + "router_probs"], dtype, sc)
        assert hybrid_ids_mismatch(bvh, g[pre + "router_probs"], n_cand, g[pre + "topk_ids"], ti.cpu().numpy(),
                                   1e-4, 1e-5 * sc if dtype == "f32" else 5e-2) == 0
        np.testing.assert_allclose(np.sort(ts.float().cpu().numpy(), axis=1),
                                   np.sort(g[pre + "topk_weights"], axis=1),
                                   rtol=1e-5 * sc if dtype == "f32" else 5e-2, atol=1e-8)
    m = _host(H, wg, tdt, cuda_device)
    replace_gate_with_bvh(m, str(calib), layer_idx=0, hybrid=False)
    wrapper = getattr(*find_gate_module(m, 0))
    wrapper.router.precision = "exact"
    rp, tw, ti = wrapper(xs)
    pre = f"pure_cal/{dtype}/"
    tol = 1e-5 if dtype == "f32" else 8e-3
    assert topk_ids_match(g[pre + "router_probs"], g[pre + "topk_ids"], ti.cpu().numpy(), tol) == 0
    np.testing.assert_allclose(rp.cpu().numpy(), g[pre + "router_probs"],
                               rtol=1e-4 if dtype == "f32" else 2e-2, atol=1e-7)
