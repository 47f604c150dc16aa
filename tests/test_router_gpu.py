"""CUDA router parity against the oracle and the reference goldens (needs a B200).

Contract:
  * route paths / expert ids identical except where the deciding logits are
    within 1e-6 of each other (oracle margins, relative to max(1, |logit|));
  * routing weights within 1e-5 relative on the fp32 (EXACT) engine and
    within 2e-2 relative on the bf16 tensor-core (FAST) engine.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ROUTER_GOLDENS, golden_router_case
from oracle import router as orouter
from parity import TIE, compare_paths, topk_ids_match

pytestmark = pytest.mark.gpu


def make_router(w, H, S, branching, device):
    from bvh_router import BVHRouter, RouterConfig
    cfg = RouterConfig(embed_dim=H, spectral_dim=S, branching=branching)
    r = BVHRouter(cfg)
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()})
    return r.to(device).eval()


def check_against(ref, got, mode, wtol, ptol=None):
    """ref: oracle dict (numpy); got: dict of torch tensors."""
    path = got["route_path"].cpu().numpy()
    bad, excused = compare_paths(ref["route_path"], path, ref["level_margins"])
    assert bad == 0, f"{bad} route paths differ beyond ties"
    keep = ~excused
    assert excused.sum() <= max(2, keep.size // 50)
    assert np.array_equal(got["expert_id"].cpu().numpy()[keep], ref["expert_id"][keep])
    probs = got["expert_probs"].cpu().numpy()
    np.testing.assert_allclose(probs[keep], ref["expert_probs"][keep],
                               rtol=ptol or wtol, atol=1e-8 if ptol is None else 1e-6)
    # confidence is a level probability: same tolerance as expert_probs
    np.testing.assert_allclose(got["confidence"].cpu().numpy()[keep], ref["confidence"][keep],
                               rtol=ptol or wtol)
    if "topk_ids" in got:
        ids = got["topk_ids"].cpu().numpy()
        tol = 1e-6 if wtol <= 1e-5 else wtol
        assert topk_ids_match(ref["expert_probs"][keep], ref["topk_ids"][keep], ids[keep], tol) == 0
        np.testing.assert_allclose(got["topk_weights"].cpu().numpy()[keep], ref["topk_weights"][keep],
                                   rtol=wtol)


@pytest.mark.parametrize("mode", ["hard", "soft"])
@pytest.mark.parametrize("name", ROUTER_GOLDENS)
def test_exact_engine_matches_reference_goldens(cuda_device, name, mode):
    w, x, g = golden_router_case(name)
    H, S = int(g["H"]), int(g["S"])
    br = tuple(int(b) for b in g["branching"])
    r = make_router(w, H, S, br, cuda_device)
    xt = torch.from_numpy(x).to(cuda_device)
    k = min(8, int(np.prod(br)))
    got = r.route(xt, select=mode, k=k, precision="exact")
    ref = orouter.router_forward(w, x, br, mode=mode, k=k)
    # oracle pinned to the reference goldens in test_oracle; here CUDA vs oracle
    check_against(ref, got, mode, wtol=1e-5, ptol=1e-4)
    # and directly against the reference's own ids where no tie is involved
    bad, _ = compare_paths(g[f"{mode}_route_path"], got["route_path"].cpu().numpy(), ref["level_margins"])
    assert bad == 0


@pytest.mark.parametrize("name", ["router_cfg0", "router_cfg0_perturbed"])
def test_fast_engine_hard_mode(cuda_device, name):
    """bf16 tensor-core encoder: ids exact (the decisions depend on the fp32 position path)."""
    w, x, g = golden_router_case(name)
    H, S = int(g["H"]), int(g["S"])
    r = make_router(w, H, S, (4, 4, 4), cuda_device)
    xb = torch.from_numpy(x).to(torch.bfloat16)
    got = r.route(xb.to(cuda_device), select="hard", k=8, precision="fast")
    ref = orouter.router_forward(w, xb.float().numpy(), (4, 4, 4), mode="hard", k=8)
    check_against(ref, got, "hard", wtol=2e-2)
    # against the oracle that rounds where the FAST engine rounds: the level
    # probabilities (one-hot x refraction) within the FAST tie window
    ref16 = orouter.router_forward(w, xb.float().numpy(), (4, 4, 4), mode="hard", k=8, arith="bf16")
    check_against(ref16, got, "hard", wtol=FAST_TIE)


# The FAST engine rounds the encoder's hidden state G and the spectral row to
# bf16.  Two fp32-or-better summation orders of the same sums (the tensor
# cores' and the oracle's float64) land on different sides of a bf16 rounding
# boundary for about 1 in 4e4 elements, and one such flip moves a level
# probability by up to 1.7e-3 relative (measured on the CPU between float64 and
# float32 summation with the same roundings).  So FAST top-8 ids are identical
# to the bf16-faithful oracle's except where two probabilities lie within
# FAST_TIE of each other; the fp32 engine is held to the 1e-6 rule.
FAST_TIE = 2e-3


def _fast_soft_check(w, xb, got):
    """FAST soft top-8 against the bf16-faithful oracle: ids identical except
    within FAST_TIE, excused positions rare, weights within FAST_TIE; against
    the fp32 (reference-arithmetic) oracle the weights stay within the bf16
    contract's 2e-2."""
    ref16 = orouter.router_forward(w, xb, (4, 4, 4), mode="soft", k=8, arith="bf16")
    ids = got["topk_ids"].cpu().numpy()
    bad = topk_ids_match(ref16["expert_probs"], ref16["topk_ids"], ids, FAST_TIE)
    assert bad == 0, f"{bad} top-8 positions differ beyond {FAST_TIE} ties"
    excused = topk_ids_match(ref16["expert_probs"], ref16["topk_ids"], ids, TIE)
    print(f"top-8 positions differing within the FAST tie window: {excused} of {ids.size}")
    assert excused <= max(4, ids.size // 500)
    np.testing.assert_allclose(got["topk_weights"].cpu().numpy(), ref16["topk_weights"], rtol=FAST_TIE)
    ref = orouter.router_forward(w, xb, (4, 4, 4), mode="soft", k=8)
    np.testing.assert_allclose(got["topk_weights"].cpu().numpy(), ref["topk_weights"], rtol=2e-2)


@pytest.mark.parametrize("name", ["router_cfg0", "router_cfg0_perturbed"])
def test_fast_engine_soft_mode(cuda_device, name):
    """bf16 encoder in soft mode (the headline's selection)."""
    w, x, g = golden_router_case(name)
    H, S = int(g["H"]), int(g["S"])
    r = make_router(w, H, S, (4, 4, 4), cuda_device)
    xb = torch.from_numpy(x).to(torch.bfloat16)
    got = r.route(xb.to(cuda_device), select="soft", k=8, precision="fast")
    _fast_soft_check(w, xb.float().numpy(), got)


@pytest.mark.parametrize("B", [4096, 1])
def test_fast_engine_soft_mode_headline_shape(cuda_device, B):
    """The headline's router: seed-0 weights, unit-RMS bf16 tokens (seed 2), 4096 tokens and one."""
    from sb200 import synth
    H, S = 2048, 256
    w = synth.router_weights(H, S, seed=0)
    r = make_router(w, H, S, (4, 4, 4), cuda_device)
    xb = synth.hidden_states(B, H, seed=2, dtype=torch.bfloat16)
    got = r.route(xb.to(cuda_device), select="soft", k=8, precision="fast")
    _fast_soft_check(w, xb.float().numpy(), got)


@pytest.mark.parametrize("B", [300, 8500])
def test_encoder_gemms_against_torch_fp32(cuda_device, B):
    """The tcgen05 GEMM chain (bf16 in, fp32 accumulate) against a torch fp32
    reference: B=300 runs the single-CTA GEMM, B=8500 (34 row blocks of 256,
    the last one ragged) the CTA-pair GEMM, both with the 3-D position tail."""
    from sb200 import synth
    H, S = 2048, 256
    w = synth.router_weights(H, S, seed=11, perturb=True)
    r = make_router(w, H, S, (4, 4, 4), cuda_device)
    x = synth.hidden_states(B, H, seed=12, dtype=torch.bfloat16, device=cuda_device)
    eng = r.sync_weights(cuda_device)
    eng.forward(x, precision="fast", select="hard", want=("expert_id",))
    ws = eng._ws
    base = (ws.data_ptr() + 1023) // 1024 * 1024 - ws.data_ptr()
    G = ws[base: base + B * H * 2].view(torch.bfloat16).view(B, H).float()
    W1 = torch.from_numpy(w["spectral.net.0.weight"]).to(cuda_device).bfloat16().float()
    b1 = torch.from_numpy(w["spectral.net.0.bias"]).to(cuda_device)
    G_ref = torch.nn.functional.gelu(x.float() @ W1.T + b1)
    err = (G - G_ref).abs() / (G_ref.abs() + 1e-2)
    assert err.max().item() < 1e-2, err.max().item()
    # the position tail: x @ W3^T + b3 from three bf16 pieces of W3 (fp32-accurate)
    pos_off = base + (B * H * 2 + 1023) // 1024 * 1024 + (B * S * 2 + 1023) // 1024 * 1024
    pos = ws[pos_off: pos_off + B * 16].view(torch.float32).view(B, 4)
    W3 = torch.from_numpy(w["to_3d.weight"]).to(cuda_device).double()
    b3 = torch.from_numpy(w["to_3d.bias"]).to(cuda_device).double()
    pos_ref = x.double() @ W3.T + b3
    torch.testing.assert_close(pos[:, :3].double(), pos_ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("B", [1, 3, 129, 256, 4096, 65536])
def test_config1_sizes_sampled_parity_and_batch_invariance(cuda_device, B):
    """Config-1 shapes: sampled rows against the oracle, all rows by properties."""
    from sb200 import synth
    H, S = 2048, 256
    w = synth.router_weights(H, S, seed=0)
    r = make_router(w, H, S, (4, 4, 4), cuda_device)
    x = synth.hidden_states(B, H, seed=1, dtype=torch.bfloat16, device=cuda_device)
    got = r.route(x, select="hard", k=8, precision="fast")
    ids, wts = got["topk_ids"], got["topk_weights"]
    probs = got["expert_probs"]
    # properties on every row
    assert ((probs > 0).sum(dim=1) == 1).all()
    assert torch.equal(got["expert_id"], got["route_path"][:, -1])
    assert torch.equal(ids[:, 0].long(), got["expert_id"])
    torch.testing.assert_close(wts.sum(dim=1), torch.ones(B, device=cuda_device), rtol=1e-5, atol=1e-6)
    assert int(ids.min()) >= 0 and int(ids.max()) < 64
    assert (ids.sort(dim=1).values.diff(dim=1) != 0).all()   # distinct ids per row
    # determinism: identical bits on a second run
    again = r.route(x, select="hard", k=8, precision="fast")
    for key in ("topk_ids", "topk_weights", "expert_probs", "route_path"):
        assert torch.equal(got[key], again[key])
    # sampled rows against the oracle
    rows = np.unique(np.linspace(0, B - 1, num=min(B, 384)).astype(np.int64))
    ref = orouter.router_forward(w, x[rows].float().cpu().numpy(), (4, 4, 4), mode="hard", k=8)
    sub = {k: v[torch.from_numpy(rows).to(cuda_device)] for k, v in got.items()}
    check_against(ref, sub, "hard", wtol=2e-2)
    # batch invariance: the sampled rows routed alone give the same bits
    alone = r.route(x[torch.from_numpy(rows).to(cuda_device)].contiguous(), select="hard", k=8,
                    precision="fast")
    for key in ("topk_ids", "route_path"):
        assert torch.equal(alone[key], sub[key])


def test_empty_batch(cuda_device):
    from sb200 import synth
    w = synth.router_weights(64, 16, seed=0)
    r = make_router(w, 64, 16, (4, 4, 4), cuda_device)
    out = r(torch.empty(0, 64, device=cuda_device))
    assert out.expert_id.shape == (0,) and out.expert_probs.shape == (0, 64)


def test_reference_api_surface(cuda_device):
    """forward(x) in eval returns RoutingResult with the reference shapes/dtypes."""
    from bvh_router import RoutingResult
    from sb200 import synth
    w = synth.router_weights(64, 16, seed=0, perturb=True)
    r = make_router(w, 64, 16, (4, 4, 4), cuda_device)
    x = synth.hidden_states(8, 64, seed=42, device=cuda_device)
    out = r(x)
    assert isinstance(out, RoutingResult)
    assert out.expert_id.shape == (8,) and out.expert_id.dtype == torch.int64
    assert out.expert_probs.shape == (8, 64) and out.route_path.shape == (8, 3)
    assert out.confidence.shape == (8,)
    # a parameter update is picked up on the next forward (weights re-uploaded)
    with torch.no_grad():
        r.to_3d.bias.add_(5.0)
    out2 = r(x)
    ref = orouter.router_forward({**w, "to_3d.bias": w["to_3d.bias"] + 5.0}, x.cpu().numpy(),
                                 (4, 4, 4), mode="hard")
    bad, _ = compare_paths(ref["route_path"], out2.route_path.cpu().numpy(), ref["level_margins"])
    assert bad == 0


@pytest.mark.parametrize("precision,dtype", [("exact", torch.float32), ("fast", torch.bfloat16)])
def test_six_level_router_4096_experts(cuda_device, precision, dtype):
    """Config-4 tree (4^6 = 4096 experts, 6 levels) against the L-level oracle
    restatement (parity beyond 3 levels is not pinned by the reference)."""
    from sb200 import synth
    H, S, br = 256, 64, (4, 4, 4, 4, 4, 4)
    w = synth.router_weights(H, S, br, seed=9, perturb=True)
    r = make_router(w, H, S, br, cuda_device)
    x = synth.hidden_states(200, H, seed=10, dtype=dtype)
    got = r.route(x.to(cuda_device), select="hard", k=8, precision=precision)
    ref = orouter.router_forward(w, x.float().numpy(), br, mode="hard", k=8)
    assert got["expert_probs"].shape == (200, 4096) and got["route_path"].shape == (200, 6)
    check_against(ref, got, "hard", wtol=1e-5 if precision == "exact" else 2e-2)
