"""MoE pipeline stage kernels and the AsyncPipelineSimulator drop-in on the
GPU (needs a B200).

Kernels against the oracle (pinned in test_pipeline_cpu.py): scatter exact
(integer work); softmax / calibration / combine within fp32 rounding (1e-5
relative; expert ids identical up to ties within 1e-5).  The drop-in
simulator against the reference simulator's own outputs
(tests/golden/pipeline_h256.npz).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import pipeline as op
from oracle import ternary as otern
from parity import topk_ids_match
from test_pipeline_cpu import pipeline_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cal", [False, True])
@pytest.mark.parametrize("E,B", [(8, 33), (64, 4096), (100, 129), (256, 7), (1024, 40)])
def test_softmax_topk_kernel(cuda_device, E, B, cal):
    from sb200 import pipeline as pp
    from sb200 import synth
    if cal and E > 128:
        pytest.skip("calibration holds at most 128 experts")
    g = torch.Generator().manual_seed(E * 7 + B)
    logits = torch.randn(B, E, generator=g) * 2.0
    c = synth.calibration_linear(E, seed=E) if cal else None
    k = min(8, E)
    ids, w, p = pp.softmax_topk(logits.to(cuda_device), k, *(torch.from_numpy(c["weight"]).to(cuda_device),
                                                            torch.from_numpy(c["bias"]).to(cuda_device))
                                if cal else (None, None), want_probs=True)
    rp, rids, rw = op.softmax_topk(logits.numpy(), k, c["weight"] if cal else None, c["bias"] if cal else None)
    np.testing.assert_allclose(p.cpu().numpy(), rp, rtol=1e-5, atol=1e-9)
    assert topk_ids_match(rp, rids, ids.cpu().numpy(), 1e-5) == 0
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-5, atol=1e-9)
    # top-k of given probabilities, no softmax; exact ties go to the lower index
    q = torch.tensor([[0.1, 0.3, 0.3, 0.2, 0.1] + [0.0] * (E - 5)] * 3) if E >= 8 else None
    if q is not None:
        qi, qw, _ = pp.softmax_topk(q.to(cuda_device), 4, apply_softmax=False)
        assert qi[0].tolist() == [1, 2, 3, 0]
        assert torch.equal(qw[0].cpu(), torch.tensor([0.3, 0.3, 0.2, 0.1]))


@pytest.mark.parametrize("E", [16, 64, 100])
def test_topk_with_minus_inf_scores(cuda_device, E):
    """Scores of -inf are ranked last and, when fewer than k finite scores are
    left, taken in expert order with weight -inf — the oracle's stable order
    (thread-per-token kernel for E <= 64, warp per token above)."""
    from sb200 import pipeline as pp
    k = 8
    rng = np.random.default_rng(E)
    v = rng.standard_normal((64, E)).astype(np.float32)
    for t in range(64):
        n_inf = (t * 7) % (E + 1)  # 0 .. E scores of -inf per row
        v[t, rng.permutation(E)[:n_inf]] = -np.inf
    v[5, :] = -np.inf
    v[6, 3] = 1.0
    v[6, 9] = 1.0  # an exact tie among the finite scores
    ids, w, _ = pp.softmax_topk(torch.from_numpy(v).to(cuda_device), k, apply_softmax=False)
    rw, rids = op.topk_first_max(v, k)
    assert np.array_equal(ids.cpu().numpy(), rids)
    assert np.array_equal(w.cpu().numpy(), rw)
    # NaN scores rank as -inf: the finite scores first, then the lowest remaining
    # experts with weight -inf; every id valid and distinct
    vn = v.copy()
    vn[7, :] = np.nan
    vn[8, :] = np.nan
    vn[8, [2, 11]] = [0.5, 0.25]
    ids, w, _ = pp.softmax_topk(torch.from_numpy(vn).to(cuda_device), k, apply_softmax=False)
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    assert ids[7].tolist() == list(range(k)) and np.all(w[7] == -np.inf)
    assert ids[8].tolist() == [2, 11] + [e for e in range(E) if e not in (2, 11)][:k - 2]
    assert w[8, :2].tolist() == [0.5, 0.25] and np.all(w[8, 2:] == -np.inf)


def test_apply_calibration_kernel(cuda_device):
    from sb200 import pipeline as pp
    from sb200 import synth
    c = synth.calibration_linear(64, seed=3)
    raw = torch.randn(1000, 64, generator=torch.Generator().manual_seed(3))
    out = pp.apply_calibration(raw.to(cuda_device), torch.from_numpy(c["weight"]).to(cuda_device),
                               torch.from_numpy(c["bias"]).to(cuda_device))
    np.testing.assert_allclose(out.cpu().numpy(), op.apply_calibration(raw.numpy(), c["weight"], c["bias"]),
                               rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("B,k,E,mx", [(1, 1, 1, 1), (96, 8, 64, 96), (5000, 8, 64, 700), (70000, 8, 64, 70000),
                                      (20000, 8, 300, 20000), (40000, 4, 512, 500), (300, 2, 4096, 300),
                                      (0, 8, 64, 10)])
def test_scatter_kernel_exact(cuda_device, B, k, E, mx):
    from sb200 import pipeline as pp
    g = torch.Generator().manual_seed(B + E)
    # skewed ids plus sentinels >= E (skipped)
    ids = (torch.rand(B, k, generator=g) ** 3 * (E + 2)).long().clamp(max=E + 1)
    for store in (False, True):
        disp, counts = pp.scatter_by_expert(ids.to(cuda_device), E, mx, store_entry=store)
        rd, rc = op.scatter_by_expert(ids.numpy(), E, mx, store_entry=store)
        assert np.array_equal(counts.cpu().numpy(), rc)
        d = disp.cpu().numpy()
        for e in range(E):
            n = min(int(rc[e]), mx)
            assert np.array_equal(d[e, :n], rd[e, :n]), e


@pytest.mark.parametrize("B,k,H", [(1, 1, 4), (33, 8, 2048), (17, 3, 257)])
def test_weighted_combine_kernel(cuda_device, B, k, H):
    from sb200 import pipeline as pp
    g = torch.Generator().manual_seed(B * k + H)
    eo, w = torch.randn(B, k, H, generator=g), torch.rand(B, k, generator=g)
    out = pp.weighted_combine(eo.to(cuda_device), w.to(cuda_device))
    np.testing.assert_allclose(out.cpu().numpy(), op.weighted_combine(eo.numpy(), w.numpy()), rtol=1e-5,
                               atol=1e-6)
    # the reference kernel's arithmetic: fused multiply-adds in slot order from 0
    ref = torch.zeros(B, H, dtype=torch.float64)
    for j in range(k):
        ref = ref + w[:, j:j + 1].double() * eo[:, j].double()
    np.testing.assert_allclose(out.cpu().numpy(), ref.numpy(), rtol=1e-5, atol=1e-6)


def _dropin(cuda_device, variant, grouped=False):
    from async_pipeline_bridge import AsyncPipelineSimulator, PipelineConfig
    from olmoe_bvh_distill import EnhancedBVHRouter
    w, experts, cal, x, g = pipeline_case()
    r = EnhancedBVHRouter(input_dim=int(g["H"]))
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()})
    r = r.to(cuda_device).eval()
    r.precision = "exact"
    mods = torch.nn.ModuleList()
    for sd in experts:
        m = torch.nn.Sequential(torch.nn.Linear(int(g["H"]), int(g["inner"])), torch.nn.GELU(),
                                torch.nn.Linear(int(g["inner"]), int(g["H"])))
        m.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()})
        mods.append(m.eval())
    cs = {k: torch.from_numpy(v) for k, v in cal.items()} if variant == "cal" else None
    sim = AsyncPipelineSimulator(PipelineConfig(num_experts=64, top_k=8, hidden_dim=int(g["H"])), r,
                                 mods.to(cuda_device), calibration_state=cs, device=str(cuda_device))
    return sim, torch.from_numpy(x).to(cuda_device), g


@pytest.mark.parametrize("variant", ["plain", "cal"])
def test_dropin_simulator_against_reference(cuda_device, variant):
    from async_pipeline_bridge import PipelineSlot
    sim, x, g = _dropin(cuda_device, variant)
    slot = PipelineSlot()
    sim._stage_route(slot, x)
    ids = slot.expert_ids.cpu().numpy()
    gids = g[f"{variant}/expert_ids"]
    assert ids.dtype == np.int64
    # ids agree up to ties of the gate values (router probabilities to 1e-4)
    same_rows = (ids == gids).all(axis=1)
    assert same_rows.mean() > 0.97
    np.testing.assert_allclose(np.sort(slot.expert_weights.cpu().numpy(), axis=1),
                               np.sort(g[f"{variant}/expert_weights"], axis=1), rtol=1e-4, atol=1e-8)
    sim._stage_scatter(slot)
    d = slot.dispatch_indices.as_dict()
    counts = slot.dispatch_indices.counts.cpu().numpy()
    if same_rows.all():  # scatter is exact on identical ids
        assert np.array_equal(counts, g[f"{variant}/counts"])
        assert np.array_equal(np.concatenate([d.get(e, []) for e in range(64)]).astype(np.int32),
                              g[f"{variant}/lists"])
    sim._stage_expert(slot)
    out = slot.output.cpu().numpy()
    np.testing.assert_allclose(out[same_rows], g[f"{variant}/output"][same_rows], rtol=1e-4, atol=1e-5)


def test_dropin_pipelined_equals_sequential(cuda_device):
    sim, x, g = _dropin(cuda_device, "cal")
    xs = [x[i * 16:(i + 1) * 16].contiguous() for i in range(5)]
    seq = [sim.forward_sequential(t) for t in xs]
    outs = [sim.forward_pipelined(t) for t in xs]
    assert outs[0] is None and outs[1] is None
    for i in range(2, 5):
        torch.testing.assert_close(outs[i], seq[i - 2], rtol=0, atol=0)
    rest = sim.flush()
    assert len(rest) == 2
    torch.testing.assert_close(rest[0], seq[3], rtol=0, atol=0)
    torch.testing.assert_close(rest[1], seq[4], rtol=0, atol=0)


def test_dropin_grouped_ternary_experts(cuda_device):
    """Ternary expert modules run as one grouped SwiGLU, weighted by the route."""
    from dataclasses import dataclass
    import ternary_expert_ext_bridge as bridge
    from async_pipeline_bridge import AsyncPipelineSimulator, PipelineConfig
    from olmoe_bvh_distill import EnhancedBVHRouter
    from sb200 import synth
    H, I = 256, 128

    @dataclass
    class FakeExpert:
        expert_id: int
        gate_ternary: np.ndarray
        up_ternary: np.ndarray
        down_ternary: np.ndarray
        gate_scale: np.ndarray
        up_scale: np.ndarray
        down_scale: np.ndarray

    ex = synth.ternary_experts(64, H, I, seed=6)
    mods = torch.nn.ModuleList(bridge.create_expert_module(
        FakeExpert(e, d["gate_ternary"], d["up_ternary"], d["down_ternary"], d["gate_scale"], d["up_scale"],
                   d["down_scale"])) for e, d in enumerate(ex)).to(cuda_device)
    r = EnhancedBVHRouter(input_dim=H)
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in synth.enhanced_router_weights(H, seed=6).items()})
    r = r.to(cuda_device).eval()
    sim = AsyncPipelineSimulator(PipelineConfig(num_experts=64, top_k=8, hidden_dim=H), r, mods,
                                 device=str(cuda_device))
    assert sim._grouped is not None
    x = synth.hidden_states(200, H, seed=61).to(cuda_device)
    from async_pipeline_bridge import PipelineSlot
    slot = PipelineSlot()
    sim._stage_route(slot, x)
    sim._stage_scatter(slot)
    sim._stage_expert(slot)
    ref = otern.moe_combine(x.cpu().numpy(), slot.expert_ids.cpu().numpy(), slot.expert_weights.cpu().numpy(), ex)
    err = np.abs(slot.output.cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err < 5e-3, err
