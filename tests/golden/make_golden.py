"""Generate the golden fixtures in tests/golden/ from the REFERENCE's own code.

Run once in a container that has the reference tree (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference /path/to/Spectral-AI

It imports the reference modules ``bvh_router`` (BVHRouter, bvh_router.py:211-329),
``olmoe_extract`` (OLMoELayer.forward_topk, olmoe_extract.py:126-157),
``micro_expert`` (quantize_ternary, micro_expert.py:185-203) and, when built by
``oracle/build_ref.py``, the reference ternary extension's host-side
``pack_ternary`` (ternary_torch_ext.cu:197-231).  The expert SwiGLU golden
follows the reference fallback ``TernaryExpertModule.forward_hidden``
(real_model_demo.py:379-398) operation by operation in torch; that module file
cannot be imported here without the OptiX/ctypes bridges it pulls in.

Weights and inputs come from the seeded recipes in sb200/synth.py; large
arrays (config 0 at H=2048) are regenerated from the recipe at test time and
only checksums plus outputs are stored.
"""

from __future__ import annotations

import argparse
import glob
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO / "spectral-ai_b200"))
from sb200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent


def checksum(a: np.ndarray) -> np.ndarray:
    a = np.asarray(a, np.float64)
    return np.array([a.sum(), (a * a).sum(), a.ravel()[:: max(1, a.size // 4099)].sum()])


def load_ref_router(ref_python: Path):
    sys.path.insert(0, str(ref_python))
    import bvh_router  # the reference module
    return bvh_router


def build_reference_router(bvh_router, H, S, branching, w):
    cfg = bvh_router.RouterConfig(embed_dim=H, spectral_dim=S, n_level1=branching[0],
                                  n_level2=branching[1], n_level3=branching[2])
    r = bvh_router.BVHRouter(cfg)
    sd = {k: torch.from_numpy(np.array(v)) for k, v in w.items()}
    missing, unexpected = r.load_state_dict(sd, strict=True), None
    r.eval()
    return r


def run_reference(bvh_router, router, x: torch.Tensor, mode: str):
    """Reference forward: eval branch (hard) or training branch without Gumbel noise (soft)."""
    if mode == "hard":
        router.eval()
        with torch.no_grad():
            res = router(x)
        router.train(False)
        return res
    saved = bvh_router.F.gumbel_softmax

    def noiseless(logits, tau=1.0, hard=False, **kw):
        return F.softmax(logits / tau, dim=-1)

    bvh_router.F.gumbel_softmax = noiseless
    try:
        router.train()
        with torch.no_grad():
            res = router(x)
    finally:
        bvh_router.F.gumbel_softmax = saved
        router.eval()
    return res


def router_case(bvh_router, name, H, S, branching, seed, perturb, batch, x_seed,
                temperature=1.0, store_full=True):
    w = synth.router_weights(H, S, branching, seed=seed, perturb=perturb, temperature=temperature)
    x = synth.hidden_states(batch, H, seed=x_seed)
    r = build_reference_router(bvh_router, H, S, branching, w)
    out = {"H": H, "S": S, "branching": np.array(branching), "seed": seed,
           "perturb": int(perturb), "batch": batch, "x_seed": x_seed,
           "temperature": temperature}
    with torch.no_grad():
        out["pos"] = r.to_3d(x).numpy()
        out["spec"] = r.spectral(x).numpy()
    for mode in ("hard", "soft"):
        res = run_reference(bvh_router, r, x, mode)
        out[f"{mode}_expert_id"] = res.expert_id.numpy()
        out[f"{mode}_expert_probs"] = res.expert_probs.numpy()
        out[f"{mode}_route_path"] = res.route_path.numpy()
        out[f"{mode}_confidence"] = res.confidence.numpy()
        # MoE consumer convention (olmoe_extract.py:105-118): topk then softmax over the k
        k = min(8, res.expert_probs.shape[1])
        v, i = res.expert_probs.topk(k, dim=-1)
        out[f"{mode}_topk_vals"] = v.numpy()
        out[f"{mode}_topk_ids"] = i.numpy()
        out[f"{mode}_topk_weights"] = F.softmax(v, dim=-1).numpy()
    if store_full:
        for key, val in w.items():
            out["w/" + key] = val
        out["x"] = x.numpy()
    else:
        out["x_checksum"] = checksum(x.numpy())
        for key, val in w.items():
            out["wsum/" + key] = checksum(val)
    np.savez_compressed(OUT / f"{name}.npz", **out)
    print(f"wrote {name}.npz")


def ternary_cases(ref_python: Path):
    sys.path.insert(0, str(ref_python))
    import micro_expert
    import olmoe_extract
    out = {}
    rng = np.random.default_rng(7)
    # per-matrix quantizer (micro_expert.py:185-203) on a latent weight
    wlat = rng.standard_normal((48, 40)).astype(np.float32)
    t, s = micro_expert.quantize_ternary(torch.from_numpy(wlat))
    out["q_latent"] = wlat
    out["q_ternary"] = t.numpy()
    out["q_scale"] = np.float32(s)

    # expert SwiGLU in the order of TernaryExpertModule.forward_hidden (real_model_demo.py:379-398)
    H, I, M = 72, 40, 24          # H, I not multiples of 16 -> ragged packing
    ex = synth.ternary_experts(1, H, I, seed=11)[0]
    ex["gate_scale"] = (ex["gate_scale"] * rng.uniform(0.5, 1.5, I)).astype(np.float32)
    ex["up_scale"] = (ex["up_scale"] * rng.uniform(0.5, 1.5, I)).astype(np.float32)
    ex["down_scale"] = (ex["down_scale"] * rng.uniform(0.5, 1.5, H)).astype(np.float32)
    x = synth.hidden_states(M, H, seed=12)
    with torch.no_grad():
        gate_w = torch.from_numpy(ex["gate_ternary"]).float() * torch.from_numpy(ex["gate_scale"]).unsqueeze(1)
        up_w = torch.from_numpy(ex["up_ternary"]).float() * torch.from_numpy(ex["up_scale"]).unsqueeze(1)
        down_w = torch.from_numpy(ex["down_ternary"]).float() * torch.from_numpy(ex["down_scale"]).unsqueeze(1)
        hidden = F.silu(F.linear(x, gate_w)) * F.linear(x, up_w)
        y = F.linear(hidden, down_w)
    for key in ("gate_ternary", "up_ternary", "down_ternary", "gate_scale", "up_scale", "down_scale"):
        out["e/" + key] = ex[key]
    out["e/x"] = x.numpy()
    out["e/y"] = y.numpy()

    # top-k combine convention (olmoe_extract.py:105-157) with the dequantized experts
    cfg = olmoe_extract.OLMoELayerConfig(hidden_size=H, intermediate_size=I, n_experts=6, top_k=3)
    layer = olmoe_extract.OLMoELayer(cfg)
    experts = synth.ternary_experts(6, H, I, seed=13)
    for e, exe in enumerate(experts):
        m = layer.experts[e]
        m.gate_proj.weight.data = torch.from_numpy(exe["gate_ternary"]).float() * torch.from_numpy(exe["gate_scale"]).unsqueeze(1)
        m.up_proj.weight.data = torch.from_numpy(exe["up_ternary"]).float() * torch.from_numpy(exe["up_scale"]).unsqueeze(1)
        m.down_proj.weight.data = torch.from_numpy(exe["down_ternary"]).float() * torch.from_numpy(exe["down_scale"]).unsqueeze(1)
        for key in ("gate_ternary", "up_ternary", "down_ternary", "gate_scale", "up_scale", "down_scale"):
            out[f"moe/{e}/{key}"] = exe[key]
    g = torch.Generator().manual_seed(14)
    layer.gate.weight.data = torch.randn(6, H, generator=g) / H ** 0.5
    xm = synth.hidden_states(32, H, seed=15)
    with torch.no_grad():
        probs, ids = layer.gate_topk(xm)
        ym = layer.forward_topk(xm, probs, ids)
    out["moe/x"] = xm.numpy()
    out["moe/ids"] = ids.numpy()
    out["moe/probs"] = probs.numpy()
    out["moe/y"] = ym.numpy()

    # reference host packer (ternary_torch_ext.cu:197-231), if oracle/build_ref.py built it
    so = glob.glob(str(REPO / "oracle" / "_ref" / "ternary_expert_ext_ref*.so"))
    if so:
        spec = importlib.util.spec_from_file_location("ternary_expert_ext_ref", so[0])
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        w8 = rng.integers(-1, 2, size=(37, 29), dtype=np.int8)
        out["pack/in"] = w8
        out["pack/out"] = mod.pack_ternary(torch.from_numpy(w8)).numpy()
        print("packed with the reference extension")
    else:
        print("reference extension not built; pack golden skipped")
    np.savez_compressed(OUT / "ternary_small.npz", **out)
    print("wrote ternary_small.npz")


def enhanced_case(ref_python: Path, name, H, seed, batch, x_seed, temperature=1.0, perturb=True,
                  head_gain=1.0):
    """EnhancedBVHRouter eval forward (olmoe_bvh_distill.py:422-625) and the
    BVHGateWrapper top-k conventions (olmoe_e2e_eval.py:226-971) on seeded
    inputs; weights regenerate from sb200.synth.enhanced_router_weights, so
    only their checksums are stored."""
    sys.path.insert(0, str(ref_python))
    import olmoe_bvh_distill
    import olmoe_e2e_eval
    w = synth.enhanced_router_weights(H, seed=seed, perturb=perturb, temperature=temperature)
    # head_gain > 1 spreads the 64 logits (random init leaves them within ~0.1)
    w["expert_head.2.weight"] = (w["expert_head.2.weight"] * head_gain).astype(np.float32)
    r = olmoe_bvh_distill.EnhancedBVHRouter(input_dim=H, feature_dim=128)
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()}, strict=True)
    r.eval()
    x = synth.hidden_states(batch, H, seed=x_seed)
    out = {"H": H, "seed": seed, "batch": batch, "x_seed": x_seed, "temperature": temperature,
           "perturb": int(perturb), "head_gain": head_gain, "x_checksum": checksum(x.numpy())}
    for key, val in w.items():
        out["wsum/" + key] = checksum(val)
    with torch.no_grad():
        probs, ids = r(x)
        out["expert_probs"] = probs.numpy()
        out["expert_ids"] = ids.numpy()
        out["logits"] = r._last_logits.numpy()
        out["geo_dist"] = r._last_geometric_distances.numpy()
        out["branch_bonus"] = r._last_branch_bonus.numpy()
        out["h"] = r.input_proj(x).numpy()
        variants = {"softmax": dict(weight_mode="softmax"),
                    "topk_softmax": dict(weight_mode="topk_softmax"),
                    "softmax_norm": dict(weight_mode="softmax", norm_topk_prob=True)}
        for vname, kw in variants.items():
            for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
                gw = olmoe_e2e_eval.BVHGateWrapper(r, top_k=8, **kw)
                rp, tw, ti = gw(x.to(dt))
                out[f"gate/{vname}/{dt_name}/router_probs"] = rp.float().numpy()
                out[f"gate/{vname}/{dt_name}/topk_weights"] = tw.float().numpy()
                out[f"gate/{vname}/{dt_name}/topk_ids"] = ti.numpy()
    np.savez_compressed(OUT / f"{name}.npz", **out)
    print(f"wrote {name}.npz")


class _GateHost(torch.nn.Module):
    """The module path replace_gate_with_bvh walks (find_gate_module,
    olmoe_e2e_eval.py:1145-1174): model.model.layers[i].mlp.gate, with the
    OLMoE gate attributes top_k and norm_topk_prob."""

    def __init__(self, gate: torch.nn.Linear):
        super().__init__()
        self.model = torch.nn.Module()
        layer = torch.nn.Module()
        layer.mlp = torch.nn.Module()
        layer.mlp.gate = gate
        self.model.layers = torch.nn.ModuleList([layer])


def gate_replacement_case(ref_python: Path, name, H, seed, gate_seed, batch, x_seed, head_gain=20.0):
    """replace_gate_with_bvh (olmoe_e2e_eval.py:1177-1404) run by the reference
    on a checkpoint it loads with torch.load: the hybrid pre-filter
    (:1264-1296) at n_candidates 16 and 48, with and without norm_topk_prob,
    on fp32 and bf16 hidden states; and the pure replacement with an affine
    calibration and an expert permutation stored in the checkpoint
    (:1305-1344)."""
    import tempfile
    sys.path.insert(0, str(ref_python))
    import olmoe_e2e_eval
    w = synth.enhanced_router_weights(H, seed=seed)
    w["expert_head.2.weight"] = (w["expert_head.2.weight"] * head_gain).astype(np.float32)
    wg = synth.dense_gate_weight(64, H, seed=gate_seed)
    x = synth.hidden_states(batch, H, seed=x_seed)
    sd = {k: torch.from_numpy(np.array(v)) for k, v in w.items()}
    cfg = {"input_dim": H, "n_level1": 4, "n_level2": 4, "n_level3": 4, "feature_dim": 128}
    g = torch.Generator().manual_seed(seed + 77)
    cal = {"scale": (torch.rand(64, generator=g) + 0.5), "bias": torch.randn(64, generator=g) * 0.1}
    perm = torch.randperm(64, generator=g)
    out = {"H": H, "seed": seed, "gate_seed": gate_seed, "batch": batch, "x_seed": x_seed,
           "head_gain": head_gain, "x_checksum": checksum(x.numpy()), "wg_checksum": checksum(wg),
           "cal_scale": cal["scale"].numpy(), "cal_bias": cal["bias"].numpy(), "expert_perm": perm.numpy()}
    with tempfile.TemporaryDirectory() as td:
        plain = Path(td) / "router.pt"
        torch.save({"config": cfg, "router_state_dict": sd, "topk_accuracy": 0.0, "top1_accuracy": 0.0}, plain)
        calib = Path(td) / "router_cal.pt"
        torch.save({"config": cfg, "router_state_dict": sd, "calibration_mode": "affine",
                    "calibration_state": cal, "expert_perm": perm.tolist()}, calib)
        for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            for n_cand in (16, 48):
                for norm in (False, True):
                    gate = torch.nn.Linear(H, 64, bias=False)
                    with torch.no_grad():
                        gate.weight.copy_(torch.from_numpy(wg))
                    gate.top_k, gate.norm_topk_prob = 8, norm
                    model = _GateHost(gate.to(dt))
                    olmoe_e2e_eval.replace_gate_with_bvh(model, str(plain), layer_idx=0, hybrid=True,
                                                         n_candidates=n_cand)
                    with torch.no_grad():
                        fp, ts, ti = model.model.layers[0].mlp.gate(x.to(dt).reshape(2, batch // 2, H))
                    pre = f"hybrid/{n_cand}/{int(norm)}/{dt_name}/"
                    out[pre + "router_probs"] = fp.float().numpy()
                    out[pre + "topk_weights"] = ts.float().numpy()
                    out[pre + "topk_ids"] = ti.numpy()
            gate = torch.nn.Linear(H, 64, bias=False)
            gate.top_k, gate.norm_topk_prob = 8, False
            model = _GateHost(gate.to(dt))
            olmoe_e2e_eval.replace_gate_with_bvh(model, str(calib), layer_idx=0, hybrid=False)
            with torch.no_grad():
                rp, tw, ti = model.model.layers[0].mlp.gate(x.to(dt))
            out[f"pure_cal/{dt_name}/router_probs"] = rp.float().numpy()
            out[f"pure_cal/{dt_name}/topk_weights"] = tw.float().numpy()
            out[f"pure_cal/{dt_name}/topk_ids"] = ti.numpy()
    np.savez_compressed(OUT / f"{name}.npz", **out)
    print(f"wrote {name}.npz")


def pipeline_case(ref_python: Path, name, H, seed, batch, x_seed, head_gain=20.0, inner=32):
    """The reference's AsyncPipelineSimulator (python/async_pipeline_bridge.py:49-255)
    on the CPU: an EnhancedBVHRouter, 64 small dense experts and, in the
    calibrated variant, a Linear(64,64) calibration; the route stage's top-k,
    the scatter stage's per-expert token lists and the expert stage's output
    of forward_sequential."""
    sys.path.insert(0, str(ref_python))
    import async_pipeline_bridge as apb
    import olmoe_bvh_distill
    w = synth.enhanced_router_weights(H, seed=seed)
    w["expert_head.2.weight"] = (w["expert_head.2.weight"] * head_gain).astype(np.float32)
    r = olmoe_bvh_distill.EnhancedBVHRouter(input_dim=H, feature_dim=128)
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()}, strict=True)
    r.eval()
    experts = torch.nn.ModuleList()
    for sd in synth.mlp_experts(64, H, inner, seed=seed):
        m = torch.nn.Sequential(torch.nn.Linear(H, inner), torch.nn.GELU(), torch.nn.Linear(inner, H))
        m.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()})
        experts.append(m.eval())
    cal = {k: torch.from_numpy(v) for k, v in synth.calibration_linear(64, seed=seed).items()}
    x = synth.hidden_states(batch, H, seed=x_seed)
    out = {"H": H, "seed": seed, "batch": batch, "x_seed": x_seed, "head_gain": head_gain, "inner": inner,
           "x_checksum": checksum(x.numpy())}
    for variant, cs in (("plain", None), ("cal", cal)):
        cfg = apb.PipelineConfig(num_experts=64, top_k=8, hidden_dim=H, use_cuda_streams=False)
        sim = apb.AsyncPipelineSimulator(cfg, r, experts, calibration_state=cs, device="cpu")
        slot = apb.PipelineSlot()
        with torch.no_grad():
            sim._stage_route(slot, x)
            sim._stage_scatter(slot)
            sim._stage_expert(slot)
            seq = sim.forward_sequential(x)
        assert torch.equal(seq, slot.output)
        out[f"{variant}/expert_ids"] = slot.expert_ids.numpy()
        out[f"{variant}/expert_weights"] = slot.expert_weights.numpy()
        counts = np.zeros(64, np.int32)
        lists = []
        for e in range(64):
            toks = slot.dispatch_indices.get(e, [])
            counts[e] = len(toks)
            lists.extend(toks)
        out[f"{variant}/counts"] = counts
        out[f"{variant}/lists"] = np.asarray(lists, np.int32)
        out[f"{variant}/output"] = slot.output.numpy()
    np.savez_compressed(OUT / f"{name}.npz", **out)
    print(f"wrote {name}.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SB_REFERENCE_ROOT"),
                    help="root of the reference checkout (default: $SB_REFERENCE_ROOT)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("pass --reference or set SB_REFERENCE_ROOT")
    ref_python = Path(a.reference) / "python"
    torch.set_num_threads(8)
    bvh = load_ref_router(ref_python)
    # small: reference test fixture shape (tests/test_bvh_router.py:20-32)
    router_case(bvh, "router_small", 64, 16, (4, 4, 4), seed=42, perturb=True, batch=64, x_seed=42)
    router_case(bvh, "router_small_t05", 64, 16, (4, 4, 4), seed=43, perturb=True, batch=64,
                x_seed=43, temperature=0.5)
    router_case(bvh, "router_small_352", 64, 16, (3, 5, 2), seed=44, perturb=True, batch=48, x_seed=44)
    # config 0: H=2048, S=256, 4x4x4, seed 0, unit-RMS fp32 inputs from seed 0
    router_case(bvh, "router_cfg0", 2048, 256, (4, 4, 4), seed=0, perturb=False, batch=256,
                x_seed=0, store_full=False)
    router_case(bvh, "router_cfg0_perturbed", 2048, 256, (4, 4, 4), seed=5, perturb=True,
                batch=256, x_seed=6, store_full=False)
    ternary_cases(ref_python)
    # EnhancedBVHRouter (the OLMoE production router) and its gate wrapper
    enhanced_case(ref_python, "enhanced_h256", 256, seed=1, batch=96, x_seed=11)
    enhanced_case(ref_python, "enhanced_h256_t05", 256, seed=2, batch=96, x_seed=12, temperature=0.5)
    enhanced_case(ref_python, "enhanced_h256_sharp", 256, seed=3, batch=96, x_seed=13, head_gain=20.0)
    enhanced_case(ref_python, "enhanced_cfg0", 2048, seed=0, batch=256, x_seed=0)
    # replace_gate_with_bvh: hybrid pre-filter and the checkpoint loader
    gate_replacement_case(ref_python, "gate_replace_h256", 256, seed=4, gate_seed=1, batch=96, x_seed=14)
    gate_replacement_case(ref_python, "gate_replace_h2048", 2048, seed=5, gate_seed=2, batch=128, x_seed=15)
    # the tri-core pipeline simulator's stages
    pipeline_case(ref_python, "pipeline_h256", 256, seed=6, batch=96, x_seed=16)


if __name__ == "__main__":
    main()
