"""Benchmark of the B200 hot path; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload router|moe_layer] [--batch B]

Workloads (seeded synthetic inputs with BASELINE.json's shapes; no datasets):
  moe_layer  (default, the headline) one OLMoE-shaped MoE layer: BVH router
             (hidden 2048, spectral 256, 4x4x4 = 64 experts, top-8, soft
             level selection so the top-8 is not degenerate) followed by the
             grouped ternary SwiGLU (64 experts, 2048 -> 1024 -> 2048, 2-bit
             weights) over 4096 bf16 tokens per GPU (config 2).  L2 is flushed
             (256 MiB write) before every timed step; each step is timed with
             its own CUDA event pair and the flush stays outside them.
  ep         (N > 1) the same layer expert-parallel: 64/N experts per GPU,
             NCCL all-to-all dispatch of bf16 token rows and combine of fp32
             expert outputs.  Reported inside the line as "ep".
  stack16    (config 3) 16 MoE layers with residual, 16384 tokens in total
             split over the GPUs; reported as "stack16".
  config4    6-level router (4096 experts, hidden 4096) at 8192 tokens per GPU
             against a dense bf16 gate (cuBLAS GEMM + top-8); "config4".
  enhanced   EnhancedBVHRouter (the OLMoE production router) + BVHGateWrapper
             softmax top-8 at 65,536 bf16 tokens per GPU; "enhanced_router".
  router     BVH router forward alone at B = 262144 bf16 tokens (config 1);
             1 GiB of input per GPU > L2, so no flush.  Reported inside the
             moe_layer line as "router".

One process per GPU (torchrun for N > 1).  The headline shards tokens with no
collective: every rank routes its own 4096 tokens and runs them through its
own copy of the 64 experts (100 MB of 2-bit weights, replicated; weak
scaling).  Timing: W
warm-up steps, then exactly K timed steps on the launching stream, bracketed
by barrier + synchronize, max over ranks.

--impl reference times the reference's CPU path on the host cores: the
restated oracle (oracle/: numpy ports of python/bvh_router.py and of the
TernaryExpertModule fp32 fallback, python/real_model_demo.py:360-403) on a
bounded token sample per step, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "spectral-ai_b200"))
sys.path.insert(0, str(REPO))

H, S, BRANCHING, TOPK = 2048, 256, (4, 4, 4), 8
E_EXPERTS, I_INTER = 64, 1024
ROUTER_FLOP_PER_TOKEN = 2 * (H * H + H * S + 3 * H + S * 84)   # 9,492,480 (hard mode evaluates 3 refraction rows)
ROUTER_BYTES_PER_TOKEN = 2 * H + TOPK * 8                       # bf16 in + ids/weights out


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def mark(self, begin: bool):
        if begin:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        rows = [r.split(",") for r in out.strip().splitlines() if r.strip()]
        sm, mx, reasons = [], [], set()
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        # samples under load: the upper half of observed clocks are the timed region
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup(n_gpus: int):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    import torch.distributed as dist
    if world > 1:
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    import torch
    import torch.distributed as dist
    if world == 1:
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU baselines: the reference's CPU path (its torch operators, restated in
# oracle/torch_ref.py) on the host cores
# ---------------------------------------------------------------------------
def blas_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:
        return os.cpu_count() or 1


def cpu_threads():
    """All host threads for the CPU baselines (torch's intra-op pool)."""
    import torch
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_router_rate(sample_tokens: int, budget_s: float = 12.0):
    """Tokens/s of the reference router's CPU path (BVHRouter.forward eval, fp32,
    the reference's torch operators as restated in oracle/torch_ref.py)."""
    import torch
    from oracle import torch_ref
    from sb200 import synth
    cpu_threads()
    r = torch_ref.TorchRouter(synth.router_weights(H, S, BRANCHING, seed=0), BRANCHING)
    x = synth.hidden_states(sample_tokens, H, seed=1)
    with torch.no_grad():
        r.topk(x, TOPK, soft=False)   # warm the thread pool
        done, t0 = 0, time.perf_counter()
        while True:
            r.topk(x, TOPK, soft=False)
            done += sample_tokens
            el = time.perf_counter() - t0
            if el >= budget_s or done >= 8 * sample_tokens:
                break
    return done / el, done, el


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
def router_workload(batch: int, device):
    import numpy as np
    import torch
    from bvh_router import BVHRouter, RouterConfig
    from sb200 import synth
    w = synth.router_weights(H, S, BRANCHING, seed=0)
    r = BVHRouter(RouterConfig(embed_dim=H, spectral_dim=S))
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()})
    r = r.to(device).eval()
    x = synth.hidden_states(batch, H, seed=1, dtype=torch.bfloat16, device=device)
    eng = r.sync_weights(device)
    outs = {"topk_ids": torch.empty(batch, TOPK, dtype=torch.int32, device=device),
            "topk_weights": torch.empty(batch, TOPK, dtype=torch.float32, device=device)}

    def step():
        eng.forward(x, precision="fast", select="hard", k=TOPK, outputs=outs)

    x_host = x.cpu().pin_memory()
    ids_host = torch.empty(batch, TOPK, dtype=torch.int32).pin_memory()
    w_host = torch.empty(batch, TOPK, dtype=torch.float32).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step():
        # public API: BVHRouter.forward_topk on a host batch copied in, results copied out
        x_dev.copy_(x_host, non_blocking=True)
        ids, wts = r.forward_topk(x_dev, k=TOPK)
        ids_host.copy_(ids, non_blocking=True)
        w_host.copy_(wts, non_blocking=True)

    meta = {"tokens_per_step": batch,
            "h2d": batch * H * 2, "d2h": batch * TOPK * 8,
            "dominant": "router_enc1_gelu_tc", "dominant_flop": 2.0 * batch * H * (H + 3),
            "dominant_bytes": batch * H * 2 * 2 + H * H * 2,
            "config": {"workload": "router_fwd_bvh_4x4x4_top8", "hidden": H, "spectral_dim": S,
                       "experts": 64, "top_k": TOPK, "batch_tokens_per_gpu": batch,
                       "select": "hard", "precision": "bf16 tcgen05 encoder, fp32 descent",
                       "l2": "inputs 1 GiB per GPU > 126 MB L2 (no flush)"}}
    return step, e2e_step, meta


def moe_workload(batch: int, device, select: str = "soft"):
    import numpy as np
    import torch
    from bvh_router import BVHRouter, RouterConfig
    from sb200 import synth
    from sb200.moe import BVHMoELayer
    from sb200.ternary import TernaryExperts
    w = synth.router_weights(H, S, BRANCHING, seed=0)
    r = BVHRouter(RouterConfig(embed_dim=H, spectral_dim=S))
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()})
    r = r.to(device).eval()
    experts = TernaryExperts(synth.ternary_experts(E_EXPERTS, H, I_INTER, seed=2), device)
    layer = BVHMoELayer(r, experts, top_k=TOPK, select=select)
    x = synth.hidden_states(batch, H, seed=2, dtype=torch.bfloat16, device=device)
    out = torch.empty(batch, H, dtype=torch.bfloat16, device=device)
    ids, _ = layer.route(x)
    counts = torch.bincount(ids.long().flatten(), minlength=E_EXPERTS).float()

    def eager_step():
        layer.forward(x, out=out)

    # the timed form: the whole layer (router + dispatch + grouped GEMMs +
    # combine, eight kernels) replayed from one CUDA graph per buffer pair
    from sb200.moe import GraphedLayer
    glayer = GraphedLayer(layer)
    glayer(x, out)

    def step():
        glayer(x, out)

    # end to end: host batches through sb200.moe.HostPipeline (copies in and out
    # on their own streams, overlapped with the neighbouring batches' compute)
    from sb200.moe import HostPipeline
    pipe = HostPipeline(glayer, batch, H, dtype=torch.bfloat16, device=device)
    x_host = [x.cpu().pin_memory() for _ in range(2)]
    out_host = [torch.empty(batch, H, dtype=torch.bfloat16).pin_memory() for _ in range(2)]

    def e2e_run(n):
        pipe.run([x_host[i & 1] for i in range(n)], [out_host[i & 1] for i in range(n)])

    x_dev = torch.empty_like(x)

    def e2e_sequential():
        # one batch at a time on one stream: copy in, layer, copy out
        x_dev.copy_(x_host[0], non_blocking=True)
        y = layer(x_dev)
        out_host[0].copy_(y, non_blocking=True)

    e2e_step = (e2e_run, e2e_sequential, eager_step)

    pairs = batch * TOPK
    meta = {"tokens_per_step": batch, "h2d": batch * H * 2, "d2h": batch * H * 2,
            "dominant": "ternary_gateup_tc", "dominant_flop": 2.0 * pairs * H * 2 * I_INTER,
            "config": {"workload": "moe_layer_bvh_route_ternary_swiglu", "hidden": H,
                       "intermediate": I_INTER, "experts": E_EXPERTS, "top_k": TOPK,
                       "tokens_per_gpu": batch, "router_select": select,
                       "expert_load_max_over_mean": round(float(counts.max() / counts.mean()), 3),
                       "experts_with_tokens": int((counts > 0).sum()),
                       "precision": "router bf16 tcgen05 + fp32 descent; ternary bf16 x {-1,0,1} "
                                    "tcgen05, fp16 hidden, fp32 accumulate; bf16 out",
                       "l2": "flushed (256 MiB write) before every timed step, outside the events"}}
    return step, e2e_step, meta


def enhanced_workload(batch: int, device, hybrid: bool = False):
    """EnhancedBVHRouter (the OLMoE production router, python/olmoe_bvh_distill.py:422-632)
    + BVHGateWrapper softmax top-8 (python/olmoe_e2e_eval.py:928-938) on bf16 tokens;
    ``hybrid``: the hybrid pre-filter gate instead (BVH top-48 candidates, the
    layer's dense 64-expert gate, olmoe_e2e_eval.py:1264-1296)."""
    import torch
    from sb200 import synth
    from sb200.enhanced import EnhancedEngine
    w = synth.enhanced_router_weights(H, seed=0)
    eng = EnhancedEngine(H, 128, BRANCHING, device)
    eng.upload(w)
    if hybrid:
        eng.set_dense_gate(torch.from_numpy(synth.dense_gate_weight(64, H, seed=0)).to(torch.bfloat16))
    x = synth.hidden_states(batch, H, seed=1, dtype=torch.bfloat16, device=device)
    outs = {"router_probs": torch.empty(batch, 64, dtype=torch.float32, device=device),
            "topk_weights": torch.empty(batch, TOPK, dtype=torch.float32, device=device),
            "topk_ids": torch.empty(batch, TOPK, dtype=torch.int32, device=device)}

    def step():
        if hybrid:
            eng.forward(x, precision="fast", want=(), gate="hybrid", k=TOPK, n_candidates=48, outputs=outs)
        else:
            eng.forward(x, precision="fast", want=(), gate="softmax", k=TOPK, outputs=outs)

    # 2 (H*512 + 512*256) + tail (levels + head) MAC per token, times 2 FLOP
    flop = 2.0 * (H * 512 + 512 * 256 + 256 * 131 + 256 * 128 + 128 * 128 + 2 * (128 * 131 + 2 * 128 * 128)
                  + 140 * 256 + 256 * 64)
    return step, flop


def pipeline_stage_rates(dev, pk, world, steps, warmup):
    """The stage kernels of the MoE pipeline (cuda/async_pipeline.cu:79-230)
    at OLMoE shape, each timed alone with inputs larger than L2:
    calibrated softmax + top-8 and the scatter over 1,048,576 tokens x 64
    experts, the weighted combine of 8 fp32 expert outputs of width 2048 for
    16,384 tokens.  Algorithmic bytes: logits in + ids/weights out; ids in +
    counts and lists out; outputs + weights in, combined rows out."""
    import torch
    from sb200 import pipeline as pp
    from sb200 import synth
    Bt, E, k = 1 << 20, 64, TOPK
    g = torch.Generator(device=dev).manual_seed(9)
    logits = torch.randn(Bt, E, generator=g, device=dev) * 2.0
    c = synth.calibration_linear(E, seed=9)
    cw, cb = torch.from_numpy(c["weight"]).to(dev), torch.from_numpy(c["bias"]).to(dev)
    ids = torch.empty(Bt, k, dtype=torch.int32, device=dev)
    wts = torch.empty(Bt, k, dtype=torch.float32, device=dev)
    lib = pp._lib.load()

    def topk_step():
        pp._lib.check(lib.sb_softmax_topk(pp._ptr(logits), Bt, E, k, pp._ptr(cw), pp._ptr(cb), 1, None,
                                          pp._ptr(ids), pp._ptr(wts), pp._stream(dev)), "sb_softmax_topk")

    disp = torch.empty(E, Bt, dtype=torch.int32, device=dev)
    counts = torch.empty(E, dtype=torch.int32, device=dev)

    def scatter_step():
        pp._lib.check(lib.sb_scatter_by_expert(pp._ptr(ids), Bt, k, E, Bt, 0, pp._ptr(disp), pp._ptr(counts),
                                               pp._stream(dev)), "sb_scatter_by_expert")

    Bc, Hc = 16384, H
    eo = torch.randn(Bc, k, Hc, generator=g, device=dev)
    cwt = torch.rand(Bc, k, generator=g, device=dev)
    cout = torch.empty(Bc, Hc, device=dev)

    def combine_step():
        pp._lib.check(lib.sb_weighted_combine(pp._ptr(eo), pp._ptr(cwt), Bc, Hc, k, pp._ptr(cout),
                                              pp._stream(dev)), "sb_weighted_combine")

    res = {}
    for name, step, nbytes in (("cal_softmax_topk", topk_step, Bt * (E * 4 + k * 8)),
                               ("scatter_by_expert", scatter_step, Bt * k * 4 * 2 + E * 4),
                               ("weighted_combine", combine_step, Bc * (k * Hc * 4 + k * 4 + Hc * 4))):
        ms, _ = time_steps(step, steps, warmup, world)
        gbs = nbytes / (ms / steps / 1e3) / 1e9
        res[name] = {"avg_ms": round(ms / steps, 4), "algorithmic_bytes": nbytes, "gbs": round(gbs, 1),
                     "hbm_frac": round(gbs / pk["hbm_gbs"], 4)}
    res["shapes"] = (f"softmax/scatter: {Bt} tokens x {E} experts, top-{k}, calibration 64x64; "
                     f"combine: {Bc} tokens x {k} x {Hc} fp32")
    return res


def legacy_tree_rates(dev, pk, world, steps, warmup):
    """The legacy ray-sphere tree router (cuda/v5/bvh_router_kernel.cu): the
    device kernel over 1,048,576 rays (outputs: expert, 64 scores, path,
    confidence; 300 algorithmic bytes per ray), and the reference's ctypes
    entry point bvh_route_batch at 1024 rays with CUDA-graph replay, host
    buffers in and out (the call the reference times at ~3 us + copies)."""
    import ctypes as C
    import time as _t
    import numpy as np
    import torch
    from sb200 import _lib, synth
    import bvh_router_ext as ext
    tree = synth.legacy_tree(0)
    ext.upload_tree(*[torch.from_numpy(np.ascontiguousarray(tree[k], np.float32))
                      for k in ("centers", "radii", "portals", "snell_w", "snell_b")])
    B = 1 << 20
    o, d = synth.rays(B, 1)
    to, td = torch.from_numpy(o).to(dev), torch.from_numpy(d).to(dev)
    spec = torch.empty(B, 64, device=dev)
    lib = _lib.load()
    h = ext._tree(dev.index if dev.index is not None else 0)
    ex = torch.empty(B, dtype=torch.int32, device=dev)
    sc = torch.empty(B, 64, device=dev)
    pa = torch.empty(B, 3, dtype=torch.int32, device=dev)
    cf = torch.empty(B, device=dev)
    P = lambda t: C.c_void_p(t.data_ptr())

    def step():
        _lib.check(lib.sb_tree_route(h, P(to), P(td), B, P(ex), P(sc), P(pa), P(cf),
                                     C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)), "sb_tree_route")

    ms, _ = time_steps(step, steps, warmup, world)
    per = ms / steps
    nbytes = B * 300
    res = {"rays": B, "kernel_ms": round(per, 4), "rays_per_s": round(B / (per / 1e3), 1),
           "gbs": round(nbytes / (per / 1e3) / 1e9, 1), "hbm_frac": round(nbytes / (per / 1e3) / 1e9 / pk["hbm_gbs"], 4)}
    # the ctypes API, host buffers, graph replay
    arrs = [np.ascontiguousarray(tree[k], np.float32) for k in ("centers", "radii", "portals", "snell_w", "snell_b")]
    Pn = lambda a: a.ctypes.data_as(C.c_void_p)
    assert lib.bvh_upload_tree(*[Pn(a) for a in arrs]) == 0 and lib.bvh_alloc_buffers(1024) == 0
    ho, hd = np.ascontiguousarray(o[:1024]), np.ascontiguousarray(d[:1024])
    hs = np.zeros((1024, 64), np.float32)
    he, hsc = np.zeros(1024, np.int32), np.zeros((1024, 64), np.float32)
    hp, hc = np.zeros((1024, 3), np.int32), np.zeros(1024, np.float32)
    args = [Pn(ho), Pn(hd), Pn(hs), Pn(he), Pn(hsc), Pn(hp), Pn(hc), 1024]
    for g in (1, 0):
        for _ in range(20):
            assert lib.bvh_route_batch(*args, g) == 0
        n = 500
        t0 = _t.perf_counter()
        for _ in range(n):
            lib.bvh_route_batch(*args, g)
        res["ctypes_us_per_call_graph" if g else "ctypes_us_per_call_nograph"] = round(
            (_t.perf_counter() - t0) / n * 1e6, 2)
    lib.bvh_free_buffers()
    res["ctypes_what"] = ("bvh_route_batch, 1024 rays, host buffers in/out (12 KB in, 300 KB out), "
                          "host clock per synchronous call, 500 calls")
    return res


def optix_route_rates(dev, world, steps, warmup):
    """The OptiX router's route / route_topk served by CUDA (optix_training_ext
    drop-in): 65,536 queries against 64 expert octahedra, one ray and the
    8-ray fan, queries/s."""
    import numpy as np
    import torch
    import optix_training_ext as ext
    g = np.random.default_rng(0)
    centers = torch.from_numpy((g.standard_normal((64, 3)) * 3.0).astype(np.float32))
    radii = torch.from_numpy((0.4 + 0.6 * g.random(64)).astype(np.float32))
    B = 65536
    pos = torch.from_numpy((g.standard_normal((B, 3)) * 2.0).astype(np.float32)).to(dev)
    d = g.standard_normal((B, 3))
    dirs = torch.from_numpy((d / np.linalg.norm(d, axis=1, keepdims=True)).astype(np.float32)).to(dev)
    ext.initialize("", "")
    ext.build_gas(centers, radii, use_triangles=True)
    res = {"queries": B, "experts": 64, "geometry": "octahedra (use_triangles=True)"}
    for name, fn in (("route", lambda: ext.route_async(pos, dirs)),
                     ("route_topk8", lambda: ext._route(pos, dirs, 8, False))):
        ms, _ = time_steps(fn, steps, warmup, world)
        res[name] = {"ms": round(ms / steps, 4), "queries_per_s": round(B / (ms / steps / 1e3), 1)}
    ext.shutdown()
    return res


def cpu_enhanced_rate(sample_tokens: int, budget_s: float = 8.0):
    """Oracle port of the enhanced router + gate on the host cores (tokens/s)."""
    from oracle import enhanced as oe
    from sb200 import synth
    w = synth.enhanced_router_weights(H, seed=0)
    x = synth.hidden_states(sample_tokens, H, seed=1).numpy()
    for _ in range(2):
        oe.gate_topk(oe.router_forward(w, x)[2], TOPK)
    done, t0 = 0, time.perf_counter()
    while True:
        oe.gate_topk(oe.router_forward(w, x)[2], TOPK)
        done += sample_tokens
        el = time.perf_counter() - t0
        if el >= budget_s or done >= 16 * sample_tokens:
            break
    return done / el, done, el


def config4_workloads(batch: int, device):
    """Config 4: 6-level router (4^6 = 4096 experts) at hidden 4096 vs a dense
    linear gate of the same shape (bf16 4096x4096 GEMM + top-8 + softmax)."""
    import numpy as np
    import torch
    from bvh_router import BVHRouter, RouterConfig
    from sb200 import synth
    H4, br = 4096, (4,) * 6
    w = synth.router_weights(H4, S, br, seed=4)
    r = BVHRouter(RouterConfig(embed_dim=H4, spectral_dim=S, branching=br))
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()})
    r = r.to(device).eval()
    eng = r.sync_weights(device)
    x = synth.hidden_states(batch, H4, seed=4, dtype=torch.bfloat16, device=device)
    outs = {"topk_ids": torch.empty(batch, TOPK, dtype=torch.int32, device=device),
            "topk_weights": torch.empty(batch, TOPK, dtype=torch.float32, device=device)}
    g = torch.Generator(device=device).manual_seed(44)
    wg = (torch.randn(4096, H4, generator=g, device=device) / H4 ** 0.5).to(torch.bfloat16)

    def router_step():
        eng.forward(x, precision="fast", select="hard", k=TOPK, outputs=outs)

    def dense_step():
        logits = x @ wg.t()
        v, i = torch.topk(logits.float(), TOPK, dim=-1)
        torch.softmax(v, dim=-1)

    return router_step, dense_step


def stack_workload(tokens: int, device, layers: int = 16, select: str = "soft", world: int = 1):
    """Config 3: a stack of MoE layers (router + 64 ternary experts each, own
    random weights per layer) with residual h <- h + MoE(h); attention omitted.
    At N > 1 every layer is expert-parallel (64/N experts per GPU, the
    peer-memory exchange, an expert placement per layer from its router's
    routing of a calibration batch), the layers sharing one workspace."""
    import numpy as np
    import torch
    from bvh_router import BVHRouter, RouterConfig
    from sb200 import synth
    from sb200.moe import BVHMoELayer
    from sb200.ternary import TernaryExperts
    stack = []
    rank = 0
    if world > 1:
        import torch.distributed as dist
        from sb200.ep import EPMoELayer
        rank = dist.get_rank()
    shared = None
    for l in range(layers):
        w = synth.router_weights(H, S, BRANCHING, seed=100 + l)
        r = BVHRouter(RouterConfig(embed_dim=H, spectral_dim=S))
        r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()})
        r = r.to(device).eval()
        if world > 1:
            el = E_EXPERTS // world
            # this layer's placement from its router on a calibration batch
            xc = synth.hidden_states(tokens, H, seed=9 + 1000 * rank, dtype=torch.bfloat16, device=device)
            placement, _ = ep_placement(r, xc, world, select, iters=1000)
            # the experts at this rank's positions (random weights either way)
            local = TernaryExperts.random(el, H, I_INTER, seed=200 + 64 * l + rank, device=device)
            layer = EPMoELayer(r, local, E_EXPERTS, TOPK, tokens, select=select, chunks=1, workspace=shared,
                               placement=placement)
            shared = layer.ep.workspace
            stack.append(layer)
        else:
            stack.append(BVHMoELayer(r, TernaryExperts.random(E_EXPERTS, H, I_INTER, seed=200 + l, device=device),
                                     top_k=TOPK, select=select))
    x = synth.hidden_states(tokens, H, seed=3, dtype=torch.bfloat16, device=device)

    def step():
        h = x
        for layer in stack:
            h = h + layer(h)
        return h

    return step


def ep_placement(router, xc, world: int, select: str, iters: int = 3000):
    """The expert placement of an expert-parallel layer from a calibration
    batch (other tokens than the timed ones): every rank routes its own
    batch, the ids are gathered so that every rank sees the same statistics,
    units of sibling experts are balanced over the ranks (sb200.ep.
    balanced_placement) and swaps then lower the modelled step time (sb200.ep.
    refine_placement, the same seeded search on every rank).  SB_EP_PLACEMENT=
    contiguous | grouped | scattered selects a simpler form for comparison."""
    import torch
    import torch.distributed as dist
    from sb200.ep import balanced_placement, refine_placement
    mode = os.environ.get("SB_EP_PLACEMENT", "refined")
    if mode == "contiguous":
        return None, mode
    ids_c, _ = router.forward_topk(xc, k=TOPK, select=select)
    ids_c = ids_c.to(torch.int32).contiguous()
    allc = torch.empty(world * ids_c.shape[0], ids_c.shape[1], dtype=ids_c.dtype, device=ids_c.device)
    dist.all_gather_into_tensor(allc, ids_c)
    allc = allc.cpu().numpy()
    import numpy as np
    loads = np.bincount(allc.ravel(), minlength=E_EXPERTS).astype(float)
    el = E_EXPERTS // world
    group = 1 if mode == "scattered" else (BRANCHING[-1] if el % BRANCHING[-1] == 0 else 1)
    perm = balanced_placement(loads.tolist(), world, group=group)
    if mode == "refined":
        perm = refine_placement(perm, allc, world, iters=iters)
    return perm, mode


def ep_workload(batch: int, device, world: int, select: str = "soft"):
    """The headline layer expert-parallel (N > 1): the same router on every
    rank, 64/N experts per GPU, the tokens exchanged by the layer's own kernels
    through peer memory (sb200.ep.ExpertParallelMoE); replayed from one CUDA
    graph like the single-GPU layer.  Returns (step, e2e pieces, meta) as
    moe_workload does."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from bvh_router import BVHRouter, RouterConfig
    from sb200 import synth
    from sb200.ep import EPMoELayer
    from sb200.moe import GraphedLayer, HostPipeline
    from sb200.ternary import TernaryExperts
    rank = dist.get_rank()
    w = synth.router_weights(H, S, BRANCHING, seed=0)
    r = BVHRouter(RouterConfig(embed_dim=H, spectral_dim=S))
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()})
    r = r.to(device).eval()
    e_local = E_EXPERTS // world
    allx = synth.ternary_experts(E_EXPERTS, H, I_INTER, seed=2)
    # expert placement from routing statistics of a calibration batch
    from sb200.ep import experts_at
    xc = synth.hidden_states(batch, H, seed=7 + 1000 * rank, dtype=torch.bfloat16, device=device)
    placement, mode = ep_placement(r, xc, world, select)
    held = experts_at(placement, rank, world) if placement else list(range(rank * e_local, (rank + 1) * e_local))
    local = TernaryExperts([allx[e] for e in held], device)
    chunks = int(os.environ.get("SB_EP_CHUNKS", "2"))
    layer = EPMoELayer(r, local, E_EXPERTS, TOPK, batch, select=select, chunks=chunks, placement=placement)
    x = synth.hidden_states(batch, H, seed=2 + 1000 * rank, dtype=torch.bfloat16, device=device)
    out = torch.empty(batch, H, dtype=torch.bfloat16, device=device)
    ids, _ = layer.route(x)
    counts = torch.bincount(ids.long().flatten(), minlength=E_EXPERTS).float()
    dist.all_reduce(counts)                      # the whole job's expert loads
    perm_t = torch.tensor(placement if placement else list(range(E_EXPERTS)), device=device)
    owner = perm_t // e_local                    # each expert's rank
    per_rank = torch.zeros(world, device=device).index_add_(0, owner, counts)
    contiguous = counts.view(world, e_local).sum(dim=1)
    dests = torch.zeros(batch, world, dtype=torch.bool, device=device)
    dests.scatter_(1, owner[ids.long()], True)
    rows_sent = float(dests.sum()) / max(batch, 1)

    def eager_step():
        layer(x, out=out)

    glayer = GraphedLayer(layer)
    glayer(x, out)

    def step():
        glayer(x, out)

    pipe = HostPipeline(glayer, batch, H, dtype=torch.bfloat16, device=device)
    x_host = [x.cpu().pin_memory() for _ in range(2)]
    out_host = [torch.empty(batch, H, dtype=torch.bfloat16).pin_memory() for _ in range(2)]

    def e2e_run(n):
        pipe.run([x_host[i & 1] for i in range(n)], [out_host[i & 1] for i in range(n)])

    x_dev = torch.empty_like(x)

    def e2e_sequential():
        x_dev.copy_(x_host[0], non_blocking=True)
        y = layer(x_dev)
        out_host[0].copy_(y, non_blocking=True)

    mine = float(per_rank[rank])   # (token, expert) entries this rank's experts process
    meta = {"tokens_per_step": batch, "h2d": batch * H * 2, "d2h": batch * H * 2,
            "dominant": "ternary_gateup_tc", "dominant_flop": 2.0 * mine * H * 2 * I_INTER,
            "layer": layer,
            "config": {"workload": "moe_layer_bvh_route_ternary_swiglu", "hidden": H,
                       "intermediate": I_INTER, "experts": E_EXPERTS, "top_k": TOPK,
                       "tokens_per_gpu": batch, "router_select": select,
                       "experts_per_gpu": e_local,
                       "entries_per_gpu_max_over_mean": round(float(per_rank.max() / per_rank.mean()), 3),
                       "expert_placement": {"refined": "balanced units of sibling experts, then swaps that "
                                                       "lower the modelled step time (sb200.ep.balanced_placement "
                                                       "+ refine_placement), from a calibration batch's routing",
                                            "grouped": "balanced units of sibling experts (sb200.ep."
                                                       "balanced_placement), from a calibration batch's routing",
                                            "scattered": "balanced single experts (sb200.ep.balanced_placement)",
                                            "contiguous": "contiguous blocks"}.get(mode, mode),
                       "entries_per_gpu_max_over_mean_contiguous": round(
                           float(contiguous.max() / contiguous.mean()), 3),
                       "expert_load_max_over_mean": round(float(counts.max() / counts.mean()), 3),
                       "rows_sent_per_token": round(rows_sent, 3),
                       "precision": "router bf16 tcgen05 + fp32 descent; ternary bf16 x {-1,0,1} "
                                    "tcgen05, fp16 hidden, fp32 accumulate; fp32 partial sums; bf16 out",
                       "l2": "flushed (256 MiB write) before every timed step, outside the events"},
            "parallelism": (f"ep{world}: {e_local} experts per GPU; each token row sent once per GPU "
                            "holding one of its experts and one fp32 partial sum returned, by the "
                            "layer's own kernels through peer memory (no host sync, no library collective); "
                            f"{chunks} token ranges on their own streams so transfers overlap the GEMMs")}
    return step, (e2e_run, e2e_sequential, eager_step), meta


def nccl_alltoall_rate(batch: int, device, world: int, steps: int, warmup: int, flush):
    """The baseline of the fused exchange: the same sharded layer over the library
    collective (sb200.ep.AllToAllMoE: torch.distributed.all_to_all_single on
    NCCL, host-synchronised split sizes, one row per slot each way)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from bvh_router import BVHRouter, RouterConfig
    from sb200 import synth
    from sb200.ep import AllToAllMoE
    from sb200.ternary import TernaryExperts
    rank = dist.get_rank()
    w = synth.router_weights(H, S, BRANCHING, seed=0)
    r = BVHRouter(RouterConfig(embed_dim=H, spectral_dim=S))
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()})
    r = r.to(device).eval()
    e_local = E_EXPERTS // world
    allx = synth.ternary_experts(E_EXPERTS, H, I_INTER, seed=2)
    local = TernaryExperts(allx[rank * e_local:(rank + 1) * e_local], device)
    layer = AllToAllMoE(lambda rows, ids, ww: local.forward(rows, ids, ww, out_dtype=torch.float32), E_EXPERTS)
    x = synth.hidden_states(batch, H, seed=2 + 1000 * rank, dtype=torch.bfloat16, device=device)

    def step():
        ids, wts = r.forward_topk(x, k=TOPK, select="soft")
        layer(x, ids, wts, out_dtype=torch.bfloat16)

    ms, _ = time_steps(step, steps, warmup, world, flush=flush)
    return {"value": round(batch * world * steps / (ms / 1e3), 1), "unit": "tokens/s",
            "ms_per_step": round(ms / steps, 4),
            "what": "sb200.ep.AllToAllMoE: all_to_all_single (NCCL) of counts, bf16 rows (one per slot), "
                    "ids, weights; fp32 outputs back; host-read split sizes; eager launches"}


def router_sweep(dev, pk, world, steps, warmup, flush, cpu: bool):
    """Config 1: the router (hard top-8, bf16 FAST engine) at B = 1, 256, 4096
    and 65536 tokens (262,144 is the "router" line).  Inputs below 126 MB sit
    in L2, so L2 is flushed before every step (outside the events).  With
    ``cpu`` the reference's CPU router (oracle/torch_ref.py) is timed at the
    same batch sizes on every host core."""
    import torch
    out = {}
    for B in (1, 256, 4096, 65536):
        step, _, meta = router_workload(B, dev)
        n = steps if B <= 4096 else max(10, steps // 4)
        ms, prof = time_steps(step, n, warmup, world, flush=flush if B <= 4096 else None, profile=True)
        per = ms / n
        row = {"batch": B, "us_per_batch": round(per * 1e3, 2),
               "mq_per_s": round(B * world / (per / 1e3) / 1e6, 4),
               "tensor_frac": round(B * ROUTER_FLOP_PER_TOKEN / (per / 1e3) / 1e12 / pk["bf16_tflops"], 4),
               "hbm_frac": round(B * ROUTER_BYTES_PER_TOKEN / (per / 1e3) / 1e9 / pk["hbm_gbs"], 4),
               "kernels": {k: round(t / max(c, 1), 4) for k, (c, t) in prof.items()},
               "l2": "flushed before every step" if B <= 4096 else "inputs > L2 (268 MB), no flush"}
        if cpu:
            from oracle import torch_ref
            from sb200 import synth
            cores = cpu_threads()
            r = torch_ref.TorchRouter(synth.router_weights(H, S, BRANCHING, seed=0), BRANCHING)
            x = synth.hidden_states(B, H, seed=1)
            with torch.no_grad():
                r.topk(x, TOPK, soft=False)
                reps = max(1, min(50, int(4096 // B)))
                t0 = time.perf_counter()
                for _ in range(reps):
                    r.topk(x, TOPK, soft=False)
                el = (time.perf_counter() - t0) / reps
            row["cpu_reference"] = {"us_per_batch": round(el * 1e6, 1), "mq_per_s": round(B / el / 1e6, 6),
                                    "cores": cores, "kind": "port",
                                    "what": "BVHRouter.forward (eval, fp32), the reference's torch operators "
                                            "(oracle/torch_ref.py)"}
        out[str(B)] = row
        del step
    return out


def small_batch_rates(dev, pk, world, steps, warmup, flush):
    """Small batches, where the expert weights set the cost: the drop-in
    ternary_gated_mlp (one OLMoE-shaped expert, fp32 input as the reference API
    takes it) at M = 1, 64, 256 tokens, and the whole MoE layer (router + 64
    ternary experts) at B = 1, 64, 256 tokens.  hbm_frac counts the 2-bit
    weights of the experts a step touches plus its activations, against the
    step's device time."""
    import numpy as np
    import torch
    import ternary_expert_ext as tx
    from sb200 import synth
    res = {"gated_mlp": {}, "moe_layer": {}}
    ex = synth.ternary_experts(1, H, I_INTER, seed=21)[0]
    packs = [tx.pack_ternary(torch.from_numpy(np.ascontiguousarray(ex[k].T))).to(dev)
             for k in ("gate_ternary", "up_ternary", "down_ternary")]
    scales = [torch.from_numpy(ex[k]).to(dev) for k in ("gate_scale", "up_scale", "down_scale")]
    wbytes = 3 * H * I_INTER // 4
    for M in (1, 64, 256):
        x = synth.hidden_states(M, H, seed=22, device=dev)
        fn = lambda: tx.ternary_gated_mlp(x, *packs, *scales)
        ms, _ = time_steps(fn, steps, warmup, world, flush=flush)
        per = ms / steps / 1e3
        nbytes = wbytes + M * H * 4 * 2
        res["gated_mlp"][str(M)] = {"us": round(per * 1e6, 2), "tokens_per_s": round(M / per, 1),
                                    "gbs": round(nbytes / per / 1e9, 1),
                                    "hbm_frac": round(nbytes / per / 1e9 / pk["hbm_gbs"], 4)}
    for B in (1, 64, 256):
        step, _, meta = moe_workload(B, dev)
        ms, prof = time_steps(step, steps, warmup, world, flush=flush)
        per = ms / steps / 1e3
        used = meta["config"]["experts_with_tokens"]
        nbytes = used * wbytes + B * H * 2 * 2
        res["moe_layer"][str(B)] = {"us": round(per * 1e6, 2), "tokens_per_s": round(B * world / per, 1),
                                    "experts_touched": used, "gbs": round(nbytes / per / 1e9, 1),
                                    "hbm_frac": round(nbytes / per / 1e9 / pk["hbm_gbs"], 4)}
    res["l2"] = "flushed before every step (outside the events)"
    return res


def reference_gpu_rates(dev, steps, warmup, flush):
    """Baseline leg: the reference's own CUDA kernels, compiled from its sources
    into oracle/_ref by oracle/build_ref.py, timed on this GPU beside ours on the
    same inputs (rank 0, 1 GPU; absent when oracle/_ref was not built):
    ternary_gated_mlp (cuda/v5/ternary_torch_ext.cu:123-191, one token per CTA)
    at M = 1, 64, 256, and the legacy tree router's bvh_route_batch
    (cuda/v5/bvh_router_kernel.cu:558-687, host buffers in and out) at 256 and
    1024 rays.  The tree kernel computes other math than BVHRouter, so it is
    timed against our implementation of the same tree router, not against the
    BVH router."""
    import ctypes as C
    import glob
    import importlib.util
    import numpy as np
    import torch
    from sb200 import _lib, synth
    out = {}
    so = glob.glob(str(REPO / "oracle" / "_ref" / "ternary_expert_ext_ref*.so"))
    if so:
        spec = importlib.util.spec_from_file_location("ternary_expert_ext_ref", so[0])
        ref = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(ref)
        import ternary_expert_ext as tx
        ex = synth.ternary_experts(1, H, I_INTER, seed=21)[0]
        packs = [ref.pack_ternary(torch.from_numpy(np.ascontiguousarray(ex[k].T))).to(dev)
                 for k in ("gate_ternary", "up_ternary", "down_ternary")]
        scales = [torch.from_numpy(ex[k]).to(dev) for k in ("gate_scale", "up_scale", "down_scale")]
        rows = {}
        for M in (1, 64, 256):
            x = synth.hidden_states(M, H, seed=22, device=dev)
            r_ms, _ = time_steps(lambda: ref.ternary_gated_mlp(x, *packs, *scales), steps, warmup, 1, flush=flush)
            o_ms, _ = time_steps(lambda: tx.ternary_gated_mlp(x, *packs, *scales), steps, warmup, 1, flush=flush)
            rows[str(M)] = {"reference_us": round(r_ms / steps * 1e3, 2), "ours_us": round(o_ms / steps * 1e3, 2),
                            "speedup": round(r_ms / o_ms, 2)}
        out["ternary_gated_mlp"] = {"shape": f"{H} -> {I_INTER} -> {H}, fp32 input, one expert", **rows}
    lib_path = REPO / "oracle" / "_ref" / "libbvh_router_ref.so"
    if lib_path.is_file():
        P = lambda a: a.ctypes.data_as(C.c_void_p)
        tree = synth.legacy_tree(0)
        arrs = [np.ascontiguousarray(tree[k], np.float32) for k in ("centers", "radii", "portals", "snell_w", "snell_b")]
        rows = {}
        for name, lib in (("reference", C.CDLL(str(lib_path))), ("ours", _lib.load())):
            assert lib.bvh_upload_tree(*[P(a) for a in arrs]) == 0
            for B in (256, 1024):
                assert lib.bvh_alloc_buffers(B) == 0
                o, d = synth.rays(B, 1)
                spec = np.zeros((B, 64), np.float32)
                he, hsc = np.zeros(B, np.int32), np.zeros((B, 64), np.float32)
                hp, hc = np.zeros((B, 3), np.int32), np.zeros(B, np.float32)
                args = [P(o), P(d), P(spec), P(he), P(hsc), P(hp), P(hc), B, 1]
                for _ in range(20):
                    assert lib.bvh_route_batch(*args) == 0
                t0 = time.perf_counter()
                for _ in range(300):
                    lib.bvh_route_batch(*args)
                rows.setdefault(str(B), {})[f"{name}_us"] = round((time.perf_counter() - t0) / 300 * 1e6, 2)
            lib.bvh_free_buffers()
        out["bvh_route_batch"] = {"what": "host buffers in and out, CUDA-graph replay, synchronous call, "
                                          "host clock over 300 calls", **rows}
    return out


def time_steps(step, steps, warmup, world, sampler=None, profile=False, flush=None):
    import torch
    from sb200 import _lib
    for _ in range(warmup):
        if flush is not None:
            flush()
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    if profile:
        _lib.profile_enable(True)
    s = torch.cuda.current_stream()
    if sampler:
        sampler.mark(True)
    if flush is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(steps):
            step()
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
    else:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        for a, b in ev:
            flush()
            a.record(s)
            step()
            b.record(s)
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in ev)
    if sampler:
        sampler.mark(False)
    barrier(world)
    prof = _lib.profile_read() if profile else {}
    if profile:
        _lib.profile_enable(False)
    return max_over_ranks(ms, world), prof


def time_pipelined(run, steps, warmup, world):
    """Device time of one pipelined run of `steps` batches (CUDA events on the
    current stream, which the pipeline makes wait for its last copy out), after
    `warmup` batches; max over ranks."""
    import torch
    s = torch.cuda.current_stream()
    run(max(warmup, 1))
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    run(steps)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    barrier(world)
    return max_over_ranks(ms, world)


def roofline_tensor(meta, prof, pk, steps_ms, steps):
    dom = prof.get(meta["dominant"], (0, 0.0))
    if not dom[0]:
        return None
    # dominant_flop is per step; a chunked layer launches the kernel several
    # times a step, each on a share of the step's rows
    flop_launch = meta["dominant_flop"] * steps / dom[0]
    avg_s = dom[1] / dom[0] / 1e3
    achieved = flop_launch / avg_s / 1e12
    out = {"kernel": meta["dominant"], "bound": "tensor", "achieved": round(achieved, 1),
           "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": round(achieved / pk["bf16_tflops"], 4),
           "peak_source": f"{pk['source']} bf16 burst (cuBLAS)",
           "traffic": scale_traffic(traffic_for(meta), steps / dom[0]), "avg_launch_ms": round(dom[1] / dom[0], 4),
           "launches_per_step": round(dom[0] / steps, 2), "algorithmic_flop_per_launch": flop_launch}
    if dom[0] > steps:
        out["note"] = ("launches of different token ranges run on their own streams and may overlap; "
                       "each launch's events include the time it shared the GPU")
    return out


def run_ours(a):
    import torch
    rank, world, local = dist_setup(a.gpus)
    dev = torch.device("cuda", torch.cuda.current_device())
    pk = peaks()
    sampler = ClockSampler(local)
    sampler.start()
    # ---- headline: the MoE layer
    batch = a.batch or 4096
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush = lambda: flush_buf.fill_(1)
    use_ep = world > 1 and not a.skip_ep
    if use_ep:
        step, e2e_step, meta = ep_workload(batch, dev, world)
        parallelism = meta["parallelism"]
        api = ("sb200.moe.HostPipeline.run over sb200.ep.EPMoELayer (BVHRouter.forward_topk + "
               "ExpertParallelMoE)")
    else:
        step, e2e_step, meta = moe_workload(batch, dev)
        parallelism = "single GPU, all 64 experts"
        api = "sb200.moe.HostPipeline.run over sb200.moe.BVHMoELayer (BVHRouter.forward_topk + TernaryExperts)"
    total_ms, _ = time_steps(step, a.steps, a.warmup, world, sampler, flush=flush)
    clocks = sampler.stop()
    # the same layer launched kernel by kernel with per-kernel CUDA events: the
    # kernel breakdown and the roofline of the dominant kernel
    prof_steps = min(a.steps, 100)
    eager_ms, prof = time_steps(e2e_step[2], prof_steps, a.warmup, world, profile=True, flush=flush)
    e2e_ms = time_pipelined(e2e_step[0], a.steps, a.warmup, world)
    seq_ms, _ = time_steps(e2e_step[1], a.steps, a.warmup, world, flush=flush)
    tokens = meta["tokens_per_step"] * a.steps * world
    value = tokens / (total_ms / 1e3)
    e2e_value = tokens / (e2e_ms / 1e3)
    launches = sum(n for n, _ in prof.values()) // prof_steps * a.steps  # kernels per step x timed steps
    out = {"metric": "MoE-layer tokens/s (BVH route + ternary SwiGLU)",
           "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": round(total_ms / a.steps, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (seeded unit-RMS Gaussian tokens, random-init router and ternary experts)",
           "config": dict(meta["config"], parallelism=parallelism),
           "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                   "h2d_bytes_per_step": meta["h2d"], "d2h_bytes_per_step": meta["d2h"],
                   "api": api + ": pinned host batches, copies in/out on their own streams "
                          "overlapped with the neighbouring batches' compute",
                   "l2": "no flush between batches; each batch streams > 400 MB through the layer "
                         "(dispatch rows 134 MB, per-slot outputs 277 MB) against a 126 MB L2",
                   "sequential_value": round(tokens / (seq_ms / 1e3), 1),
                   "sequential": "the layer's __call__ one batch at a time on one stream (copy in, "
                                 "layer, copy out; L2 flushed between batches)"},
           "gpu_launches": launches,
           "launch_mode": (f"timed steps replay one CUDA graph of the layer ({launches // a.steps} kernels "
                           f"per step); kernel breakdown from {prof_steps} eager steps with per-kernel "
                           f"events ({round(eager_ms / prof_steps, 4)} ms/step eager)"),
           "kernels": {k: {"launches": n, "avg_ms": round(t / max(n, 1), 4),
                           "share": round(t / max(sum(v[1] for v in prof.values()), 1e-9), 4)}
                       for k, (n, t) in prof.items()},
           "roofline": roofline_tensor(meta, prof, pk, eager_ms, prof_steps), "clocks": clocks}
    # ---- N > 1: the replicated form (every GPU all 64 experts, its own tokens,
    #      no exchange) and the library-collective form of the sharded layer
    if use_ep:
        rstep, _, rmeta = moe_workload(batch, dev)
        r_ms, _ = time_steps(rstep, a.steps, a.warmup, world, flush=flush)
        out["replicated"] = {"metric": "MoE-layer tokens/s, experts replicated", "unit": "tokens/s",
                             "value": round(tokens / (r_ms / 1e3), 1), "ms_per_step": round(r_ms / a.steps, 4),
                             "parallelism": f"token-shard x{world}: all 64 experts (100 MB of 2-bit weights) "
                                            "on every GPU, no exchange"}
        del rstep
        out["nccl_all_to_all"] = nccl_alltoall_rate(batch, dev, world, min(a.steps, 20), a.warmup, flush)
    # ---- config 3: 16-layer MoE stack, 16384 tokens sharded over the ranks
    if not a.skip_stack:
        stok = max(1, 16384 // world)
        sstep = stack_workload(stok, dev, world=world)
        st_steps = min(a.steps, 10)
        s_ms, sprof = time_steps(sstep, st_steps, 2, world, profile=True)
        out["stack16"] = {"metric": "16-layer MoE stack tokens/s (config 3)", "unit": "tokens/s",
                          "value": round(stok * world * st_steps / (s_ms / 1e3), 1),
                          "ms_per_step": round(s_ms / st_steps, 3), "tokens_total": stok * world,
                          "tokens_per_gpu": stok, "layers": 16, "steps": st_steps,
                          "scaling": "strong (16384 tokens in total, split over the GPUs)",
                          "parallelism": (f"ep{world} per layer ({E_EXPERTS // world} experts per GPU, "
                                          "peer-memory exchange, expert placement per layer)" if world > 1 else "single GPU"),
                          "l2": "weights of 16 layers (1.7 GB) stream every step; no flush"}
    # ---- config 4: 6-level 4096-expert router at hidden 4096 vs a dense gate
    if not a.skip_config4:
        c4tok = 65536 // 8
        rstep4, dstep4 = config4_workloads(c4tok, dev)
        c4_steps = min(a.steps, 50)
        r4_ms, r4prof = time_steps(rstep4, c4_steps, a.warmup, world, profile=True, flush=flush)
        d4_ms, _ = time_steps(dstep4, c4_steps, a.warmup, world, flush=flush)
        out["config4"] = {"metric": "tokens/s, 6-level BVH router (4096 experts, hidden 4096) vs dense gate",
                          "unit": "tokens/s", "tokens_per_gpu": c4tok,
                          "bvh_router": round(c4tok * world * c4_steps / (r4_ms / 1e3), 1),
                          "dense_gate_cublas": round(c4tok * world * c4_steps / (d4_ms / 1e3), 1),
                          "bvh_ms_per_step": round(r4_ms / c4_steps, 4), "dense_ms_per_step": round(d4_ms / c4_steps, 4),
                          "bvh_kernels": {k: {"launches": n, "avg_ms": round(t / max(n, 1), 4)}
                                          for k, (n, t) in r4prof.items()},
                          "dense_gate": "torch bf16 x @ W^T (cuBLAS, 4096 x 4096) + topk(8) + softmax",
                          "l2": "flushed before every step"}
    # ---- enhanced router (the OLMoE production router) + softmax top-8 gate
    if not a.skip_enhanced:
        etok = 65536
        estep, eflop = enhanced_workload(etok, dev)
        e_steps = min(a.steps, 50)
        e_ms, eprof = time_steps(estep, e_steps, a.warmup, world, profile=True, flush=flush)
        dom = eprof.get("enh_proj0_gelu_tc", (0, 0.0))
        out["enhanced_router"] = {
            "metric": "EnhancedBVHRouter + BVHGateWrapper top-8, Mq/s", "unit": "Mq/s",
            "value": round(etok * world * e_steps / (e_ms / 1e3) / 1e6, 3), "tokens_per_gpu": etok,
            "ms_per_step": round(e_ms / e_steps, 4), "flop_per_token": eflop,
            "tensor_frac_of_step": round(etok * eflop / (e_ms / e_steps / 1e3) / 1e12 / pk["bf16_tflops"], 4),
            "kernels": {k: {"launches": n, "avg_ms": round(t / max(n, 1), 4)} for k, (n, t) in eprof.items()},
            "proj0_tflops": round(etok * 2.0 * H * 512 / (dom[1] / max(dom[0], 1) / 1e3) / 1e12, 1) if dom[0] else None,
            "precision": "bf16 tcgen05 input projection, fp32 levels/head/gate",
            "l2": "flushed before every step"}
        hstep, _ = enhanced_workload(etok, dev, hybrid=True)
        h_ms, hprof = time_steps(hstep, e_steps, a.warmup, world, profile=True, flush=flush)
        out["enhanced_router"]["hybrid_gate"] = {
            "what": "hybrid pre-filter: BVH top-48 candidates + dense 64-expert gate (bf16 GEMM) softmax, top-8",
            "value": round(etok * world * e_steps / (h_ms / 1e3) / 1e6, 3), "unit": "Mq/s",
            "ms_per_step": round(h_ms / e_steps, 4),
            "kernels": {k: {"launches": n, "avg_ms": round(t / max(n, 1), 4)} for k, (n, t) in hprof.items()}}
        if rank == 0 and world == 1 and not a.no_cpu_baseline:
            rate, done, el = cpu_enhanced_rate(2048)
            out["enhanced_router"]["cpu_baseline"] = {
                "value": round(rate / 1e6, 6), "unit": "Mq/s", "cores": blas_threads(), "kind": "port",
                "sample": f"{done} tokens through the numpy port of EnhancedBVHRouter + the gate (fp32) "
                          f"in {el:.1f} s"}
    # ---- the pipeline's stage kernels around the expert GEMMs (HBM-bound)
    if not a.skip_enhanced:
        out["pipeline_stages"] = pipeline_stage_rates(dev, pk, world, min(a.steps, 50), a.warmup)
        out["legacy_tree"] = legacy_tree_rates(dev, pk, world, min(a.steps, 50), a.warmup)
        out["optix_route"] = optix_route_rates(dev, world, min(a.steps, 50), a.warmup)
    # ---- router alone (config 1), same process
    if not a.skip_router:
        rstep, _, rmeta = router_workload(a.router_batch, dev)
        rsampler = ClockSampler(local)
        rsampler.start()
        r_ms, rprof = time_steps(rstep, a.router_steps, a.warmup, world, profile=True)
        rclocks = rsampler.stop()
        # the same-shape plain GEMM through cuBLAS (no bias, GELU or position
        # tail), timed the same way right after: the like-for-like yardstick
        # for encoder GEMM 1 under the clocks this loop runs at
        gx = torch.randn(a.router_batch, H, device=dev).to(torch.bfloat16)
        gw = (torch.randn(H, H, device=dev) / H ** 0.5).to(torch.bfloat16)
        gout = torch.empty(a.router_batch, H, device=dev, dtype=torch.bfloat16)
        c_ms, _ = time_steps(lambda: torch.mm(gx, gw.t(), out=gout), a.router_steps, a.warmup, world)
        del gx, gw, gout
        rtok = rmeta["tokens_per_step"] * a.router_steps * world
        out["router"] = {"metric": "router Mq/s", "value": round(rtok / (r_ms / 1e3) / 1e6, 3),
                         "unit": "Mq/s", "batch_per_gpu": a.router_batch,
                         "ms_per_step": round(r_ms / a.router_steps, 4),
                         "hbm_frac": round(rmeta["tokens_per_step"] * ROUTER_BYTES_PER_TOKEN /
                                           (r_ms / a.router_steps / 1e3) / 1e9 / pk["hbm_gbs"], 4),
                         "tensor_frac_of_step": round(rmeta["tokens_per_step"] * ROUTER_FLOP_PER_TOKEN /
                                                      (r_ms / a.router_steps / 1e3) / 1e12 /
                                                      pk["bf16_tflops"], 4),
                         "kernels": {k: {"launches": n, "avg_ms": round(t / max(n, 1), 4)}
                                     for k, (n, t) in rprof.items()},
                         "roofline": roofline_tensor(rmeta, rprof, pk, r_ms, a.router_steps),
                         "clocks": rclocks,
                         "cublas_same_gemm": {
                             "what": f"torch.mm bf16 [{a.router_batch},{H}] x [{H},{H}]^T (cuBLAS), "
                                     "same loop length",
                             "avg_ms": round(c_ms / a.router_steps, 4),
                             "tflops": round(2.0 * a.router_batch * H * H / (c_ms / a.router_steps / 1e3) / 1e12, 1)}}
        if rank == 0 and world == 1 and not a.no_cpu_baseline:
            rate, done, el = cpu_router_rate(4096)
            out["router"]["cpu_baseline"] = {
                "value": round(rate / 1e6, 6), "unit": "Mq/s", "cores": cpu_threads(), "kind": "port",
                "sample": f"{done} tokens through BVHRouter.forward (eval, fp32) as the reference's torch "
                          f"operators (oracle/torch_ref.py) in {el:.1f} s"}
    # ---- config-1 sweep and the small-batch regime
    if not a.skip_sweeps:
        sw_steps = min(a.steps, 100)
        out["router_sweep"] = router_sweep(dev, pk, world, sw_steps, a.warmup, flush,
                                           cpu=(rank == 0 and world == 1 and not a.no_cpu_baseline))
        out["small_batch"] = small_batch_rates(dev, pk, world, sw_steps, a.warmup, flush)
        if rank == 0 and world == 1 and not a.no_cpu_baseline:
            out["reference_gpu"] = reference_gpu_rates(dev, sw_steps, a.warmup, flush)
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        rate, done, el = cpu_moe_rate(batch)
        out["cpu_baseline"] = {"value": round(rate, 2), "unit": "tokens/s", "cores": cpu_threads(),
                               "kind": "port",
                               "sample": f"{done} tokens of the same workload ({batch}-token batches: "
                                         f"BVHRouter soft top-8 + OLMoELayer.forward_topk over 64 "
                                         f"TernaryExpertModule experts, fp32, the reference's torch "
                                         f"operators as restated in oracle/torch_ref.py) in {el:.1f} s"}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def cpu_moe_layer(tokens: int):
    """The reference's CPU MoE layer (oracle/torch_ref.py: BVHRouter soft top-8 +
    OLMoELayer.forward_topk over TernaryExpertModule experts) and its input: the
    headline's tokens (seed 2, rounded to bf16 as the GPU arm reads them) in fp32."""
    import torch
    from oracle import torch_ref
    from sb200 import synth
    layer = torch_ref.TorchMoELayer(synth.router_weights(H, S, BRANCHING, seed=0),
                                    synth.ternary_experts(E_EXPERTS, H, I_INTER, seed=2), BRANCHING, TOPK)
    x = synth.hidden_states(tokens, H, seed=2, dtype=torch.bfloat16).float()
    return layer, x


def cpu_moe_rate(tokens: int, budget_s: float = 20.0):
    """Tokens/s of the reference's CPU layer on the host cores: whole batches of
    the headline's token count until the budget is spent (at least one)."""
    cpu_threads()
    layer, x = cpu_moe_layer(tokens)
    layer(x[:64])   # warm the thread pool
    done, t0 = 0, time.perf_counter()
    while True:
        layer(x)
        done += tokens
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return done / el, done, el


# committed ncu summary that holds the DRAM traffic of each dominant kernel
TRAFFIC_PROFILES = {
    "router_enc1_gelu_tc": "router_enc1_gelu_tc.json",
    "ternary_gateup_tc": "ternary_pair_gateup_moe4096.json",
}


def scale_traffic(t, f):
    return None if t is None else int(t * f)


def traffic_for(meta):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary:
    bytes per token (measured on a smaller case, traffic grows with the tokens) or
    bytes per launch of this very workload (scaled by tokens when they differ)."""
    name = TRAFFIC_PROFILES.get(meta["dominant"])
    p = REPO / "profiles" / name if name else None
    if p is None or not p.exists():
        return None
    d = json.loads(p.read_text())
    if "dram_bytes_per_token" in d:
        return int(d["dram_bytes_per_token"] * meta["tokens_per_step"])
    return int(d["dram_bytes_per_launch"] * meta["tokens_per_step"] / d["tokens"])


def run_reference(a):
    """The reference arm: the reference's CPU path (its torch operators, restated
    op for op in oracle/torch_ref.py and checked there against the reference's
    own outputs) over the headline's 4096 tokens per step, on every host core.
    Rank 0 only; a step that would not let W + K steps end within about four
    minutes is cut to a smaller token sample (reported in the config)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = cpu_threads()
    tokens = a.batch or 4096
    layer, x = cpu_moe_layer(tokens)
    t0 = time.perf_counter()
    layer(x[:256])
    per_tok = (time.perf_counter() - t0) / 256
    budget = 240.0 / max(a.steps + a.warmup, 1)
    sample = int(max(64, min(tokens, budget / max(per_tok, 1e-9))))
    xs = x[:sample]
    for _ in range(a.warmup):
        layer(xs)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        layer(xs)
    el = time.perf_counter() - t0
    value = sample * a.steps / el
    out = {"impl": "reference", "metric": "MoE-layer tokens/s (BVH route + ternary SwiGLU)",
           "value": round(value, 2), "unit": "tokens/s", "n_gpus": 0, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": round(el / a.steps * 1e3, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic (seeded unit-RMS Gaussian tokens, random-init router and ternary experts)",
           "config": {"workload": "moe_layer_bvh_route_ternary_swiglu", "hidden": H,
                      "intermediate": I_INTER, "experts": E_EXPERTS, "top_k": TOPK,
                      "tokens_per_step": sample, "tokens_per_gpu": tokens, "router_select": "soft",
                      "parallelism": "host cores"},
           "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": cores, "kind": "port",
                            "sample": f"{sample} tokens per step: BVHRouter soft top-8 + OLMoELayer.forward_topk "
                                      "over 64 TernaryExpertModule experts, the reference's torch operators in "
                                      "its order (oracle/torch_ref.py; equal outputs to the reference modules), "
                                      f"fp32, torch.set_num_threads({cores})"},
           "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=0, help="MoE-layer tokens per GPU (default 4096)")
    ap.add_argument("--router-batch", type=int, default=262144)
    ap.add_argument("--router-steps", type=int, default=100)
    ap.add_argument("--skip-router", action="store_true")
    ap.add_argument("--skip-ep", action="store_true")
    ap.add_argument("--skip-stack", action="store_true")
    ap.add_argument("--skip-config4", action="store_true")
    ap.add_argument("--skip-enhanced", action="store_true")
    ap.add_argument("--skip-sweeps", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3) if a.impl == "ours" else a.warmup
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
