"""Expert-parallel dispatch/combine host logic on 2 CPU ranks (gloo), no GPU.

The experts are a CPU stand-in (the oracle's fp32 SwiGLU, test infrastructure
only); what is under test is the all-to-all plan: every (token, slot) pair
reaches the rank that owns its expert, comes back to its slot, and the slots
are summed in order.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_q, case):
    sys.path.insert(0, str(REPO / "spectral-ai_b200"))
    sys.path.insert(0, str(REPO))
    import torch.distributed as dist
    from oracle import ternary as otern
    from sb200 import synth
    from sb200.ep import ExpertParallelMoE
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        E, H, I, B, k = case
        experts = synth.ternary_experts(E, H, I, seed=31)
        e_local = E // world
        mine = experts[rank * e_local:(rank + 1) * e_local]

        def expert_fn(rows, local_ids, w):
            rows = rows.float().numpy()
            out = np.zeros_like(rows)
            for i in range(rows.shape[0]):
                ex = mine[int(local_ids[i, 0])]
                out[i] = float(w[i, 0]) * otern.gated_mlp_f32(rows[i:i + 1], ex["gate_ternary"], ex["up_ternary"],
                                                              ex["down_ternary"], ex["gate_scale"],
                                                              ex["up_scale"], ex["down_scale"])[0]
            return torch.from_numpy(out)

        x = synth.hidden_states(B, H, seed=40 + rank)          # each rank routes its own tokens
        ids_np, w_np = synth.zipf_routing(B, E, k, seed=50 + rank)
        layer = ExpertParallelMoE(expert_fn, E)
        y = layer(x, torch.from_numpy(ids_np), torch.from_numpy(w_np), out_dtype=torch.float32)
        ref = otern.moe_combine(x.numpy(), ids_np, w_np, experts)
        assert tuple(y.shape) == (B, H)
        out_q.put((rank, float(np.abs(y.numpy() - ref).max(initial=0.0)), float(np.abs(ref).max(initial=0.0))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [(8, 32, 48, 13, 3), (4, 16, 16, 1, 2), (6, 24, 32, 0, 2)])
def test_ep_two_ranks_matches_single_process(case):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, case)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    res = [q.get(timeout=5) for _ in range(world)]
    for rank, err, scale in res:
        assert err <= 1e-4 * max(scale, 1e-3), (rank, err, scale)
