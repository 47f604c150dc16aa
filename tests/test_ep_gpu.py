"""Expert parallelism over 2 B200s (NCCL): sharded output == single-GPU output, bit for bit.

Skipped unless the box has at least 2 GPUs.  Each rank runs as a spawned
child process with its own GPU; both ranks take the same collective steps.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    sys.path.insert(0, str(REPO / "spectral-ai_b200"))
    sys.path.insert(0, str(REPO))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime
    import torch.distributed as dist
    from sb200 import synth
    from sb200.ep import ExpertParallelMoE
    from sb200.ternary import TernaryExperts
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        E, H, I, B, k = 16, 512, 256, 700 + 37 * rank, 4
        experts = synth.ternary_experts(E, H, I, seed=61)
        e_local = E // world
        local = TernaryExperts(experts[rank * e_local:(rank + 1) * e_local], dev)
        full = TernaryExperts(experts, dev)
        x = synth.hidden_states(B, H, seed=70 + rank, dtype=torch.bfloat16, device=dev)
        ids_np, w_np = synth.zipf_routing(B, E, k, seed=80 + rank)
        ids = torch.from_numpy(ids_np).to(dev)
        w = torch.from_numpy(w_np).to(dev)
        layer = ExpertParallelMoE(lambda r, i, ww: local.forward(r, i, ww, out_dtype=torch.float32), E)
        y_ep = layer(x, ids, w, out_dtype=torch.float32)
        y_one = full.forward(x, ids, w, out_dtype=torch.float32)
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(y_ep, y_one)), float((y_ep - y_one).abs().max())))
    finally:
        dist.destroy_process_group()


def test_ep_two_gpus_bitwise():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    res = sorted(q.get(timeout=5) for _ in range(world))
    for rank, equal, err in res:
        assert equal, f"rank {rank}: max |diff| {err}"
