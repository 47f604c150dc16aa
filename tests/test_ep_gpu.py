"""The expert-parallel layer on B200s (csrc/ep.cu through the C ABI).

* One GPU (world 1): the layer's dispatch, planning, grouped GEMMs, return and
  combine on one rank equal the single-GPU layer (sb_ternary_moe_swiglu) bit
  for bit, for empty, one-token and full batches, several forwards in a row.
* A wait that runs out: a bounded wait on a flag no rank writes is reported by
  sb_ep_status and the device status word, and the GPU keeps working.
* All GPUs of the box, 2, 4 or 8 (skipped on a 1-GPU box): every rank's output
  equals the single-GPU layer over all experts (run on all ranks' tokens at
  once, so that every expert sees the same rows) bit for bit, over several
  forwards and with both set-up paths (handles exchanged by torch.distributed,
  or by the library over an NCCL communicator, the latter with an expert
  placement); then rank 0 runs a forward the others skip, and its waits report
  the timeout instead of hanging.
* An expert placement on one rank: the layer equals the single-GPU layer over
  the experts in position order fed ids perm[ids].
"""

from __future__ import annotations

import ctypes as C
import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def _layers(E, H, I, k, cap, dev, seed=61, timeout_ms=2000):
    from sb200 import synth
    from sb200.ep import ExpertParallelMoE
    from sb200.ternary import TernaryExperts
    experts = synth.ternary_experts(E, H, I, seed=seed)
    full = TernaryExperts(experts, dev)
    ep = ExpertParallelMoE(TernaryExperts(experts, dev), E, k, cap, timeout_ms=timeout_ms)
    return full, ep


@pytest.mark.parametrize("E,H,I,k", [(64, 2048, 1024, 8), (16, 512, 256, 4), (8, 256, 128, 8)])
def test_single_rank_equals_single_gpu_layer(cuda_device, E, H, I, k):
    from sb200 import synth
    full, ep = _layers(E, H, I, k, 4096, cuda_device)
    try:
        for call, B in enumerate([700, 0, 1, 4096, 333]):
            x = synth.hidden_states(B, H, seed=90 + call, dtype=torch.bfloat16, device=cuda_device)
            ids_np, w_np = synth.zipf_routing(B, E, k, seed=95 + call)
            ids = torch.from_numpy(ids_np).to(cuda_device)
            w = torch.from_numpy(w_np).to(cuda_device)
            for dt in (torch.float32, torch.bfloat16):
                y_ep = ep(x, ids, w, out_dtype=dt)
                y_one = full.forward(x, ids, w, out_dtype=dt)
                torch.cuda.synchronize()
                assert y_ep.shape == (B, H) and y_ep.dtype == dt
                assert torch.equal(y_ep, y_one), f"B={B} {dt}: max |diff| {(y_ep.float() - y_one.float()).abs().max()}"
        ep.status()
    finally:
        ep.close()


def test_single_rank_placement_equals_the_relabelled_layer(cuda_device):
    """With an expert placement (perm[e] = position), the layer equals the
    single-GPU layer over the experts in position order fed ids perm[ids]."""
    import numpy as np
    from sb200 import synth
    from sb200.ep import ExpertParallelMoE, experts_at
    from sb200.ternary import TernaryExperts
    E, H, I, k = 16, 512, 256, 4
    experts = synth.ternary_experts(E, H, I, seed=62)
    perm = [int(p) for p in np.random.default_rng(7).permutation(E)]
    ordered = [experts[e] for e in experts_at(perm, 0, 1)]
    full = TernaryExperts(ordered, cuda_device)
    ep = ExpertParallelMoE(TernaryExperts(ordered, cuda_device), E, k, 1024, placement=perm)
    try:
        perm_t = torch.tensor(perm, dtype=torch.int64, device=cuda_device)
        for call, B in enumerate([300, 1024, 1]):
            x = synth.hidden_states(B, H, seed=63 + call, dtype=torch.bfloat16, device=cuda_device)
            ids_np, w_np = synth.zipf_routing(B, E, k, seed=64 + call)
            ids = torch.from_numpy(ids_np).to(cuda_device)
            w = torch.from_numpy(w_np).to(cuda_device)
            y_ep = ep(x, ids, w, out_dtype=torch.float32)
            y_one = full.forward(x, perm_t[ids.long()].to(torch.int32), w, out_dtype=torch.float32)
            torch.cuda.synchronize()
            assert torch.equal(y_ep, y_one), f"B={B}: max |diff| {(y_ep - y_one).abs().max()}"
        ep.status()
        with pytest.raises(RuntimeError, match="permutation"):
            ExpertParallelMoE(TernaryExperts(ordered, cuda_device), E, k, 64, placement=[0] * E)
    finally:
        ep.close()


@pytest.mark.parametrize("chunks", [1, 3])
def test_sharded_layer_equals_single_gpu_layer(cuda_device, chunks):
    """The whole layer (router top-k, then the exchange) against BVHMoELayer,
    with the batch split into token ranges on their own streams, eagerly and
    replayed from a CUDA graph."""
    import numpy as np
    from bvh_router import BVHRouter, RouterConfig
    from sb200 import synth
    from sb200.ep import EPMoELayer
    from sb200.moe import BVHMoELayer, GraphedLayer
    from sb200.ternary import TernaryExperts
    H, S, E, I, k, B = 2048, 256, 64, 1024, 8, 1000
    w = synth.router_weights(H, S, (4, 4, 4), seed=0)
    r = BVHRouter(RouterConfig(embed_dim=H, spectral_dim=S))
    r.load_state_dict({kk: torch.from_numpy(np.array(v)) for kk, v in w.items()})
    r = r.to(cuda_device).eval()
    experts = synth.ternary_experts(E, H, I, seed=2)
    one = BVHMoELayer(r, TernaryExperts(experts, cuda_device), top_k=k)
    sharded = EPMoELayer(r, TernaryExperts(experts, cuda_device), E, k, B, chunks=chunks)
    try:
        x = synth.hidden_states(B, H, seed=5, dtype=torch.bfloat16, device=cuda_device)
        y1 = one(x)
        y2 = sharded(x)
        out = torch.empty_like(y1)
        g = GraphedLayer(sharded)
        g(x, out)
        g(x, out)
        torch.cuda.synchronize()
        assert torch.equal(y1, y2)
        assert torch.equal(y1, out)
        sharded.status()
    finally:
        sharded.close()


def test_stale_wait_is_reported_and_the_gpu_keeps_working(cuda_device):
    from sb200 import _lib, synth
    full, ep = _layers(8, 256, 128, 4, 64, cuda_device, timeout_ms=200)
    lib = _lib.load()
    try:
        s = torch.cuda.current_stream(cuda_device).cuda_stream
        _lib.check(lib.sb_ep_inject_stale_wait(ep.handle, C.c_void_p(s)), "sb_ep_inject_stale_wait")
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="ran out"):
            ep.status()
        assert lib.sb_device_status(0) == -4      # SB_ERR_DEVICE_TIMEOUT; reading clears it
        assert lib.sb_device_status(0) == 0
        # the context is intact: the single-GPU layer still runs and matches itself
        x = synth.hidden_states(50, 256, seed=3, dtype=torch.bfloat16, device=cuda_device)
        ids_np, w_np = synth.zipf_routing(50, 8, 4, seed=4)
        ids, w = torch.from_numpy(ids_np).to(cuda_device), torch.from_numpy(w_np).to(cuda_device)
        a = full.forward(x, ids, w)
        b = full.forward(x, ids, w)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
    finally:
        ep.close()


def test_bad_arguments_are_rejected_on_the_host(cuda_device):
    from sb200 import _lib
    lib = _lib.load()
    h = C.c_void_p()
    for desc in [_lib.EpDesc(0, 0, 64, 8, 16, 256, 128, 0), _lib.EpDesc(2, 2, 64, 8, 16, 256, 128, 0),
                 _lib.EpDesc(3, 0, 64, 8, 16, 256, 128, 0), _lib.EpDesc(1, 0, 64, 17, 16, 256, 128, 0),
                 _lib.EpDesc(1, 0, 64, 8, 16, 250, 128, 0)]:
        assert lib.sb_ep_create(C.byref(desc), C.byref(h)) == -1
    full, ep = _layers(8, 256, 128, 4, 64, cuda_device)
    try:
        x = torch.zeros(65, 256, dtype=torch.bfloat16, device=cuda_device)
        ids = torch.zeros(65, 4, dtype=torch.int32, device=cuda_device)
        w = torch.ones(65, 4, device=cuda_device)
        with pytest.raises(RuntimeError, match="max_tokens"):
            ep(x, ids, w)
        with pytest.raises(RuntimeError, match="bf16"):
            ep(x[:8].float(), ids[:8], w[:8])
        with pytest.raises(RuntimeError, match="has not run"):
            h2 = C.c_void_p()
            _lib.check(lib.sb_ep_create(C.byref(_lib.EpDesc(2, 0, 8, 4, 16, 256, 128, 0)), C.byref(h2)), "create")
            try:
                _lib.check(lib.sb_ep_forward(h2, None, 1, 0, None, None, None, None, None, None, None, None,
                                             None, 0, None, 0, None), "sb_ep_forward")
            finally:
                lib.sb_ep_destroy(h2)
    finally:
        ep.close()


# ---------------------------------------------------------------------------
# several GPUs
# ---------------------------------------------------------------------------
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, use_nccl):
    sys.path.insert(0, str(REPO / "spectral-ai_b200"))
    sys.path.insert(0, str(REPO))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist
    from sb200 import _lib, synth
    from sb200.ep import ExpertParallelMoE
    from sb200.ternary import TernaryExperts
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    lib = _lib.load()
    comm = None
    results = []
    try:
        import numpy as np
        from sb200.ep import experts_at
        E, H, I, k = 64, 2048, 1024, 8
        experts = synth.ternary_experts(E, H, I, seed=61)
        el = E // world
        # the NCCL set-up path also runs with an expert placement (the same
        # seeded permutation on every rank); the reference then takes the
        # experts in position order and ids perm[ids]
        perm = [int(p) for p in np.random.default_rng(11).permutation(E)] if use_nccl else list(range(E))
        order = experts_at(perm, 0, 1)
        full = TernaryExperts([experts[e] for e in order], dev)
        perm_t = torch.tensor(perm, dtype=torch.int64, device=dev)
        if use_nccl:
            uid = C.create_string_buffer(128)
            if rank == 0:
                _lib.check(lib.sb_nccl_unique_id(uid), "sb_nccl_unique_id")
            box = [uid.raw]
            dist.broadcast_object_list(box, src=0)
            cp = C.c_void_p()
            _lib.check(lib.sb_nccl_comm_init(world, rank, C.c_char_p(box[0]), C.byref(cp)), "sb_nccl_comm_init")
            comm = cp.value
        mine = [experts[e] for e in experts_at(perm, rank, world)]
        ep = ExpertParallelMoE(TernaryExperts(mine, dev), E, k, 4096, timeout_ms=1000, nccl_comm=comm,
                               placement=perm if use_nccl else None)
        sizes = [[700 + 37 * r for r in range(world)], [4096] * world, [5] + [0] * (world - 1),
                 [2000] * world]
        for step, Bs in enumerate(sizes):
            # every rank's tokens of this step (each rank routes its own); the
            # single-GPU layer runs them all at once, so every expert sees the
            # same rows in both layers
            xs, idss, ws = [], [], []
            for r in range(world):
                xs.append(synth.hidden_states(Bs[r], H, seed=70 + 10 * step + r, dtype=torch.bfloat16, device=dev))
                ids_np, w_np = synth.zipf_routing(Bs[r], E, k, seed=80 + 10 * step + r)
                idss.append(torch.from_numpy(ids_np).to(dev))
                ws.append(torch.from_numpy(w_np).to(dev))
            y_ep = ep(xs[rank], idss[rank], ws[rank], out_dtype=torch.float32)
            ids_pos = perm_t[torch.cat(idss).long()].to(torch.int32)
            y_all = full.forward(torch.cat(xs), ids_pos, torch.cat(ws), out_dtype=torch.float32)
            lo = sum(Bs[:rank])
            y_one = y_all[lo:lo + Bs[rank]]
            torch.cuda.synchronize()
            results.append((step, bool(torch.equal(y_ep, y_one)),
                            float((y_ep - y_one).abs().max()) if Bs[rank] else 0.0))
        ep.status()
        # a rank that skips a forward: the other's waits run out and it says so
        dist.barrier()
        if rank == 0:
            x = synth.hidden_states(64, H, seed=5, dtype=torch.bfloat16, device=dev)
            ids_np, w_np = synth.zipf_routing(64, E, k, seed=6)
            ep(x, torch.from_numpy(ids_np).to(dev), torch.from_numpy(w_np).to(dev))
            torch.cuda.synchronize()
            try:
                ep.status()
                results.append(("skip", False, 0.0))
            except RuntimeError as e:
                results.append(("skip", "ran out" in str(e), 0.0))
            lib.sb_device_status(rank)   # clear this GPU's status word
        dist.barrier()
        ep.close()
        q.put((rank, results))
    finally:
        if comm is not None:
            lib.sb_nccl_comm_destroy(C.c_void_p(comm))
        dist.destroy_process_group()


@pytest.mark.parametrize("use_nccl", [False, True])
def test_all_gpus_bitwise_and_a_skipped_forward(use_nccl):
    """On every GPU of the box (the largest power of two, at most 8)."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = 8 if n >= 8 else 4 if n >= 4 else 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, use_nccl)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    res = dict(q.get(timeout=5) for _ in range(world))
    for rank, rows in res.items():
        for step, ok, err in rows:
            assert ok, f"rank {rank} step {step}: max |diff| {err}"
    assert any(step == "skip" for step, _, _ in res[0])
