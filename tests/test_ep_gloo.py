"""The expert-parallel layer's host side on 2 CPU ranks (gloo), no GPU.

* The exchange protocol of csrc/ep.cu stated on the CPU (oracle/ep.py) and run
  between two real ranks over torch.distributed: every token reaches each rank
  that holds one of its experts once, the partial sums come back, and the
  result equals the single-process tree sum bit for bit.
* A rank that leaves between steps: the survivor's next exchange ends with an
  error inside the process group's timeout instead of hanging.
* The set-up collective of sb200.ep.ExpertParallelMoE (exchange_handles):
  every rank gets every rank's handle bytes in rank order, and a rank that
  never joins makes the others raise.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys
import time
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


def _init(rank, world, port, timeout_s=60):
    sys.path.insert(0, str(REPO / "spectral-ai_b200"))
    sys.path.insert(0, str(REPO))
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _expert_rows(experts, x_rows, ids_rows, w_rows, select):
    """Weighted slot outputs y[i, j] = w * expert_{ids[i,j]}(x[i]) for the slots
    `select(e)` accepts (others 0); one row at a time so every rank computes the
    same fp32 value for the same (row, expert)."""
    from oracle import ternary as otern
    B, k = ids_rows.shape
    y = np.zeros((B, k, x_rows.shape[1]), np.float32)
    for i in range(B):
        for j in range(k):
            e = int(ids_rows[i, j])
            if select(e):
                ex = experts[e]
                y[i, j] = np.float32(w_rows[i, j]) * otern.gated_mlp_f32(
                    x_rows[i:i + 1], ex["gate_ternary"], ex["up_ternary"], ex["down_ternary"],
                    ex["gate_scale"], ex["up_scale"], ex["down_scale"])[0]
    return y


def _exchange_step(dist, rank, world, E, experts, x, ids, w):
    """One forward of the protocol between the ranks (all_to_all over gloo)."""
    from oracle import ep as oep
    el = E // world
    H = x.shape[1]
    k = ids.shape[1]
    send_pos, lists = oep.plan_destinations(ids, E, world)
    counts = torch.tensor([len(l) for l in lists], dtype=torch.int64)
    rcounts = torch.empty_like(counts)
    dist.all_to_all_single(rcounts, counts)
    sc, rc = counts.tolist(), rcounts.tolist()
    order = [t for g in range(world) for t in lists[g]]
    send_x = torch.from_numpy(np.ascontiguousarray(x[order], np.float32)).reshape(-1, H)
    send_i = torch.from_numpy(np.ascontiguousarray(ids[order], np.int32)).reshape(-1, k)
    send_w = torch.from_numpy(np.ascontiguousarray(w[order], np.float32)).reshape(-1, k)
    recv_x = torch.empty(sum(rc), H)
    recv_i = torch.empty(sum(rc), k, dtype=torch.int32)
    recv_w = torch.empty(sum(rc), k)
    dist.all_to_all_single(recv_x, send_x, rc, sc)
    dist.all_to_all_single(recv_i, send_i, rc, sc)
    dist.all_to_all_single(recv_w, send_w, rc, sc)
    y = _expert_rows(experts, recv_x.numpy(), recv_i.numpy(), recv_w.numpy(), lambda e: e // el == rank)
    part = oep.destination_partials(recv_i.numpy(), y, rank, E, world) if len(y) else np.zeros((0, H), np.float32)
    back = torch.empty(sum(sc), H)
    dist.all_to_all_single(back, torch.from_numpy(np.ascontiguousarray(part)).reshape(-1, H), sc, rc)
    back = back.numpy()
    partials, o = [], 0
    for g in range(world):
        partials.append(back[o:o + sc[g]])
        o += sc[g]
    return oep.source_combine(send_pos, partials)


def _protocol_worker(rank, world, port, q, case):
    dist = _init(rank, world, port)
    try:
        from oracle import ep as oep
        from sb200 import synth
        E, H, I, B, k = case
        experts = synth.ternary_experts(E, H, I, seed=31)
        x = synth.hidden_states(B, H, seed=40 + rank).numpy()
        ids, w = synth.zipf_routing(B, E, k, seed=50 + rank)
        got = _exchange_step(dist, rank, world, E, experts, x, ids, w)
        y_all = _expert_rows(experts, x, ids, w, lambda e: True)
        ref = oep.combine_single(ids, y_all) if B else np.zeros((0, H), np.float32)
        q.put((rank, bool(np.array_equal(got, ref)), float(np.abs(got - ref).max(initial=0.0))))
    finally:
        dist.destroy_process_group()


def _run(target, world, args, timeout=180):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
    codes = [p.exitcode for p in procs]
    res = []
    while not q.empty():
        res.append(q.get(timeout=5))
    return codes, sorted(res)


@pytest.mark.parametrize("case", [(8, 32, 48, 13, 3), (4, 16, 16, 1, 2), (6, 24, 32, 0, 2), (16, 16, 16, 40, 8)])
def test_protocol_two_ranks_matches_single_process_bitwise(case):
    codes, res = _run(_protocol_worker, 2, (case,))
    assert codes == [0, 0]
    assert len(res) == 2
    for rank, equal, err in res:
        assert equal, (rank, err)


def _flush_exit(q):
    """Leave at once, after the queue's feeder thread has handed over what was put."""
    q.close()
    q.join_thread()
    os._exit(0)


def _leave_worker(rank, world, port, q):
    dist = _init(rank, world, port, timeout_s=8)
    from sb200 import synth
    E, H, I, B, k = 8, 16, 16, 9, 2
    experts = synth.ternary_experts(E, H, I, seed=31)
    x = synth.hidden_states(B, H, seed=40 + rank).numpy()
    ids, w = synth.zipf_routing(B, E, k, seed=50 + rank)
    _exchange_step(dist, rank, world, E, experts, x, ids, w)       # step 1 on both ranks
    if rank == 1:
        q.put((1, "left", 0.0))
        _flush_exit(q)                                               # leaves between steps
    t0 = time.time()
    try:
        _exchange_step(dist, rank, world, E, experts, x, ids, w)   # step 2: the peer is gone
        q.put((0, "completed", time.time() - t0))
    except Exception as e:  # gloo reports the closed peer or the timeout
        q.put((0, "raised:" + type(e).__name__, time.time() - t0))
    _flush_exit(q)


def test_rank_leaving_between_steps_ends_the_next_step_with_an_error():
    codes, res = _run(_leave_worker, 2, (), timeout=120)
    assert codes == [0, 0]
    d = {r: (what, dt) for r, what, dt in res}
    assert d[1][0] == "left"
    assert d[0][0].startswith("raised"), d[0]
    assert d[0][1] < 60.0


def _handles_worker(rank, world, port, q, missing):
    dist = _init(rank, world, port, timeout_s=6)
    from sb200.ep import exchange_handles
    mine = bytes([rank + 1]) * 128
    if missing and rank == 1:
        q.put((1, "absent", b""))
        _flush_exit(q)
    try:
        got = exchange_handles(mine)
        q.put((rank, "ok", got))
    except Exception as e:
        q.put((rank, "raised:" + type(e).__name__, b""))
    _flush_exit(q)


def test_handle_exchange_gathers_in_rank_order():
    codes, res = _run(_handles_worker, 2, (False,))
    assert codes == [0, 0]
    for rank, what, got in res:
        assert what == "ok"
        assert got == bytes([1]) * 128 + bytes([2]) * 128


def test_handle_exchange_raises_when_a_rank_never_joins():
    codes, res = _run(_handles_worker, 2, (True,), timeout=120)
    assert codes == [0, 0]
    d = {r: what for r, what, _ in res}
    assert d[1] == "absent"
    assert d[0].startswith("raised"), d[0]
