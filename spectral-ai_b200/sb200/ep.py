"""Expert-parallel MoE layer over the GPUs of one node (one process per GPU).

With E experts on W ranks, rank r holds experts [r*E/W, (r+1)*E/W).  The
layer's own kernels (``sb_ep_forward``, csrc/ep.cu) move every token row once
to each rank that holds one of its experts and bring back one partial sum per
(token, rank), all through peer memory over NVLink: there is no host
synchronisation and no library collective on the data path.  The output equals
the single-GPU layer (``TernaryExperts.forward``) bit for bit when E/W is a
power of two, because both add a token's expert outputs along the same binary
tree over the expert ids (csrc/tree_sum.cuh).

The reference has no multi-GPU code; this replaces its per-slot Python
dispatch loop (python/olmoe_extract.py:146-155) when the experts are spread
over GPUs.

``torch.distributed`` is the plumbing of the set-up only: the ranks exchange
the 128-byte IPC handles of their receive buffers (``exchange_handles``), or
the C ABI does it over an NCCL communicator (``sb_ep_connect_nccl``).

``AllToAllMoE`` is the same layer over the library collective
(``torch.distributed.all_to_all_single``, NCCL), kept as the measured baseline
of the fused exchange.
"""

from __future__ import annotations

import ctypes as C
from typing import Callable, Optional, Sequence

import torch
import torch.distributed as dist

from . import _lib


def exchange_handles(mine: bytes, group: Optional[dist.ProcessGroup] = None) -> bytes:
    """Every rank's handle bytes, concatenated in rank order (a collective).
    Raises if a rank does not join within the process group's timeout."""
    world = dist.get_world_size(group)
    got = [None] * world
    dist.all_gather_object(got, bytes(mine), group=group)
    if any(g is None or len(g) != len(mine) for g in got):
        raise RuntimeError("handle exchange: a rank sent no handle")
    return b"".join(got)


def balanced_placement(loads: Sequence[float], world: int, group: int = 1) -> list:
    """An expert placement (``perm[e]`` = expert e's position; rank r holds
    positions [r*E/W, (r+1)*E/W)) that evens out the ranks' expert loads:
    units of ``group`` consecutive experts, in falling order of load, each to
    the least-loaded rank that still has room (longest-processing-time first,
    E/W experts per rank), each rank's experts then in ascending id.
    ``loads`` are per-expert entry counts from routing statistics (a
    calibration batch).  Keeping groups of experts that a router tends to
    select together (the BVH router's sibling leaves) on one rank keeps the
    number of ranks a token visits close to contiguous blocks' while the
    loads even out; ``group=1`` balances best and scatters most."""
    E = len(loads)
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    el = E // world
    if group < 1 or el % group:
        raise ValueError(f"group {group} does not divide the {el} experts of a rank")
    units = E // group
    uload = [sum(float(loads[u * group + j]) for j in range(group)) for u in range(units)]
    order = sorted(range(units), key=lambda u: (-uload[u], u))
    cap = el // group
    bins = [[] for _ in range(world)]
    tot = [0.0] * world
    for u in order:
        r = min((r for r in range(world) if len(bins[r]) < cap), key=lambda r: (tot[r], r))
        bins[r].append(u)
        tot[r] += uload[u]
    perm = [0] * E
    for r in range(world):
        for j, u in enumerate(sorted(bins[r])):
            for i in range(group):
                perm[u * group + i] = r * el + j * group + i
    return perm


def refine_placement(perm: Sequence[int], ids, world: int, iters: int = 3000, entry_ns: float = 12.0,
                     row_ns: float = 37.0, seed: int = 0) -> list:
    """Improves a placement against routing statistics: random swaps of two
    experts on different ranks, kept when they lower the modelled step time
        entry_ns * (entries on the busiest rank) + row_ns * (rows sent) / W,
    the first term the grouped GEMMs of the rank everyone waits for, the
    second the exchange (each token goes once to each rank holding any of its
    experts).  The default weights are per-entry GEMM and per-row exchange
    costs measured on 8 B200s (the expert-parallel layer's launch breakdown).
    ``ids``: [T, k] expert ids of calibration tokens (all ranks' tokens, the
    same array on every rank, so that every rank gets the same placement)."""
    import numpy as np
    ids = np.asarray(ids, dtype=np.int64)
    E = len(perm)
    el = E // world
    perm = np.asarray(perm, dtype=np.int64).copy()
    T, k = ids.shape
    load = np.bincount(ids.ravel(), minlength=E).astype(np.float64)
    # cnt[t, r]: slots of token t whose expert lives on rank r
    cnt = np.zeros((T, world), np.int32)
    np.add.at(cnt, (np.repeat(np.arange(T), k), (perm[ids] // el).ravel()), 1)
    ent = np.bincount((perm // el), weights=load, minlength=world)
    rows = float((cnt > 0).sum())
    # each expert's tokens and how many of their slots name it
    flat_t = np.repeat(np.arange(T), k)
    order = np.argsort(ids.ravel(), kind="stable")
    bounds = np.searchsorted(ids.ravel()[order], np.arange(E + 1))
    toks, mult = [], []
    for e in range(E):
        t, m = np.unique(flat_t[order[bounds[e]:bounds[e + 1]]], return_counts=True)
        toks.append(t)
        mult.append(m.astype(np.int32))
    cost = entry_ns * ent.max() + row_ns * rows / world
    rng = np.random.default_rng(seed)
    for _ in range(iters):
        e1, e2 = (int(v) for v in rng.integers(0, E, 2))
        r1, r2 = int(perm[e1] // el), int(perm[e2] // el)
        if r1 == r2:
            continue
        tt = np.union1d(toks[e1], toks[e2])
        before = (cnt[tt][:, [r1, r2]] > 0).sum()
        cnt[toks[e1], r1] -= mult[e1]
        cnt[toks[e1], r2] += mult[e1]
        cnt[toks[e2], r2] -= mult[e2]
        cnt[toks[e2], r1] += mult[e2]
        after = (cnt[tt][:, [r1, r2]] > 0).sum()
        d = load[e2] - load[e1]
        ent[r1] += d
        ent[r2] -= d
        new_rows = rows + float(after - before)
        new_cost = entry_ns * ent.max() + row_ns * new_rows / world
        if new_cost < cost:
            cost, rows = new_cost, new_rows
            perm[e1], perm[e2] = perm[e2], perm[e1]
        else:  # undo
            cnt[toks[e1], r1] += mult[e1]
            cnt[toks[e1], r2] -= mult[e1]
            cnt[toks[e2], r2] += mult[e2]
            cnt[toks[e2], r1] -= mult[e2]
            ent[r1] -= d
            ent[r2] += d
    # each rank's experts in ascending id (any order within a rank is valid;
    # this one keeps a unit's experts adjacent)
    out = [0] * E
    for r in range(world):
        held = sorted(e for e in range(E) if perm[e] // el == r)
        for j, e in enumerate(held):
            out[e] = r * el + j
    return out


def experts_at(perm: Sequence[int], rank: int, world: int) -> list:
    """The expert ids rank ``rank`` holds under ``perm``, in position order."""
    E = len(perm)
    el = E // world
    inv = [0] * E
    for e, p in enumerate(perm):
        inv[p] = e
    return inv[rank * el:(rank + 1) * el]


class ExpertParallelMoE:
    """The grouped ternary SwiGLU with this rank's experts and the token
    exchange on the device.  ``local_experts`` (``TernaryExperts``) holds the
    experts at positions [rank*E/W, (rank+1)*E/W) in position order: experts
    [rank*E/W, ...) themselves, or ``experts_at(placement, rank, W)`` with a
    ``placement``.  ``forward`` is collective: every rank calls it equally
    often."""

    def __init__(self, local_experts, n_experts: int, top_k: int, max_tokens: int,
                 group: Optional[dist.ProcessGroup] = None, timeout_ms: int = 2000,
                 nccl_comm: Optional[int] = None, workspace: Optional[torch.Tensor] = None,
                 placement: Optional[Sequence[int]] = None):
        """``workspace``: a uint8 device buffer to use (and grow) instead of a
        private one, for layers that run one after another on one stream (a
        stack); ``self.workspace`` is the buffer in use.  ``placement``: expert
        id -> position (``balanced_placement``), the same on every rank."""
        self.lib = _lib.load()
        self.experts = local_experts
        self.device = local_experts.device
        if self.device.type != "cuda":
            raise RuntimeError("the expert-parallel layer runs on CUDA devices only")
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if n_experts % self.world or local_experts.E != n_experts // self.world:
            raise ValueError(f"{local_experts.E} local experts do not make {n_experts} over {self.world} ranks")
        self.n_experts, self.top_k, self.max_tokens = int(n_experts), int(top_k), int(max_tokens)
        desc = _lib.EpDesc(self.world, self.rank, self.n_experts, self.top_k, self.max_tokens,
                           local_experts.H, local_experts.I, int(timeout_ms))
        self.handle = C.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(self.lib.sb_ep_create(C.byref(desc), C.byref(self.handle)), "sb_ep_create")
            try:
                if self.world > 1:
                    if nccl_comm is not None:
                        s = torch.cuda.current_stream(self.device).cuda_stream
                        _lib.check(self.lib.sb_ep_connect_nccl(self.handle, C.c_void_p(nccl_comm), C.c_void_p(s)),
                                   "sb_ep_connect_nccl")
                    else:
                        buf = C.create_string_buffer(_lib.SB_EP_HANDLE_BYTES)
                        _lib.check(self.lib.sb_ep_export(self.handle, buf), "sb_ep_export")
                        allb = exchange_handles(buf.raw, group)
                        _lib.check(self.lib.sb_ep_connect(self.handle, C.c_char_p(allb)), "sb_ep_connect")
                if placement is not None:
                    perm = (C.c_int32 * self.n_experts)(*[int(p) for p in placement])
                    if len(placement) != self.n_experts:
                        raise ValueError(f"placement names {len(placement)} experts, the layer has {self.n_experts}")
                    _lib.check(self.lib.sb_ep_set_placement(self.handle, perm), "sb_ep_set_placement")
            except Exception:
                self.lib.sb_ep_destroy(self.handle)
                self.handle = None
                raise
            nbytes = int(self.lib.sb_ep_workspace_bytes(self.handle))
            if workspace is not None and workspace.numel() >= nbytes + 1024:
                self.workspace = workspace
            else:
                self.workspace = torch.empty(nbytes + 1024, dtype=torch.uint8, device=self.device)
            base = self.workspace.data_ptr()
            self._ws = (base + 1023) // 1024 * 1024
            self._ws_bytes = nbytes

    def forward(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                out_dtype=torch.bfloat16, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.handle is None:
            raise RuntimeError("the layer was closed")
        if not (x.is_cuda and x.dtype == torch.bfloat16):
            raise RuntimeError("activations must be bf16 CUDA tensors")
        x = x.contiguous()
        ids = ids.to(torch.int32).contiguous()
        weights = weights.to(torch.float32).contiguous()
        B = ids.shape[0]
        if ids.shape[1] != self.top_k:
            raise RuntimeError(f"ids carry {ids.shape[1]} slots, the layer was set up for {self.top_k}")
        if out is None:
            out = torch.empty(B, self.experts.H, dtype=out_dtype, device=x.device)
        e = self.experts
        s = torch.cuda.current_stream(x.device).cuda_stream
        with torch.cuda.device(x.device):
            rc = self.lib.sb_ep_forward(
                self.handle, C.c_void_p(x.data_ptr()), _lib.SB_BF16, B, C.c_void_p(ids.data_ptr()),
                C.c_void_p(weights.data_ptr()), C.c_void_p(e.gate.data_ptr()), C.c_void_p(e.up.data_ptr()),
                C.c_void_p(e.down.data_ptr()), C.c_void_p(e.gate_scale.data_ptr()),
                C.c_void_p(e.up_scale.data_ptr()), C.c_void_p(e.down_scale.data_ptr()),
                C.c_void_p(out.data_ptr()), _lib.SB_BF16 if out.dtype == torch.bfloat16 else _lib.SB_F32,
                C.c_void_p(self._ws), self._ws_bytes, C.c_void_p(s))
        _lib.check(rc, "sb_ep_forward")
        return out

    __call__ = forward

    def status(self) -> None:
        """Raises if a wait for a peer ran out (synchronises the device)."""
        _lib.check(self.lib.sb_ep_status(self.handle), "sb_ep_status")

    def close(self) -> None:
        """Collective: a barrier, then the buffers are released on every rank."""
        if self.handle is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        self.lib.sb_ep_destroy(self.handle)
        self.handle = None


class AllToAllMoE:
    """The same layer over the library collective: ``all_to_all_single``
    (NCCL) of the counts, then of the token rows (one per slot), local expert
    ids and weights; fp32 expert outputs back; the token's slots summed in slot
    order.  Host-synchronised split sizes.  Kept as the baseline the fused
    exchange is measured against."""

    def __init__(self, expert_fn: Callable, n_experts: int, group: Optional[dist.ProcessGroup] = None):
        """expert_fn(x_rows [R,H], local_ids [R,1] int32, weights [R,1] fp32) -> fp32 [R,H]."""
        self.expert_fn = expert_fn
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not divide over {self.world} ranks")
        self.n_experts = n_experts
        self.e_local = n_experts // self.world

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                out_dtype=None) -> torch.Tensor:
        B, k = ids.shape
        H = x.shape[1]
        dev = x.device
        flat_ids = ids.reshape(-1).to(torch.int64)
        if B and (int(flat_ids.min()) < 0 or int(flat_ids.max()) >= self.n_experts):
            raise RuntimeError("expert id out of range")
        dest = torch.div(flat_ids, self.e_local, rounding_mode="floor")
        order = torch.sort(dest, stable=True).indices
        send_counts = torch.bincount(dest, minlength=self.world).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)
        sc = send_counts.tolist()
        rc = recv_counts.tolist()
        R_send, R_recv = sum(sc), sum(rc)

        send_rows = x.index_select(0, torch.div(order, k, rounding_mode="floor")).contiguous()
        send_eid = (flat_ids.index_select(0, order) - dest.index_select(0, order) * self.e_local).to(torch.int32)
        send_w = weights.reshape(-1).to(torch.float32).index_select(0, order).contiguous()

        recv_rows = torch.empty(R_recv, H, dtype=x.dtype, device=dev)
        recv_eid = torch.empty(R_recv, dtype=torch.int32, device=dev)
        recv_w = torch.empty(R_recv, dtype=torch.float32, device=dev)
        self._a2a(recv_rows, send_rows, rc, sc)
        self._a2a(recv_eid, send_eid.contiguous(), rc, sc)
        self._a2a(recv_w, send_w, rc, sc)

        if R_recv:
            y_recv = self.expert_fn(recv_rows, recv_eid.view(-1, 1), recv_w.view(-1, 1))
        else:
            y_recv = torch.empty(0, H, dtype=torch.float32, device=dev)
        y_send = torch.empty(R_send, H, dtype=torch.float32, device=dev)
        self._a2a(y_send, y_recv.to(torch.float32).contiguous(), sc, rc)

        y_slots = torch.empty(B * k, H, dtype=torch.float32, device=dev)
        y_slots.index_copy_(0, order, y_send)
        y_slots = y_slots.view(B, k, H)
        out = torch.zeros(B, H, dtype=torch.float32, device=dev)
        for j in range(k):
            out.add_(y_slots[:, j])
        return out.to(out_dtype or x.dtype)

    __call__ = forward



class EPMoELayer:
    """The MoE layer with its experts sharded: the router's top-k on this rank's
    tokens, then the expert-parallel exchange.  Same call as
    ``sb200.moe.BVHMoELayer`` (``layer(x, out=...)``), so it can be replayed
    from a CUDA graph (``sb200.moe.GraphedLayer``: the exchange's flags carry an
    epoch kept in device memory, and no host work sits between the kernels).

    ``chunks`` > 1 splits each batch into that many consecutive token ranges,
    each with its own exchange handle and stream, so one range's transfers over
    NVLink run while another range's grouped GEMMs hold the tensor cores (the
    exchange kernels fit on the SMs beside a GEMM's persistent CTA)."""

    def __init__(self, router, local_experts, n_experts: int, top_k: int, max_tokens: int,
                 select: str = "soft", chunks: int = 1, group: Optional[dist.ProcessGroup] = None,
                 timeout_ms: int = 2000, workspace: Optional[torch.Tensor] = None,
                 placement: Optional[Sequence[int]] = None):
        """``workspace``: a buffer shared with layers that run one after
        another on the same stream (``chunks`` == 1 only).  ``placement``: as
        for ``ExpertParallelMoE`` (``local_experts`` in position order)."""
        self.router = router
        self.top_k = int(top_k)
        self.select = select
        self.chunks = max(1, int(chunks))
        per = (int(max_tokens) + self.chunks - 1) // self.chunks
        self.eps = [ExpertParallelMoE(local_experts, n_experts, top_k, per, group=group, timeout_ms=timeout_ms,
                                      workspace=workspace if self.chunks == 1 else None, placement=placement)
                    for _ in range(self.chunks)]
        self.per = per
        dev = local_experts.device
        self.streams = [torch.cuda.Stream(dev) for _ in range(self.chunks)] if self.chunks > 1 else []

    @property
    def ep(self):
        return self.eps[0]

    def route(self, x: torch.Tensor):
        return self.router.forward_topk(x, k=self.top_k, select=self.select)

    def forward(self, x: torch.Tensor, out_dtype=None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        ids, w = self.route(x)
        B = x.shape[0]
        if out is None:
            out = torch.empty(B, x.shape[1], dtype=out_dtype or x.dtype, device=x.device)
        if self.chunks == 1:
            return self.eps[0](x, ids, w, out=out)
        main = torch.cuda.current_stream(x.device)
        for c, (ep, s) in enumerate(zip(self.eps, self.streams)):
            lo, hi = min(c * self.per, B), min((c + 1) * self.per, B)
            s.wait_stream(main)
            with torch.cuda.stream(s):
                ep(x[lo:hi], ids[lo:hi], w[lo:hi], out=out[lo:hi])
            for t in (x, ids, w, out):
                t.record_stream(s)
        for s in self.streams:
            main.wait_stream(s)
        return out

    __call__ = forward

    def status(self) -> None:
        for ep in self.eps:
            ep.status()

    def close(self) -> None:
        for ep in self.eps:
            ep.close()
