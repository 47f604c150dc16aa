"""Expert-parallel MoE layer: experts sharded over the ranks of a process group,
tokens exchanged with all-to-all (NCCL over NVLink on B200; gloo on CPU for tests).

The reference has no multi-GPU code; this is the layer's distributed form.
With E experts on W ranks, rank r holds experts [r*E/W, (r+1)*E/W).  One
forward on every rank:

  1. local routing (ids, weights [B, k]) -> destination rank of every
     (token, slot) pair = ids // (E/W); pairs are grouped by destination with
     a stable sort;
  2. all-to-all of the pair counts, then of the token rows, local expert ids
     and routing weights (dispatch);
  3. the local experts run on the received rows (one slot per row, weight
     applied in the down-projection epilogue);
  4. all-to-all of the fp32 expert outputs back to the senders (combine), and
     out[t] = sum_j y[t, j] accumulated in slot order j = 0..k-1.

Because every row's expert output is computed by the same kernel with the
same arithmetic as in the single-GPU layer, and the final sum runs in the
same slot order, the sharded output equals the single-GPU output bit for bit.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


class ExpertParallelMoE:
    def __init__(self, expert_fn: Callable, n_experts: int, group: Optional[dist.ProcessGroup] = None):
        """expert_fn(x_rows [R,H], local_ids [R,1] int32, weights [R,1] fp32) -> fp32 [R,H]
        runs this rank's experts (``TernaryExperts.forward`` on a GPU)."""
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
        for j in range(k):   # 0 + y_0 + y_1 + ... in slot order, like the single-GPU combine
            out.add_(y_slots[:, j])
        return out.to(out_dtype or x.dtype)

    __call__ = forward
