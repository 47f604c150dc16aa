"""Drop-in ``async_pipeline_bridge`` for the B200 MoE pipeline.

Mirrors python/async_pipeline_bridge.py of the reference: ``PipelineConfig``
(:26-35), ``PipelineSlot`` (:38-46) and ``AsyncPipelineSimulator`` (:49-255)
with the same constructor, stages and entry points (``forward_sequential``,
``forward_pipelined`` with three slots two steps deep, ``flush``,
``benchmark``).  The stages run on the device instead of Python loops:

  route    the router (any module returning ``(probs, _)``; the drop-in
           EnhancedBVHRouter runs its sb_enh kernels), then ``sb_softmax_topk``:
           with a calibration state the Linear(E,E) calibration of the raw
           logits, softmax and top-k fused in one kernel (:99-105); without it
           the top-k of the router probabilities (:108-110);
  scatter  ``sb_scatter_by_expert``: per-expert token lists in token order on
           the device (the reference builds a dict with .item() per entry, :113-126);
  expert   experts that are ternary expert modules of equal shape run as one
           grouped ternary SwiGLU (sb_ternary_moe_swiglu); other modules run
           per expert on their gathered rows, and ``sb_weighted_combine`` sums
           the weighted outputs (:128-150).

``PipelineSlot.dispatch_indices`` holds the device lists as a
``DispatchTable``; ``as_dict()`` gives the reference's {expert: [tokens]}.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.nn as nn

from sb200 import pipeline as _pipe


@dataclass(frozen=True)
class PipelineConfig:
    """Configuration for the async pipeline."""
    num_experts: int = 64
    top_k: int = 8
    hidden_dim: int = 2048
    inter_dim: int = 1024
    max_batch: int = 512
    num_buffers: int = 3  # triple buffering
    use_cuda_streams: bool = True


@dataclass
class DispatchTable:
    """Per-expert routing entries on the device: ``entries[e, :counts[e]]``
    are the entry indices t*k + j of expert e in ascending order."""
    entries: torch.Tensor
    counts: torch.Tensor
    top_k: int

    def as_dict(self) -> Dict[int, List[int]]:
        """{expert: [token, ...]} as the reference's scatter stage builds it."""
        counts = self.counts.cpu().tolist()
        ent = self.entries.cpu()
        return {e: (ent[e, :c] // self.top_k).tolist() for e, c in enumerate(counts) if c > 0}


@dataclass
class PipelineSlot:
    """One slot in the triple buffer."""
    hidden: Optional[torch.Tensor] = None
    expert_ids: Optional[torch.Tensor] = None
    expert_weights: Optional[torch.Tensor] = None
    dispatch_indices: Optional[DispatchTable] = None
    output: Optional[torch.Tensor] = None
    batch_size: int = 0


def _grouped_ternary(experts, device):
    """One TernaryExperts block when every expert is a ternary expert module
    (packed reference layout, no output projection, equal shapes)."""
    try:
        from ternary_expert_ext_bridge import CUDATernaryExpertModule
        from sb200.ternary import TernaryExperts
    except Exception:
        return None
    if len(experts) == 0 or not all(isinstance(m, CUDATernaryExpertModule) and m.output_proj is None
                                    for m in experts):
        return None
    try:
        return TernaryExperts.from_packed_modules(list(experts), device)
    except RuntimeError:
        return None


class AsyncPipelineSimulator:
    """The tri-core MoE pipeline (route -> scatter -> expert) on one GPU."""

    def __init__(self, config: PipelineConfig, router: nn.Module, experts: nn.ModuleList,
                 calibration_state: Optional[dict] = None, device: str = "cuda"):
        self.config = config
        self.router = router
        self.experts = experts
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("the B200 pipeline runs on a CUDA device (there is no CPU path)")
        self.cal_layer: Optional[nn.Linear] = None
        if calibration_state is not None:
            self.cal_layer = nn.Linear(config.num_experts, config.num_experts)
            self.cal_layer.load_state_dict(calibration_state)
            self.cal_layer = self.cal_layer.to(self.device).eval()
        self.slots = [PipelineSlot() for _ in range(config.num_buffers)]
        self.step = 0
        self.streams: Optional[list] = None
        if config.use_cuda_streams:
            self.streams = [torch.cuda.Stream(device=self.device) for _ in range(3)]
        self._grouped = _grouped_ternary(experts, self.device)

    # ---- stages
    def _stage_route(self, slot: PipelineSlot, hidden: torch.Tensor) -> None:
        """Stage 0: route tokens to experts, top-k on the device.  A reused
        slot's scatter and output are cleared (the reference keeps them, so
        its flush can return a stale output of the slot's previous input)."""
        slot.hidden = hidden
        slot.batch_size = hidden.shape[0]
        slot.dispatch_indices = None
        slot.output = None
        k = self.config.top_k
        with torch.no_grad():
            probs, _ = self.router(hidden)
            if self.cal_layer is not None:
                ids, w, _ = _pipe.softmax_topk(self.router._last_logits, k, self.cal_layer.weight,
                                               self.cal_layer.bias, apply_softmax=True)
            else:
                ids, w, _ = _pipe.softmax_topk(probs, k, apply_softmax=False)
        slot.expert_ids = ids.long()
        slot.expert_weights = w

    def _stage_scatter(self, slot: PipelineSlot) -> None:
        """Stage 1: group the routing entries by expert (device, token order)."""
        ent, counts = _pipe.scatter_by_expert(slot.expert_ids, len(self.experts), store_entry=True)
        slot.dispatch_indices = DispatchTable(ent, counts, self.config.top_k)

    def _stage_expert(self, slot: PipelineSlot) -> None:
        """Stage 2: expert forward passes and the weighted combine."""
        hidden = slot.hidden
        B, H = hidden.shape
        k = self.config.top_k
        with torch.no_grad():
            if self._grouped is not None:
                slot.output = self._grouped.forward(hidden, slot.expert_ids, slot.expert_weights,
                                                    out_dtype=torch.float32).to(hidden.dtype)
                return
            table = slot.dispatch_indices
            eo = torch.zeros(B * k, H, dtype=torch.float32, device=hidden.device)
            counts = table.counts.cpu().tolist()
            for e, c in enumerate(counts):
                if c == 0:
                    continue
                rows = table.entries[e, :c].long()
                y = self.experts[e](hidden[rows // k])
                eo[rows] = y.detach().float()
            slot.output = _pipe.weighted_combine(eo.view(B, k, H), slot.expert_weights).to(hidden.dtype)

    # ---- entry points (same control flow as the reference, :152-208)
    def forward_sequential(self, hidden: torch.Tensor) -> torch.Tensor:
        """Sequential (non-pipelined) forward."""
        slot = PipelineSlot()
        self._stage_route(slot, hidden)
        self._stage_scatter(slot)
        self._stage_expert(slot)
        return slot.output

    def forward_pipelined(self, hidden: torch.Tensor) -> Optional[torch.Tensor]:
        """Pipelined forward: route step N, scatter N-1, expert N-2 on three
        streams; returns the output of the input given two calls earlier
        (None while the pipeline fills)."""
        if self.streams is None:
            return self.forward_sequential(hidden)
        nb = self.config.num_buffers
        slot = self.slots[self.step % nb]
        cur = torch.cuda.current_stream(self.device)
        self.streams[0].wait_stream(cur)
        with torch.cuda.stream(self.streams[0]):
            self._stage_route(slot, hidden)
        if self.step >= 1:
            prev = self.slots[(self.step - 1) % nb]
            self.streams[1].wait_stream(self.streams[0])
            with torch.cuda.stream(self.streams[1]):
                self._stage_scatter(prev)
        if self.step >= 2:
            pprev = self.slots[(self.step - 2) % nb]
            self.streams[2].wait_stream(self.streams[1])
            with torch.cuda.stream(self.streams[2]):
                self._stage_expert(pprev)
        self.step += 1
        if self.step >= 3:
            done = self.slots[(self.step - 3) % nb]
            cur.wait_stream(self.streams[2])
            return done.output
        return None

    def flush(self) -> List[torch.Tensor]:
        """Runs the stages still pending after the last input; returns their outputs."""
        if self.streams is not None:
            cur = torch.cuda.current_stream(self.device)
            for st in self.streams:
                cur.wait_stream(st)
        outputs = []
        for _ in range(2):
            self.step += 1
            if self.step >= 3:
                slot = self.slots[(self.step - 3) % self.config.num_buffers]
                if slot.dispatch_indices is None:
                    self._stage_scatter(slot)
                if slot.output is None:
                    self._stage_expert(slot)
                outputs.append(slot.output)
        return outputs

    def benchmark(self, batch_size: int = 64, num_steps: int = 100, warmup: int = 10) -> dict:
        """Sequential and pipelined time per step (host clock around a
        synchronize, as the reference measures)."""
        hidden = torch.randn(batch_size, self.config.hidden_dim, device=self.device)
        for _ in range(warmup):
            self.forward_sequential(hidden)
        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        for _ in range(num_steps):
            self.forward_sequential(hidden)
        torch.cuda.synchronize(self.device)
        seq_time = (time.perf_counter() - t0) / num_steps
        self.step = 0
        for _ in range(warmup):
            self.forward_pipelined(hidden)
        torch.cuda.synchronize(self.device)
        self.step = 0
        t0 = time.perf_counter()
        for _ in range(num_steps + 2):
            self.forward_pipelined(hidden)
        torch.cuda.synchronize(self.device)
        pipe_time = (time.perf_counter() - t0) / num_steps
        return {"sequential_ms": seq_time * 1000, "pipelined_ms": pipe_time * 1000,
                "speedup": seq_time / pipe_time if pipe_time > 0 else 0,
                "batch_size": batch_size, "num_steps": num_steps}
