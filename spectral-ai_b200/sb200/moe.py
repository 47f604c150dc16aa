"""The MoE layer of the hot path: BVH router top-k -> grouped ternary SwiGLU.

``BVHMoELayer.forward(x)`` = router top-k (``BVHRouter.forward_topk``) followed by
``sum_j w[t,j] * expert_{ids[t,j]}(x[t])`` over ternary experts, i.e. the
composition the reference runs as ``BVHGateWrapper`` + the Python dispatch loop
of ``OLMoELayer.forward_topk`` (python/olmoe_extract.py:126-157) over
``CUDATernaryExpertModule`` experts (python/ternary_expert_ext_bridge.py:75-175).
Everything runs on the device: no host round trip between routing and experts.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch

from .ternary import TernaryExperts


class BVHMoELayer:
    def __init__(self, router, experts, top_k: int = 8, select: str = "soft",
                 device: Optional[torch.device] = None):
        """router: a ``bvh_router.BVHRouter`` (on ``device``); experts: a
        ``TernaryExperts`` or a sequence of expert containers."""
        self.router = router
        self.device = torch.device(device) if device is not None else router.to_3d.weight.device
        self.experts = experts if isinstance(experts, TernaryExperts) else TernaryExperts(experts, self.device)
        self.top_k = int(top_k)
        self.select = select

    def route(self, x: torch.Tensor):
        return self.router.forward_topk(x, k=self.top_k, select=self.select)

    def forward(self, x: torch.Tensor, out_dtype=None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        ids, w = self.route(x)
        return self.experts.forward(x, ids, w, out_dtype=out_dtype or x.dtype, out=out)

    __call__ = forward

    def forward_topk(self, hidden_states: torch.Tensor, topk_probs: torch.Tensor,
                     topk_ids: torch.Tensor) -> torch.Tensor:
        """Same signature as OLMoELayer.forward_topk (olmoe_extract.py:126-157)."""
        return self.experts.forward(hidden_states, topk_ids, topk_probs, out_dtype=hidden_states.dtype)


class GraphedLayer:
    """A layer replayed from CUDA graphs: the first call with a given
    (input, output) buffer pair runs the layer twice to warm every cached
    workspace and kernel attribute, then captures one forward into a graph;
    later calls with the same buffers replay it on the current stream (one
    launch instead of the layer's eight, no per-kernel launch gaps).

    Valid while the buffers, the batch shape and the layer's weights stay in
    place: a weight re-upload that moves device memory needs ``reset()``.
    Calls with new buffers capture another graph (up to ``max_graphs``).
    """

    def __init__(self, layer, max_graphs: int = 8):
        self.layer = layer
        self.max_graphs = int(max_graphs)
        self._graphs = {}

    def reset(self) -> None:
        self._graphs.clear()

    def _key(self, x: torch.Tensor, out: torch.Tensor):
        return (x.data_ptr(), tuple(x.shape), x.dtype, out.data_ptr(), tuple(out.shape), out.dtype)

    def __call__(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        key = self._key(x, out)
        g = self._graphs.get(key)
        if g is None:
            if len(self._graphs) >= self.max_graphs:
                self._graphs.pop(next(iter(self._graphs)))
            cur = torch.cuda.current_stream(x.device)
            side = torch.cuda.Stream(x.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                for _ in range(2):
                    self.layer(x, out=out)
            cur.wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                self.layer(x, out=out)
            cur.wait_stream(side)
            self._graphs[key] = g
        g.replay()
        return out


class HostPipeline:
    """Runs a stream of host-resident batches through a layer with the copies
    overlapped: while the layer computes batch i on the compute stream, batch
    i+1 is copied in on one copy stream and batch i-1's result copied out on
    another (two device buffers each way).  Every batch still makes its full
    host->device and device->host trip; only their timing overlaps.

    ``layer`` is any callable ``layer(x_dev, out=y_dev)`` on the device, such as
    ``BVHMoELayer``.  Host tensors should be pinned for the copies to be
    asynchronous.
    """

    def __init__(self, layer, batch: int, hidden: int, dtype=torch.bfloat16,
                 device: Optional[torch.device] = None, out_dtype=None):
        self.layer = layer
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.xin = [torch.empty(batch, hidden, dtype=dtype, device=self.device) for _ in range(2)]
        self.yout = [torch.empty(batch, hidden, dtype=out_dtype or dtype, device=self.device) for _ in range(2)]
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        ev = lambda: [torch.cuda.Event() for _ in range(2)]
        self.in_ready, self.in_free, self.out_ready, self.out_free = ev(), ev(), ev(), ev()

    def run(self, inputs: Sequence[torch.Tensor], outputs: Sequence[torch.Tensor]) -> None:
        """outputs[i] <- layer(inputs[i]) for every i; returns when all copies are queued
        (synchronise the current stream, or wait on ``done_event``, to read them)."""
        compute = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(compute)
        self.h2d.wait_event(start)
        self.d2h.wait_event(start)
        for i, (xh, yh) in enumerate(zip(inputs, outputs)):
            b = i & 1
            with torch.cuda.stream(self.h2d):
                if i >= 2:
                    self.h2d.wait_event(self.in_free[b])   # compute of batch i-2 has read xin[b]
                self.xin[b].copy_(xh, non_blocking=True)
                self.in_ready[b].record(self.h2d)
            compute.wait_event(self.in_ready[b])
            if i >= 2:
                compute.wait_event(self.out_free[b])       # batch i-2's result has left yout[b]
            self.layer(self.xin[b], out=self.yout[b])
            self.in_free[b].record(compute)
            self.out_ready[b].record(compute)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.out_ready[b])
                yh.copy_(self.yout[b], non_blocking=True)
                self.out_free[b].record(self.d2h)
        # the caller's stream is done when the last copy out is
        last = (len(inputs) - 1) & 1 if len(inputs) else 0
        if len(inputs):
            compute.wait_event(self.out_free[last])
            if len(inputs) > 1:
                compute.wait_event(self.out_free[last ^ 1])
