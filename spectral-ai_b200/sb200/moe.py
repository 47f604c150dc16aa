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
