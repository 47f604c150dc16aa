"""Drop-in ``bvh_router_bridge`` for the B200 router.

Mirrors the reference's python/bvh_router_bridge.py surface that callers use:
``HAS_TORCH_EXT``, ``HAS_CUDA_ROUTER`` and ``HybridBVHRouter(cfg, device,
lib_path)`` with ``pytorch_router`` (so its state_dict keys are unchanged),
``sync_to_cuda``/``sync_to_torch_ext`` and ``forward`` (:109-429).

The reference's hybrid router switches, once synced, to its own CUDA kernel,
whose ray-sphere math differs from BVHRouter's (its route_path is even left
zero, :344-349).  Here every backend is the same B200 kernel that computes the
BVHRouter forward itself, so syncing only uploads the weights and the results
match the PyTorch router's semantics.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from bvh_router import BVHRouter, RouterConfig, RoutingResult

try:
    from sb200 import _lib as _sb_lib
    _sb_lib.load()
    HAS_TORCH_EXT = True
    HAS_CUDA_ROUTER = True
except (RuntimeError, OSError):
    HAS_TORCH_EXT = False
    HAS_CUDA_ROUTER = False


class HybridBVHRouter(nn.Module):
    def __init__(self, cfg: RouterConfig, device: torch.device = torch.device("cpu"),
                 lib_path: Optional[str] = None):
        super().__init__()
        self.cfg = cfg
        self._device = torch.device(device)
        self.pytorch_router = BVHRouter(cfg)
        self._synced = False

    def sync_to_cuda(self, batch_size: int = 1):
        """Upload the current parameters to the GPU (the reference's ctypes path)."""
        dev = self._device if self._device.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
        self.pytorch_router.sync_weights(dev)
        self._synced = True

    def sync_to_torch_ext(self):
        """Same as sync_to_cuda: there is one B200 backend."""
        self.sync_to_cuda()

    def forward(self, prompt_embedding: torch.Tensor, hard: bool = False) -> RoutingResult:
        if self.training:
            return self.pytorch_router(prompt_embedding, hard=hard)
        return self.pytorch_router(prompt_embedding, hard=True)

    def anneal_temperature(self):
        self.pytorch_router.anneal_temperature()

    def reset_expert_counts(self):
        self.pytorch_router.reset_expert_counts()

    def load_balancing_loss(self) -> torch.Tensor:
        return self.pytorch_router.load_balancing_loss()
