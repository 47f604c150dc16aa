"""Drop-in ``olmoe_bvh_distill`` for the B200 enhanced router.

Mirrors the inference surface of the reference's python/olmoe_bvh_distill.py:
``HierarchicalLevel`` (:324-419) and ``EnhancedBVHRouter`` (:422-640) with the
same submodule names, so state_dicts load unchanged.  The eval forward
(``forward(x, n_rays=1)`` -> ``(expert_probs, expert_ids)``, with the side
attributes ``_last_logits``, ``_last_geometric_distances`` and
``_last_branch_bonus``) runs as three kernels of libspectral_b200.so
(``sb_enh_*``).  Not part of this inference path: the distillation training
loop, spectral_mode (SmoothBVHHit / RT bridge / spectral gate), the
multi-ray ensemble (its noise is unseeded) and the training-mode
Gumbel-softmax forward; they raise.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from sb200.enhanced import EnhancedEngine

_CPU_MSG = "EnhancedBVHRouter (B200) runs on CUDA tensors only; move the input to a GPU"


class HierarchicalLevel(nn.Module):
    """Parameters of one level (olmoe_bvh_distill.py:340-365, spectral_mode off)."""

    def __init__(self, input_dim: int, n_children: int, feature_dim: int = 128, spectral_mode: bool = False):
        super().__init__()
        if spectral_mode:
            raise NotImplementedError("spectral_mode (SmoothBVHHit) is not part of the B200 inference path")
        self.n_children = n_children
        self.feature_dim = feature_dim
        self.spectral_mode = False
        self.to_3d = nn.Linear(input_dim, 3)
        self.centers = nn.Parameter(torch.randn(n_children, 3) * 0.3)
        self.log_radii = nn.Parameter(torch.zeros(n_children))
        self.feature_net = nn.Sequential(nn.Linear(input_dim, feature_dim), nn.GELU(),
                                         nn.Linear(feature_dim, feature_dim))
        self.route_head = nn.Linear(feature_dim + 3, n_children)


class EnhancedBVHRouter(nn.Module):
    """Same constructor and state_dict as the reference (olmoe_bvh_distill.py:438-516)."""

    def __init__(self, input_dim: int = 2048, n_level1: int = 4, n_level2: int = 4, n_level3: int = 4,
                 feature_dim: int = 128, temperature_init: float = 1.0, spectral_mode: bool = False,
                 spectral_dim: int = 64, encoder_hidden: int = None):
        super().__init__()
        if spectral_mode:
            raise NotImplementedError("spectral_mode is not part of the B200 inference path")
        self.input_dim = input_dim
        self.n_level1, self.n_level2, self.n_level3 = n_level1, n_level2, n_level3
        self.n_experts = n_level1 * n_level2 * n_level3
        self.feature_dim = feature_dim
        self.spectral_mode = False
        self.spectral_enabled = False
        self.input_proj = nn.Sequential(nn.Linear(input_dim, 512), nn.GELU(), nn.Linear(512, 256),
                                        nn.LayerNorm(256))
        self.level1 = HierarchicalLevel(256, n_level1, feature_dim)
        self.level2 = HierarchicalLevel(feature_dim, n_level2, feature_dim)
        self.level3 = HierarchicalLevel(feature_dim, n_level3, feature_dim)
        head_input_dim = feature_dim + n_level1 + n_level2 + n_level3
        self.expert_head = nn.Sequential(nn.Linear(head_input_dim, 256), nn.GELU(),
                                         nn.Linear(256, self.n_experts))
        self.register_buffer("temperature", torch.tensor(temperature_init))
        self.register_buffer("expert_counts", torch.zeros(self.n_experts))
        self.precision: Optional[str] = None  # "fast" | "exact" | None (from the input dtype)
        self._engine: Optional[EnhancedEngine] = None
        self._engine_device = None
        self._synced = None

    # ---- device engine
    def _param_signature(self):
        return tuple((n, t.data_ptr(), t._version) for n, t in
                     list(self.named_parameters()) + list(self.named_buffers()) if n != "expert_counts")

    def sync_weights(self, device=None) -> EnhancedEngine:
        """Uploads the current parameters to the device (done automatically on change)."""
        device = torch.device(device) if device is not None else self.level1.centers.device
        if device.type != "cuda":
            raise RuntimeError(_CPU_MSG)
        if self._engine is None or self._engine_device != device:
            self._engine = EnhancedEngine(self.input_dim, self.feature_dim,
                                          (self.n_level1, self.n_level2, self.n_level3), device)
            self._engine_device = device
            self._synced = None
        sig = self._param_signature()
        if sig != self._synced:
            self._engine.upload(self.state_dict())
            self._synced = sig
        return self._engine

    def route(self, x: torch.Tensor, precision: Optional[str] = None,
              want=("logits", "expert_probs", "expert_ids", "geo_dist", "branch_bonus"), **gate):
        """All outputs as a dict; ``gate=...`` adds the BVHGateWrapper top-k."""
        if not isinstance(x, torch.Tensor) or not x.is_cuda:
            raise RuntimeError(_CPU_MSG)
        eng = self.sync_weights(x.device)
        return eng.forward(x, precision=precision or self.precision or "auto", want=want, **gate)

    def forward(self, x: torch.Tensor, n_rays: int = 1) -> Tuple[torch.Tensor, torch.Tensor]:
        """(expert_probs [B,E], expert_ids [B]) — olmoe_bvh_distill.py:593-632, eval."""
        if self.training:
            raise NotImplementedError("the training-mode Gumbel-softmax forward is not part of the B200 "
                                      "inference path; call .eval()")
        if n_rays != 1:
            raise NotImplementedError("the multi-ray ensemble (unseeded noise) is not part of the B200 path")
        out = self.route(x)
        self._last_logits = out["logits"]
        self._last_geometric_distances = out["geo_dist"]
        self._last_branch_bonus = out["branch_bonus"]
        return out["expert_probs"], out["expert_ids"]

    def anneal_temperature(self, decay: float = 0.95):
        new_temp = max(0.1, self.temperature.item() * decay)
        self.temperature.fill_(new_temp)

    def reset_expert_counts(self):
        self.expert_counts.zero_()

    def load_balancing_loss(self) -> torch.Tensor:
        total = self.expert_counts.sum()
        if total < 1:
            return torch.tensor(0.0, device=self.expert_counts.device)
        usage = self.expert_counts / total
        target = 1.0 / self.n_experts
        return ((usage - target) ** 2).sum()
