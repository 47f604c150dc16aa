"""Drop-in ``bvh_router`` module backed by the B200 router kernels.

Same import name, classes, constructor arguments, submodule names and
``state_dict`` keys as the reference python/bvh_router.py (RouterConfig
:28-65, RoutingResult :72-77, SpectralEncoder :84-97, AffinePortal :100-114,
PrismaticRefraction :117-125, RouterLevel :132-204, BVHRouter :211-329), so a
checkpoint saved from the reference loads unchanged and callers keep their
imports.  The forward runs hand-written sm_100a CUDA through
libspectral_b200.so:

  * eval mode, or ``hard=True``   -> the reference eval branch (argmax + one_hot),
  * bf16 input                    -> bf16 tcgen05 encoder GEMMs (FAST),
  * fp32 input                    -> fp32 FFMA encoder GEMMs (EXACT),
  * CPU input                     -> RuntimeError (there is no CPU path).

The training-mode Gumbel-softmax forward is not part of this inference path
and raises.  ``RouterConfig`` accepts an optional ``branching`` tuple that
generalises the three hard-coded levels to L levels (levels 1..L-1 carry
portals); with the default it is the reference's 3-level router.
"""

from __future__ import annotations

import math
from typing import NamedTuple, Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from sb200.router import RouterEngine


class RouterConfig:
    """Router hyper-parameters (python/bvh_router.py:28-65)."""

    __slots__ = (
        'embed_dim', 'spectral_dim',
        'n_level1', 'n_level2', 'n_level3',
        'total_l1', 'total_l2', 'total_l3',
        'n_experts',
        'temperature_init', 'temperature_min', 'temperature_decay',
        'gumbel_hard', 'dropout', 'branching',
    )

    def __init__(self, embed_dim: int = 256, spectral_dim: int = 64, n_level1: int = 4,
                 n_level2: int = 4, n_level3: int = 4, temperature_init: float = 1.0,
                 temperature_min: float = 0.1, temperature_decay: float = 0.95,
                 gumbel_hard: bool = False, dropout: float = 0.1,
                 branching: Optional[Sequence[int]] = None):
        self.embed_dim = embed_dim
        self.spectral_dim = spectral_dim
        if branching is None:
            branching = (n_level1, n_level2, n_level3)
        self.branching = tuple(int(b) for b in branching)
        b = self.branching + (1, 1, 1)
        self.n_level1, self.n_level2, self.n_level3 = b[0], b[1], b[2]
        self.total_l1 = self.n_level1
        self.total_l2 = self.n_level1 * self.n_level2
        self.total_l3 = self.n_level1 * self.n_level2 * self.n_level3
        self.n_experts = math.prod(self.branching)
        self.temperature_init = temperature_init
        self.temperature_min = temperature_min
        self.temperature_decay = temperature_decay
        self.gumbel_hard = gumbel_hard
        self.dropout = dropout

    @property
    def n_levels(self) -> int:
        return len(self.branching)

    def level_sizes(self):
        out, n = [], 1
        for b in self.branching:
            n *= b
            out.append(n)
        return out


class RoutingResult(NamedTuple):
    """Router result (python/bvh_router.py:72-77)."""
    expert_id: torch.Tensor
    expert_probs: torch.Tensor
    route_path: torch.Tensor
    confidence: torch.Tensor


class SpectralEncoder(nn.Module):
    """Linear(H,H) -> GELU -> Linear(H,S) -> Tanh (python/bvh_router.py:84-97)."""

    def __init__(self, embed_dim: int, spectral_dim: int = 64):
        super().__init__()
        self.net = nn.Sequential(nn.Linear(embed_dim, embed_dim), nn.GELU(),
                                 nn.Linear(embed_dim, spectral_dim), nn.Tanh())

    def forward(self, context: torch.Tensor) -> torch.Tensor:
        return self.net(context)


class AffinePortal(nn.Module):
    """Per-node 3x4 affine transform, identity at init (python/bvh_router.py:100-114)."""

    def __init__(self, n_portals: int):
        super().__init__()
        eye = torch.zeros(n_portals, 3, 4)
        for i in range(3):
            eye[:, i, i] = 1.0
        self.transform = nn.Parameter(eye)

    def apply_all(self, pos_3d: torch.Tensor) -> torch.Tensor:
        ones = torch.ones(*pos_3d.shape[:-1], 1, device=pos_3d.device, dtype=pos_3d.dtype)
        return torch.einsum('kij,bj->bki', self.transform, torch.cat([pos_3d, ones], dim=-1))


class PrismaticRefraction(nn.Module):
    """n = sigmoid(W spec + b) (python/bvh_router.py:117-125)."""

    def __init__(self, n_spheres: int, spectral_dim: int):
        super().__init__()
        self.W_dispersion = nn.Linear(spectral_dim, n_spheres)

    def forward(self, spectral: torch.Tensor) -> torch.Tensor:
        return torch.sigmoid(self.W_dispersion(spectral))


class RouterLevel(nn.Module):
    """Parameters of one level (python/bvh_router.py:132-154); the level math
    runs inside the fused descent kernel."""

    def __init__(self, n_spheres: int, parent_spheres: int = 1):
        super().__init__()
        self.n_spheres = n_spheres
        self.parent_spheres = parent_spheres
        total = parent_spheres * n_spheres
        self.centers = nn.Parameter(torch.randn(total, 3) * 0.5)
        self.log_radii = nn.Parameter(torch.zeros(total))

    @property
    def radii(self) -> torch.Tensor:
        return F.softplus(self.log_radii)


class BVHRouter(nn.Module):
    """Hierarchical BVH router (python/bvh_router.py:211-329) on B200."""

    def __init__(self, cfg: RouterConfig):
        super().__init__()
        self.cfg = cfg
        sizes = cfg.level_sizes()
        L = len(sizes)
        self.to_3d = nn.Linear(cfg.embed_dim, 3)
        self.spectral = SpectralEncoder(cfg.embed_dim, cfg.spectral_dim)
        parent = 1
        for l in range(L):
            setattr(self, f"level{l + 1}", RouterLevel(cfg.branching[l], parent_spheres=parent))
            if l < L - 1:
                setattr(self, f"portal{l + 1}", AffinePortal(sizes[l]))
            setattr(self, f"refract{l + 1}", PrismaticRefraction(sizes[l], cfg.spectral_dim))
            parent = sizes[l]
        self.register_buffer('temperature', torch.tensor(cfg.temperature_init))
        self.register_buffer('expert_counts', torch.zeros(cfg.n_experts))
        self._engine: Optional[RouterEngine] = None
        self._engine_device = None
        self._synced = None
        self.precision = "auto"   # "auto" | "fast" | "exact"

    # -- reference bookkeeping (python/bvh_router.py:257-267, 331-345) ----------------
    def anneal_temperature(self):
        new_temp = max(self.cfg.temperature_min, self.temperature.item() * self.cfg.temperature_decay)
        self.temperature.fill_(new_temp)

    def reset_expert_counts(self):
        self.expert_counts.zero_()

    def load_balancing_loss(self) -> torch.Tensor:
        total = self.expert_counts.sum()
        if total < 1:
            return torch.tensor(0.0, device=self.expert_counts.device)
        usage = self.expert_counts / total
        target = 1.0 / self.cfg.n_experts
        return ((usage - target) ** 2).sum()

    # -- B200 engine -------------------------------------------------------------------
    def _param_signature(self):
        return tuple((n, t.data_ptr(), t._version) for n, t in
                     list(self.named_parameters()) + [("temperature", self.temperature)])

    def sync_weights(self, device=None) -> RouterEngine:
        """Uploads the current parameters to the device (done automatically on change)."""
        device = torch.device(device) if device is not None else self.to_3d.weight.device
        if device.type != "cuda":
            raise RuntimeError("BVHRouter (B200) runs on CUDA tensors only; move the input to a GPU")
        if self._engine is None or self._engine_device != device:
            self._engine = RouterEngine(self.cfg.embed_dim, self.cfg.spectral_dim,
                                        self.cfg.branching, device)
            self._engine_device = device
            self._synced = None
        sig = self._param_signature()
        if sig != self._synced:
            self._engine.upload(self.state_dict())
            self._synced = sig
        return self._engine

    def route(self, x: torch.Tensor, select: str = "hard", k: int = 0, precision: Optional[str] = None,
              want=("expert_id", "expert_probs", "route_path", "confidence")):
        """All router outputs as a dict (``select`` = "hard" | "soft")."""
        if not isinstance(x, torch.Tensor) or not x.is_cuda:
            raise RuntimeError("BVHRouter (B200) runs on CUDA tensors only; move the input to a GPU")
        eng = self.sync_weights(x.device)
        return eng.forward(x, precision=precision or self.precision, select=select, k=k, want=want)

    def forward(self, prompt_embedding: torch.Tensor, hard: bool = False) -> RoutingResult:
        use_hard = hard or not self.training
        if not use_hard:
            raise NotImplementedError(
                "the training-mode Gumbel-softmax forward is not part of the B200 inference "
                "path; call eval() or pass hard=True")
        r = self.route(prompt_embedding, select="hard")
        if self.training:   # reference updates the balance counters in training mode (:317-319)
            self.expert_counts.index_add_(0, r["expert_id"].to(self.expert_counts.device),
                                          torch.ones_like(r["expert_id"], dtype=self.expert_counts.dtype,
                                                          device=self.expert_counts.device))
        return RoutingResult(expert_id=r["expert_id"], expert_probs=r["expert_probs"],
                             route_path=r["route_path"], confidence=r["confidence"])

    def forward_topk(self, x: torch.Tensor, k: int = 8, select: str = "hard") -> Tuple[torch.Tensor, torch.Tensor]:
        """Top-k expert ids (int32 [B,k]) and softmax weights (fp32 [B,k]) for the MoE layer."""
        r = self.route(x, select=select, k=k, want=())
        return r["topk_ids"], r["topk_weights"]


class BranchSpecificBVHRouter(nn.Module):
    """Not provided by the B200 hot path (reference variant, python/bvh_router.py:348-492)."""

    def __init__(self, *a, **kw):
        raise NotImplementedError("BranchSpecificBVHRouter is outside the B200 hot path")
