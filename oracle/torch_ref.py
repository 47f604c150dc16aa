"""The reference's CPU path restated in torch ops (test and baseline infrastructure only).

Only ``tests/`` and ``bench.py``'s CPU-baseline legs (``cpu_baseline`` and
``--impl reference``) use this module; the product path never does.

The numpy restatements in ``oracle/router.py`` and ``oracle/ternary.py`` are the
parity checkers.  This module is the *timed* CPU baseline: the reference runs
its MoE layer on the host as PyTorch modules, so the fair CPU number comes from
the same torch operators in the same order, on the same thread pool
(``torch.set_num_threads``), not from a numpy port.  It follows, op for op:

  * ``BVHRouter.forward``            python/bvh_router.py:269-329
      to_3d Linear, SpectralEncoder (Linear, exact-erf GELU, Linear, tanh)
      :84-97; per level: PrismaticRefraction sigmoid(Linear) :117-125,
      RouterLevel d^2 over all nodes, logits = -d^2 / (2 T^2 + 1e-8), parent
      log-mask log(repeat_interleave(p) + 1e-10), eval argmax + one_hot
      :156-204 (or, for ``soft``, the training branch with the Gumbel noise
      removed: softmax(logits / clamp(T, 0.01)) :200-202); p = p*n / (sum +
      1e-8); AffinePortal.apply_all einsum :100-114.
  * top-k convention                 python/olmoe_extract.py:105-118
      ids, vals = topk(p3, k); weights = softmax(vals).
  * ``OLMoELayer.forward_topk``      python/olmoe_extract.py:126-157
      for each slot k, for each expert in eids.unique(): the expert on the
      masked rows, out[mask] += w * y.
  * ``TernaryExpertModule.forward_hidden``  python/real_model_demo.py:379-398
      W = T.float() * s[:, None] dequantised on every call; gate/up/down
      F.linear; F.silu.

``tests/test_oracle.py`` checks these outputs against the goldens made by the
reference's own modules.
"""

from __future__ import annotations

from typing import Dict, Sequence

import numpy as np
import torch
import torch.nn.functional as F


def _t(a) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32)))


class TorchRouter:
    """BVHRouter eval forward (and the noiseless soft branch) in torch fp32."""

    def __init__(self, w: Dict[str, np.ndarray], branching: Sequence[int] = (4, 4, 4)):
        self.branching = tuple(int(b) for b in branching)
        self.L = len(self.branching)
        self.w = {k: _t(v) for k, v in w.items()}
        self.T = self.w["temperature"].reshape(())

    def level(self, l: int, pos: torch.Tensor, parent: torch.Tensor, soft: bool):
        c = self.w[f"level{l}.centers"]
        diff = pos.unsqueeze(1) - c.unsqueeze(0)
        d_sq = (diff ** 2).sum(dim=-1)
        logits = -d_sq / (2.0 * self.T ** 2 + 1e-8)
        if parent is not None:
            logits = logits + torch.log(parent.repeat_interleave(self.branching[l - 1], dim=1) + 1e-10)
        if soft:
            probs = F.softmax(logits / self.T.clamp(min=0.01), dim=-1)
            choice = probs.argmax(dim=-1)
        else:
            choice = logits.argmax(dim=-1)
            probs = F.one_hot(choice, c.shape[0]).float()
        return probs, choice

    def forward(self, x: torch.Tensor, soft: bool = False):
        w = self.w
        pos = F.linear(x, w["to_3d.weight"], w["to_3d.bias"])
        g = F.gelu(F.linear(x, w["spectral.net.0.weight"], w["spectral.net.0.bias"]))
        spec = torch.tanh(F.linear(g, w["spectral.net.2.weight"], w["spectral.net.2.bias"]))
        p, path = None, []
        for l in range(1, self.L + 1):
            n = torch.sigmoid(F.linear(spec, w[f"refract{l}.W_dispersion.weight"],
                                       w[f"refract{l}.W_dispersion.bias"]))
            pl, cl = self.level(l, pos, p, soft)
            pl = pl * n
            pl = pl / (pl.sum(dim=-1, keepdim=True) + 1e-8)
            path.append(cl)
            if l < self.L:
                A = w[f"portal{l}.transform"]
                pos_h = torch.cat([pos, torch.ones(pos.shape[0], 1)], dim=-1)
                pos = (torch.einsum("kij,bj->bki", A, pos_h) * pl.unsqueeze(-1)).sum(dim=1)
            p = pl
        return p, torch.stack(path, dim=-1)

    def topk(self, x: torch.Tensor, k: int = 8, soft: bool = True):
        p, _ = self.forward(x, soft=soft)
        vals, ids = p.topk(k, dim=-1)
        return F.softmax(vals, dim=-1), ids


class TorchTernaryExpert:
    """TernaryExpertModule (int8 weights + per-row scales, dequantised per call)."""

    def __init__(self, ex: Dict[str, np.ndarray]):
        self.gate_t = torch.from_numpy(np.ascontiguousarray(ex["gate_ternary"]))
        self.up_t = torch.from_numpy(np.ascontiguousarray(ex["up_ternary"]))
        self.down_t = torch.from_numpy(np.ascontiguousarray(ex["down_ternary"]))
        self.gate_s, self.up_s, self.down_s = _t(ex["gate_scale"]), _t(ex["up_scale"]), _t(ex["down_scale"])

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x = x.float()
        gate_w = self.gate_t.float() * self.gate_s.unsqueeze(1)
        up_w = self.up_t.float() * self.up_s.unsqueeze(1)
        hidden = F.silu(F.linear(x, gate_w)) * F.linear(x, up_w)
        down_w = self.down_t.float() * self.down_s.unsqueeze(1)
        return F.linear(hidden, down_w)


def forward_topk(x: torch.Tensor, probs: torch.Tensor, ids: torch.Tensor, experts) -> torch.Tensor:
    """OLMoELayer.forward_topk: slot by slot, expert by expert, out[mask] += w * y."""
    out = torch.zeros_like(x)
    for ki in range(ids.shape[-1]):
        eids, weights = ids[:, ki], probs[:, ki]
        for eid in eids.unique():
            mask = eids == eid
            if not mask.any():
                continue
            out[mask] += weights[mask].unsqueeze(-1) * experts[int(eid)](x[mask])
    return out


class TorchMoELayer:
    """Router top-k (soft selection) + ternary experts, the reference's CPU layer."""

    def __init__(self, router_w, experts, branching=(4, 4, 4), k: int = 8, soft: bool = True):
        self.router = TorchRouter(router_w, branching)
        self.experts = [TorchTernaryExpert(e) for e in experts]
        self.k, self.soft = int(k), bool(soft)

    @torch.no_grad()
    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        probs, ids = self.router.topk(x, self.k, self.soft)
        return forward_topk(x, probs, ids, self.experts)
