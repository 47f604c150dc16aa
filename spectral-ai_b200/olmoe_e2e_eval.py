"""Drop-in ``olmoe_e2e_eval.BVHGateWrapper`` for the B200 enhanced router.

Mirrors python/olmoe_e2e_eval.py:226-971 of the reference for the weight
conventions the OLMoE layer uses by default:
  * weight_mode "softmax" (:928-938): router_probs = softmax(logits) over all
    experts, top-k of it, renormalised when norm_topk_prob;
  * weight_mode "topk_softmax" / topk_softmax=True (:521-529): softmax over
    the top-k logits, scaled by topk_scale, scattered into router_probs;
after the logits are rounded to the hidden-state dtype (:380).  The
calibration transforms ("affine", "topk_preserving", "linear"; :371-378) and
the expert permutation (:385-387) act on the logits before that rounding and
are folded into the expert head's last layer, so the whole gate is the three
sb_enh kernels.  The experimental weight modes, logit temperature / LogitNorm,
confidence gating and the OptiX path are not part of this inference path and
raise.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from olmoe_bvh_distill import EnhancedBVHRouter
from sb200.enhanced import EnhancedEngine

_SUPPORTED_MODES = ("softmax", "topk_softmax")


class BVHGateWrapper(nn.Module):
    def __init__(self, router: EnhancedBVHRouter, top_k: int = 8, norm_topk_prob: bool = False,
                 calibration_mode: str = None, calibration_state: dict = None,
                 logit_temperature: float = None, logit_norm: bool = False, topk_softmax: bool = False,
                 topk_scale: float = None, weight_mode: str = "softmax", n_rays: int = 1,
                 hybrid_alpha: float = 0.98):
        super().__init__()
        self.router = router
        self.router.eval()
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.calibration_mode = calibration_mode
        self.logit_temperature = logit_temperature
        self.logit_norm = logit_norm
        self.n_rays = n_rays
        self.hybrid_alpha = hybrid_alpha
        self.weight_mode = "topk_softmax" if (topk_softmax and weight_mode == "softmax") else weight_mode
        self.topk_scale = topk_scale
        self._expert_perm = None
        self._original_gate_weight = None
        self._confidence_threshold = None
        self._optix_bridge = None
        if calibration_mode == "affine" and calibration_state is not None:
            self.register_buffer("cal_scale", calibration_state["scale"])
            self.register_buffer("cal_bias", calibration_state["bias"])
        elif calibration_mode == "topk_preserving" and calibration_state is not None:
            self.register_buffer("cal_inv_temp", calibration_state.get("inv_temp", torch.ones(1)))
            self.register_buffer("cal_bias", calibration_state["bias"])
        elif calibration_mode == "linear" and calibration_state is not None:
            n = int(calibration_state["weight"].shape[0])
            self.cal_linear = nn.Linear(n, n)
            self.cal_linear.load_state_dict(calibration_state)
            self.cal_linear.eval()
        elif calibration_mode is not None and calibration_state is not None:
            raise NotImplementedError(f"calibration mode {calibration_mode!r}")
        self.weight = nn.Parameter(torch.empty(0), requires_grad=False)
        self._engine: Optional[EnhancedEngine] = None
        self._engine_device = None
        self._synced = None

    def _check_supported(self):
        if self.weight_mode not in _SUPPORTED_MODES:
            raise NotImplementedError(f"weight mode {self.weight_mode!r} is not part of the B200 inference path "
                                      f"(supported: {', '.join(_SUPPORTED_MODES)})")
        if self.logit_temperature is not None or self.logit_norm:
            raise NotImplementedError("logit temperature / LogitNorm are not part of the B200 inference path")
        if self._confidence_threshold is not None or (self._optix_bridge is not None
                                                      and getattr(self._optix_bridge, "available", False)):
            raise NotImplementedError("confidence gating / OptiX routing are not part of the B200 path")
        if self.n_rays != 1:
            raise NotImplementedError("the multi-ray ensemble is not part of the B200 path")

    def _folded_state(self):
        """The router's parameters with the calibration and expert permutation
        folded into expert_head.2 (logits = W u + b -> transformed logits)."""
        sd = dict(self.router.state_dict())
        W = sd["expert_head.2.weight"].detach().float().clone()
        b = sd["expert_head.2.bias"].detach().float().clone()
        E = W.shape[0]
        if self.calibration_mode in ("affine", "topk_preserving") and hasattr(self, "cal_bias"):
            s = (self.cal_scale if self.calibration_mode == "affine" else self.cal_inv_temp).detach().float()
            s = s.to(W.device).expand(E)
            W = W * s[:, None]
            b = b * s + self.cal_bias.detach().float().to(W.device).expand(E)
        elif self.calibration_mode == "linear" and hasattr(self, "cal_linear"):
            Wc = self.cal_linear.weight.detach().float().to(W.device)
            W = Wc @ W
            b = Wc @ b + self.cal_linear.bias.detach().float().to(W.device)
        if self._expert_perm is not None:
            inv = torch.argsort(self._expert_perm.to(W.device))
            W, b = W[inv], b[inv]
        sd["expert_head.2.weight"], sd["expert_head.2.bias"] = W, b
        return sd

    def _signature(self):
        sig = [(n, t.data_ptr(), t._version) for n, t in
               list(self.router.named_parameters()) + list(self.router.named_buffers()) if n != "expert_counts"]
        sig += [(n, t.data_ptr(), t._version) for n, t in self.named_buffers(recurse=False)]
        if hasattr(self, "cal_linear"):
            sig += [(n, t.data_ptr(), t._version) for n, t in self.cal_linear.named_parameters()]
        perm = self._expert_perm
        sig.append(None if perm is None else (perm.data_ptr(), perm._version))
        return tuple(sig)

    def _engine_for(self, device) -> EnhancedEngine:
        if self._engine is None or self._engine_device != device:
            r = self.router
            self._engine = EnhancedEngine(r.input_dim, r.feature_dim, (r.n_level1, r.n_level2, r.n_level3), device)
            self._engine_device = device
            self._synced = None
        sig = self._signature()
        if sig != self._synced:
            self._engine.upload(self._folded_state())
            self._synced = sig
        return self._engine

    def forward(self, hidden_states: torch.Tensor):
        """(router_logits-as-probs [T,E] f32, top_k_weights [T,k] hidden dtype,
        top_k_index [T,k] int64) like OlmoeTopKRouter (olmoe_e2e_eval.py:316-971)."""
        self._check_supported()
        if not hidden_states.is_cuda:
            raise RuntimeError("BVHGateWrapper (B200) runs on CUDA tensors only")
        h2d = hidden_states.reshape(-1, hidden_states.shape[-1])
        eng = self._engine_for(h2d.device)
        out = eng.forward(h2d, precision=self.router.precision or "auto", want=(),
                          gate=self.weight_mode, k=self.top_k, norm_topk_prob=self.norm_topk_prob,
                          round_dtype=hidden_states.dtype)
        probs, w, ids = out["router_probs"], out["topk_weights"], out["topk_ids"].long()
        if self.weight_mode == "topk_softmax" and self.topk_scale is not None:
            w = w * self.topk_scale
            probs = probs * self.topk_scale
        return probs, w.to(hidden_states.dtype), ids
