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

Also here: ``find_gate_module`` and ``replace_gate_with_bvh`` (:1145-1404),
which load a trained router checkpoint into a model's layer, and the hybrid
pre-filter gate (``HybridGate``, :1264-1296) that ``hybrid=True`` installs.
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


def find_gate_module(model, layer_idx: int):
    """(mlp, attribute name) of layer ``layer_idx``'s gate, walking the same
    module paths as olmoe_e2e_eval.py:1145-1174 (model.model.layers or
    model.layers; mlp or block_sparse_moe; gate or router)."""
    try:
        if hasattr(model, "model") and hasattr(model.model, "layers"):
            layer = model.model.layers[layer_idx]
        elif hasattr(model, "layers"):
            layer = model.layers[layer_idx]
        else:
            raise AttributeError("Cannot find layers attribute")
        if hasattr(layer, "mlp"):
            mlp = layer.mlp
        elif hasattr(layer, "block_sparse_moe"):
            mlp = layer.block_sparse_moe
        else:
            raise AttributeError(f"Cannot find mlp in layer {layer_idx}")
        for attr in ("gate", "router"):
            if hasattr(mlp, attr):
                return mlp, attr
        children = [a for a in dir(mlp) if not a.startswith("_") and isinstance(getattr(mlp, a, None), nn.Module)]
        raise AttributeError(f"Cannot find gate in layer {layer_idx} mlp. Module children: {children}")
    except (AttributeError, IndexError) as e:
        raise RuntimeError(f"Cannot find gate at layer {layer_idx}: {e}")


class HybridGate:
    """The hybrid pre-filter forward that replace_gate_with_bvh(hybrid=True)
    installs on a layer's dense gate (olmoe_e2e_eval.py:1264-1296): BVH top-n
    candidates, the dense gate's full fp32 softmax over all experts, top-k of
    it among the candidates, renormalised when norm_topk_prob.  One
    sb_enh_forward_hybrid call: the router kernels, the dense gate GEMM and the
    selection in the router's tail kernel.

    A plain object (not an nn.Module) so that installing its ``forward`` on
    the gate leaves the model's state_dict unchanged, as the reference's
    closure does."""

    def __init__(self, router: EnhancedBVHRouter, weight: torch.Tensor, n_candidates: int = 16,
                 top_k: int = 8, norm_topk_prob: bool = False):
        self.router = router
        self.weight = weight
        self.n_candidates = int(n_candidates)
        self.top_k = int(top_k)
        self.norm_topk_prob = bool(norm_topk_prob)
        self._gate_sig = None

    def forward(self, hidden_states: torch.Tensor):
        """(full_probs [T,E] f32, top-k weights [T,k] in the hidden dtype,
        top-k expert ids [T,k] int64)."""
        if not hidden_states.is_cuda:
            raise RuntimeError("the hybrid gate (B200) runs on CUDA tensors only")
        h2d = hidden_states.reshape(-1, self.weight.shape[1])
        eng = self.router.sync_weights(h2d.device)
        sig = (eng, self.weight.data_ptr(), self.weight._version, self.weight.device)
        if sig != self._gate_sig:
            eng.set_dense_gate(self.weight)
            self._gate_sig = sig
        out = eng.forward(h2d, precision=self.router.precision or "auto", want=(), gate="hybrid",
                          k=self.top_k, norm_topk_prob=self.norm_topk_prob, round_dtype=hidden_states.dtype,
                          n_candidates=self.n_candidates)
        return out["router_probs"], out["topk_weights"].to(hidden_states.dtype), out["topk_ids"].long()

    __call__ = forward


def _load_checkpoint(path: str):
    try:
        return torch.load(path, map_location="cpu", weights_only=True)
    except Exception:
        return torch.load(path, map_location="cpu", weights_only=False)


def replace_gate_with_bvh(model, router_checkpoint: str, layer_idx: int = 8, hybrid: bool = False,
                          n_candidates: int = 16, logit_temperature: float = None, no_calibration: bool = False,
                          logit_norm: bool = False, topk_softmax: bool = False, topk_scale: float = None,
                          weight_mode: str = "softmax", n_rays: int = 1, hybrid_alpha: float = 0.98,
                          use_optix: bool = False, selectivity_data: dict = None,
                          confidence_threshold: float = None) -> tuple:
    """Replaces layer ``layer_idx``'s gate with the trained BVH router, as
    olmoe_e2e_eval.py:1177-1404: loads the reference checkpoint format
    (``config``, ``router_state_dict``, optional ``calibration_mode`` /
    ``calibration_state`` or the older ``calibration_scale`` /
    ``calibration_bias``, ``expert_perm``).  ``hybrid=True`` keeps the gate
    module and installs the hybrid pre-filter as its forward; otherwise the
    gate is replaced by a BVHGateWrapper.  Returns (original_gate,
    original_forward or None).  Not on the B200 path: the MLP baseline router
    and spectral-mode routers (NotImplementedError); OptiX (the CUDA kernels
    serve the routing, as the reference does when its OptiX extension is
    absent); selectivity and confidence gating (stored; the wrapper's forward
    refuses them)."""
    ckpt = _load_checkpoint(router_checkpoint)
    config = ckpt["config"]
    if ckpt.get("router_type", "bvh") == "mlp":
        raise NotImplementedError("the MLP baseline router is not part of the B200 path")
    sd = ckpt["router_state_dict"]
    spectral_mode = config.get("spectral_mode", ckpt.get("spectral_mode", False)) or \
        "spectral_encoder.2.weight" in sd
    router = EnhancedBVHRouter(input_dim=config["input_dim"], n_level1=config["n_level1"],
                               n_level2=config["n_level2"], n_level3=config["n_level3"],
                               feature_dim=config["feature_dim"], spectral_mode=bool(spectral_mode))
    router.load_state_dict(sd)
    router.eval()
    mlp, gate_attr = find_gate_module(model, layer_idx)
    original_gate = getattr(mlp, gate_attr)
    try:
        gate_device = next(original_gate.parameters()).device
        if str(gate_device) == "meta":
            gate_device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    except StopIteration:
        gate_device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    router = router.to(gate_device)
    norm = getattr(original_gate, "norm_topk_prob", False)
    top_k = getattr(original_gate, "top_k", 8)
    if hybrid:
        orig_forward = original_gate.forward
        hg = HybridGate(router, original_gate.weight.data, n_candidates=n_candidates, top_k=top_k,
                        norm_topk_prob=norm)
        original_gate.forward = hg.forward
        mode_str = f"HYBRID (BVH->{n_candidates} candidates, full softmax, norm={norm})"
    else:
        orig_forward = None
        cal_mode = ckpt.get("calibration_mode", None)
        cal_state = ckpt.get("calibration_state", None)
        if cal_mode is None and "calibration_scale" in ckpt:
            cal_mode = "affine"
            cal_state = {"scale": ckpt["calibration_scale"], "bias": ckpt["calibration_bias"]}
        if cal_state is not None:
            cal_state = {k: torch.as_tensor(v).to(gate_device) for k, v in cal_state.items()}
        if no_calibration:
            cal_mode, cal_state = None, None
        wrapper = BVHGateWrapper(router, top_k=top_k, norm_topk_prob=norm, calibration_mode=cal_mode,
                                 calibration_state=cal_state, logit_temperature=logit_temperature,
                                 logit_norm=logit_norm, topk_softmax=topk_softmax, topk_scale=topk_scale,
                                 weight_mode=weight_mode, n_rays=n_rays, hybrid_alpha=hybrid_alpha).to(gate_device)
        if getattr(original_gate, "weight", None) is not None:
            wrapper._original_gate_weight = original_gate.weight.data.to(gate_device)
        perm = ckpt.get("expert_perm", None)
        if perm is not None:
            wrapper._expert_perm = torch.as_tensor(perm, dtype=torch.long, device=gate_device)
        if selectivity_data is not None:
            sel = selectivity_data.get("per_layer_selectivity", {}).get(str(layer_idx), {})
            if sel:
                wrapper._expert_selectivity = sel
                wrapper._layer_idx_for_sel = layer_idx
        if confidence_threshold is not None:
            wrapper._confidence_threshold = confidence_threshold
        if use_optix:
            print("  [WARNING] OptiX is not part of the B200 path; routing runs on the CUDA kernels")
        setattr(mlp, gate_attr, wrapper)
        mode_str = f"BVH Router (pure, calibration={cal_mode or 'none'})"
    print(f"  Replaced layer {layer_idx} gate with {mode_str}")
    return original_gate, orig_forward
