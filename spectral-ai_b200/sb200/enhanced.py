"""Torch-facing wrapper of the C-ABI enhanced router handle (sb_enh_*).

``EnhancedEngine`` owns one ``sb_enh`` handle per device: the
EnhancedBVHRouter eval forward (python/olmoe_bvh_distill.py:422-632) and the
BVHGateWrapper "softmax" / "topk_softmax" weights (python/olmoe_e2e_eval.py:316-971)
in three kernels on the current stream, and the hybrid pre-filter gate of
replace_gate_with_bvh(hybrid=True) (python/olmoe_e2e_eval.py:1264-1296) with one
more GEMM for the layer's dense gate.  Outputs are ``torch.empty`` on the
input's device.
"""

from __future__ import annotations

import ctypes as C
from typing import Dict, Mapping, Optional, Sequence

import numpy as np
import torch

from . import _lib

PRECISIONS = {"fast": _lib.SB_PREC_FAST, "exact": _lib.SB_PREC_EXACT}
GATE_MODES = {"softmax": _lib.SB_GATE_SOFTMAX, "topk_softmax": _lib.SB_GATE_TOPK_SOFTMAX}
OUTPUTS = ("logits", "expert_probs", "expert_ids", "geo_dist", "branch_bonus", "router_probs",
           "topk_weights", "topk_ids")


class EnhancedEngine:
    """One enhanced-router handle on one CUDA device."""

    def __init__(self, hidden: int, feature: int, branching: Sequence[int], device):
        self.lib = _lib.load()
        self.hidden, self.feature = int(hidden), int(feature)
        self.branching = tuple(int(b) for b in branching)
        if len(self.branching) != 3:
            raise RuntimeError("the enhanced router has exactly three levels")
        self.n_experts = int(np.prod(self.branching))
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("EnhancedEngine needs a CUDA device (there is no CPU path)")
        desc = _lib.EnhDesc()
        desc.hidden, desc.feature = self.hidden, self.feature
        for i, b in enumerate(self.branching):
            desc.branching[i] = b
        self.dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        h = C.c_void_p()
        _lib.check(self.lib.sb_enh_create(C.byref(desc), self.dev_index, C.byref(h)), "sb_enh_create")
        self.handle = h
        self._ws: Optional[torch.Tensor] = None

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                self.lib.sb_enh_destroy(h)
            except Exception:
                pass
            self.handle = None

    def upload(self, params: Mapping[str, object]) -> None:
        """params: EnhancedBVHRouter state_dict names -> tensors/arrays."""
        keep = []

        def ptr(name, required=True):
            v = params.get(name)
            if v is None:
                if required:
                    raise KeyError(name)
                return None
            if isinstance(v, torch.Tensor):
                a = v.detach().to("cpu", torch.float32).contiguous().numpy()
            else:
                a = np.ascontiguousarray(np.asarray(v, np.float32))
            keep.append(a)
            return a.ctypes.data

        w = _lib.EnhWeights()
        w.in0_w, w.in0_b = ptr("input_proj.0.weight"), ptr("input_proj.0.bias", False)
        w.in2_w, w.in2_b = ptr("input_proj.2.weight"), ptr("input_proj.2.bias", False)
        w.ln_w, w.ln_b = ptr("input_proj.3.weight", False), ptr("input_proj.3.bias", False)
        for l in range(3):
            n = f"level{l + 1}"
            lv = w.level[l]
            lv.centers = ptr(f"{n}.centers")
            lv.to3d_w, lv.to3d_b = ptr(f"{n}.to_3d.weight"), ptr(f"{n}.to_3d.bias", False)
            lv.feat0_w, lv.feat0_b = ptr(f"{n}.feature_net.0.weight"), ptr(f"{n}.feature_net.0.bias", False)
            lv.feat2_w, lv.feat2_b = ptr(f"{n}.feature_net.2.weight"), ptr(f"{n}.feature_net.2.bias", False)
            lv.head_w, lv.head_b = ptr(f"{n}.route_head.weight"), ptr(f"{n}.route_head.bias", False)
        w.eh0_w, w.eh0_b = ptr("expert_head.0.weight"), ptr("expert_head.0.bias", False)
        w.eh2_w, w.eh2_b = ptr("expert_head.2.weight"), ptr("expert_head.2.bias", False)
        t = params.get("temperature", 1.0)
        w.temperature = float(t.item() if isinstance(t, torch.Tensor) else np.asarray(t))
        with torch.cuda.device(self.dev_index):
            _lib.check(self.lib.sb_enh_upload(self.handle, C.byref(w)), "sb_enh_upload")

    def set_dense_gate(self, weight: torch.Tensor) -> None:
        """The layer's dense gate weight [E, hidden] (fp32 or bf16, any device)
        for the hybrid gate."""
        w = weight.detach()
        if w.dtype not in (torch.float32, torch.bfloat16):
            w = w.float()
        if tuple(w.shape) != (self.n_experts, self.hidden):
            raise RuntimeError(f"dense gate weight must be [{self.n_experts}, {self.hidden}], got {tuple(w.shape)}")
        w = w.to(self.device).contiguous()
        with torch.cuda.device(self.dev_index):
            torch.cuda.current_stream(self.device).synchronize()
            _lib.check(self.lib.sb_enh_set_dense_gate(
                self.handle, C.c_void_p(w.data_ptr()), _lib.SB_BF16 if w.dtype == torch.bfloat16 else _lib.SB_F32,
                w.shape[0], w.shape[1]), "sb_enh_set_dense_gate")

    def workspace(self, batch: int, precision: int) -> torch.Tensor:
        need = int(self.lib.sb_enh_workspace_bytes(self.handle, batch, precision))
        if self._ws is None or self._ws.numel() < need + 1024:
            self._ws = torch.empty(max(need, 1) + 1024, dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(self, x: torch.Tensor, precision: str = "auto", want=("logits", "expert_probs", "expert_ids"),
                gate: Optional[str] = None, k: int = 8, norm_topk_prob: bool = False,
                round_dtype: Optional[torch.dtype] = None, n_candidates: int = 16,
                outputs: Optional[Dict[str, torch.Tensor]] = None) -> Dict[str, torch.Tensor]:
        """Router outputs named in ``want`` (any of OUTPUTS[:5]); with ``gate``
        set also router_probs, topk_weights (fp32) and topk_ids of that mode,
        logits rounded to ``round_dtype`` (default: x's dtype) first.
        ``gate="hybrid"``: top-k of the dense gate's softmax among the
        ``n_candidates`` experts of largest BVH probability (set_dense_gate)."""
        if not x.is_cuda:
            raise RuntimeError("router input must be a CUDA tensor (there is no CPU path)")
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise RuntimeError(f"router input must be [B, {self.hidden}], got {tuple(x.shape)}")
        if x.dtype not in (torch.float32, torch.bfloat16):
            raise RuntimeError(f"router input dtype {x.dtype} must be float32 or bfloat16")
        x = x.contiguous()
        if precision == "auto":
            precision = "fast" if x.dtype == torch.bfloat16 else "exact"
        prec = PRECISIONS[precision]
        B, E, dev = x.shape[0], self.n_experts, x.device
        res: Dict[str, torch.Tensor] = {} if outputs is None else dict(outputs)
        if outputs is None:
            shapes = {"logits": (B, E), "expert_probs": (B, E), "geo_dist": (B, E), "branch_bonus": (B, E)}
            for name in want:
                if name == "expert_ids":
                    res[name] = torch.empty(B, dtype=torch.int64, device=dev)
                else:
                    res[name] = torch.empty(*shapes[name], dtype=torch.float32, device=dev)
            if gate is not None:
                res["router_probs"] = torch.empty(B, E, dtype=torch.float32, device=dev)
                res["topk_weights"] = torch.empty(B, k, dtype=torch.float32, device=dev)
                res["topk_ids"] = torch.empty(B, k, dtype=torch.int32, device=dev)
        o = _lib.EnhOutputs()
        for name in OUTPUTS:
            t = res.get(name)
            setattr(o, name, t.data_ptr() if t is not None else None)
        rd = round_dtype if round_dtype is not None else x.dtype
        ws = self.workspace(B, prec)
        base = ws.data_ptr()
        aligned = (base + 1023) // 1024 * 1024
        stream = torch.cuda.current_stream(dev).cuda_stream
        xd = _lib.SB_BF16 if x.dtype == torch.bfloat16 else _lib.SB_F32
        rdt = _lib.SB_BF16 if rd == torch.bfloat16 else _lib.SB_F32
        wsb = ws.numel() - (aligned - base)
        with torch.cuda.device(dev):
            if gate == "hybrid":
                rc = self.lib.sb_enh_forward_hybrid(
                    self.handle, C.c_void_p(x.data_ptr()), xd, B, prec, int(n_candidates),
                    int(bool(norm_topk_prob)), rdt, int(k), C.byref(o), C.c_void_p(aligned), wsb,
                    C.c_void_p(stream))
            else:
                rc = self.lib.sb_enh_forward(
                    self.handle, C.c_void_p(x.data_ptr()), xd, B, prec, GATE_MODES[gate or "softmax"],
                    int(bool(norm_topk_prob)), rdt, int(k), C.byref(o), C.c_void_p(aligned), wsb,
                    C.c_void_p(stream))
        _lib.check(rc, "sb_enh_forward_hybrid" if gate == "hybrid" else "sb_enh_forward")
        return res
