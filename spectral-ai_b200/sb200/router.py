"""Torch-facing wrapper of the C-ABI router handle (sb_router_*).

``RouterEngine`` owns one ``sb_router`` handle per device, uploads fp32
parameters from a state-dict-like mapping, and runs the forward on torch CUDA
tensors on the current stream.  Outputs are allocated with ``torch.empty`` on
the input's device, like the reference extension (cuda/v5/bvh_torch_ext.cu:328-331).
"""

from __future__ import annotations

import ctypes as C
from typing import Dict, Mapping, Optional, Sequence

import numpy as np
import torch

from . import _lib

PRECISIONS = {"fast": _lib.SB_PREC_FAST, "exact": _lib.SB_PREC_EXACT}
SELECTS = {"hard": _lib.SB_SELECT_HARD, "soft": _lib.SB_SELECT_SOFT}


def _level_sizes(branching: Sequence[int]):
    out, n = [], 1
    for b in branching:
        n *= int(b)
        out.append(n)
    return out


class RouterEngine:
    """One router handle on one CUDA device."""

    def __init__(self, hidden: int, spectral: int, branching: Sequence[int], device):
        self.lib = _lib.load()
        self.hidden, self.spectral = int(hidden), int(spectral)
        self.branching = tuple(int(b) for b in branching)
        self.sizes = _level_sizes(self.branching)
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("RouterEngine needs a CUDA device (there is no CPU path)")
        desc = _lib.RouterDesc()
        desc.hidden, desc.spectral, desc.n_levels = self.hidden, self.spectral, len(self.branching)
        for i, b in enumerate(self.branching):
            desc.branching[i] = b
        h = C.c_void_p()
        dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.dev_index = dev_index
        _lib.check(self.lib.sb_router_create(C.byref(desc), dev_index, C.byref(h)), "sb_router_create")
        self.handle = h
        self._ws: Optional[torch.Tensor] = None

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                self.lib.sb_router_destroy(h)
            except Exception:
                pass
            self.handle = None

    def upload(self, params: Mapping[str, object]) -> None:
        """params: state_dict names -> tensors/arrays (any dtype/device)."""
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

        w = _lib.RouterWeights()
        w.to3d_w, w.to3d_b = ptr("to_3d.weight"), ptr("to_3d.bias", False)
        w.enc1_w, w.enc1_b = ptr("spectral.net.0.weight"), ptr("spectral.net.0.bias", False)
        w.enc2_w, w.enc2_b = ptr("spectral.net.2.weight"), ptr("spectral.net.2.bias", False)
        L = len(self.branching)
        for l in range(L):
            w.centers[l] = ptr(f"level{l + 1}.centers")
            w.refract_w[l] = ptr(f"refract{l + 1}.W_dispersion.weight")
            w.refract_b[l] = ptr(f"refract{l + 1}.W_dispersion.bias", False)
            if l < L - 1:
                w.portals[l] = ptr(f"portal{l + 1}.transform")
        t = params.get("temperature", 1.0)
        w.temperature = float(t.item() if isinstance(t, torch.Tensor) else np.asarray(t))
        with torch.cuda.device(self.dev_index):
            _lib.check(self.lib.sb_router_upload(self.handle, C.byref(w)), "sb_router_upload")

    def workspace(self, batch: int, precision: int) -> torch.Tensor:
        need = int(self.lib.sb_router_workspace_bytes(self.handle, batch, precision))
        if self._ws is None or self._ws.numel() < need + 1024:
            self._ws = torch.empty(max(need, 1) + 1024, dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(self, x: torch.Tensor, precision: str = "auto", select: str = "hard",
                k: int = 0, want=("expert_id", "expert_probs", "route_path", "confidence"),
                outputs: Optional[Dict[str, torch.Tensor]] = None) -> Dict[str, torch.Tensor]:
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
        sel = SELECTS[select]
        B = x.shape[0]
        L, NL = len(self.branching), self.sizes[-1]
        dev = x.device
        res: Dict[str, torch.Tensor] = {} if outputs is None else dict(outputs)
        if outputs is None:
            if "expert_id" in want:
                res["expert_id"] = torch.empty(B, dtype=torch.int64, device=dev)
            if "expert_probs" in want:
                res["expert_probs"] = torch.empty(B, NL, dtype=torch.float32, device=dev)
            if "route_path" in want:
                res["route_path"] = torch.empty(B, L, dtype=torch.int64, device=dev)
            if "confidence" in want:
                res["confidence"] = torch.empty(B, dtype=torch.float32, device=dev)
            if k:
                res["topk_ids"] = torch.empty(B, k, dtype=torch.int32, device=dev)
                res["topk_weights"] = torch.empty(B, k, dtype=torch.float32, device=dev)
        o = _lib.RouterOutputs()
        for name in ("topk_ids", "topk_weights", "expert_id", "expert_probs", "route_path", "confidence"):
            t = res.get(name)
            setattr(o, name, t.data_ptr() if t is not None else None)
        ws = self.workspace(B, prec)
        base = ws.data_ptr()
        aligned = (base + 1023) // 1024 * 1024
        stream = torch.cuda.current_stream(dev).cuda_stream
        with torch.cuda.device(dev):
            rc = self.lib.sb_router_forward(
                self.handle, C.c_void_p(x.data_ptr()),
                _lib.SB_BF16 if x.dtype == torch.bfloat16 else _lib.SB_F32,
                B, prec, sel, int(k), C.byref(o), C.c_void_p(aligned),
                ws.numel() - (aligned - base), C.c_void_p(stream))
        _lib.check(rc, "sb_router_forward")
        return res
