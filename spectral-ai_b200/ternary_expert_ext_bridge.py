"""Drop-in ``ternary_expert_ext_bridge`` backed by the B200 ternary kernels.

Mirrors python/ternary_expert_ext_bridge.py of the reference:
  * ``HAS_TERNARY_EXT`` — True when libspectral_b200.so loads (:28-72),
  * ``CUDATernaryExpertModule(expert, output_proj=None)`` with the same
    buffers (gate_packed/up_packed/down_packed in the reference packed layout,
    gate_s/up_s/down_s), ``forward_hidden``, ``forward`` and ``memory_bytes``
    (:75-175),
  * ``create_expert_module(expert, output_proj, prefer_cuda, fallback_class)`` (:178-196).
The forward calls ``ternary_expert_ext.ternary_gated_mlp`` exactly as the
reference does, which here runs the tcgen05 ternary kernels.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch
import torch.nn as nn

HAS_TERNARY_EXT = False
try:
    import ternary_expert_ext
    from sb200 import _lib as _sb_lib
    _sb_lib.load()
    HAS_TERNARY_EXT = True
except (ImportError, RuntimeError, OSError):
    ternary_expert_ext = None


class CUDATernaryExpertModule(nn.Module):
    """Ternary SwiGLU expert; weights packed 2 bits per value."""

    def __init__(self, expert, output_proj: Optional[nn.Linear] = None):
        super().__init__()
        if not HAS_TERNARY_EXT:
            raise RuntimeError("ternary_expert_ext not available. "
                               "Build it with: python spectral-ai_b200/build.py")
        self.expert_id = expert.expert_id
        gate_int8 = torch.from_numpy(np.asarray(expert.gate_ternary).T.copy().astype(np.int8))
        up_int8 = torch.from_numpy(np.asarray(expert.up_ternary).T.copy().astype(np.int8))
        down_int8 = torch.from_numpy(np.asarray(expert.down_ternary).T.copy().astype(np.int8))
        self.register_buffer('gate_packed', ternary_expert_ext.pack_ternary(gate_int8))
        self.register_buffer('up_packed', ternary_expert_ext.pack_ternary(up_int8))
        self.register_buffer('down_packed', ternary_expert_ext.pack_ternary(down_int8))
        self.register_buffer('gate_s', torch.from_numpy(np.asarray(expert.gate_scale, np.float32).copy()))
        self.register_buffer('up_s', torch.from_numpy(np.asarray(expert.up_scale, np.float32).copy()))
        self.register_buffer('down_s', torch.from_numpy(np.asarray(expert.down_scale, np.float32).copy()))
        self.output_proj = output_proj
        self._in_dim = np.asarray(expert.gate_ternary).shape[1]
        self._inter_dim = np.asarray(expert.gate_ternary).shape[0]
        self._out_dim = np.asarray(expert.down_ternary).shape[0]

    def forward_hidden(self, x: torch.Tensor) -> torch.Tensor:
        B, S, H = x.shape
        x_flat = x.reshape(B * S, H).float().contiguous()
        out_flat = ternary_expert_ext.ternary_gated_mlp(
            x_flat, self.gate_packed, self.up_packed, self.down_packed,
            self.gate_s, self.up_s, self.down_s)
        return out_flat.reshape(B, S, -1)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out = self.forward_hidden(x)
        if self.output_proj is not None:
            return self.output_proj(out)
        return out

    def memory_bytes(self) -> int:
        packed_bytes = (self.gate_packed.numel() + self.up_packed.numel() + self.down_packed.numel()) * 4
        scale_bytes = (self.gate_s.numel() + self.up_s.numel() + self.down_s.numel()) * 4
        return packed_bytes + scale_bytes


def create_expert_module(expert, output_proj=None, prefer_cuda=True, fallback_class=None):
    """Best available expert module (reference factory semantics)."""
    if prefer_cuda and HAS_TERNARY_EXT:
        return CUDATernaryExpertModule(expert, output_proj)
    if fallback_class is not None:
        return fallback_class(expert, output_proj)
    raise RuntimeError(
        "ternary_expert_ext not available and no fallback_class provided. "
        "Either build the library (python spectral-ai_b200/build.py) "
        "or pass fallback_class=TernaryExpertModule.")
