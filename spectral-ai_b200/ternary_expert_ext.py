"""Drop-in ``ternary_expert_ext`` module backed by libspectral_b200.so.

Same module name and functions as the reference torch extension
(cuda/v5/ternary_torch_ext.cu:345-362), which python/ternary_expert_ext_bridge.py
imports by name:

  pack_ternary(weights_int8)                        CPU int8 [K,N] -> int32 [ceil(K/16), N]
  ternary_linear(input, packed_weights, scale, bias=None)      -> float32 [batch, out]
  ternary_gated_mlp(input, gate_packed, up_packed, down_packed,
                    gate_scale, up_scale, down_scale)          -> float32 [batch, in]

Packed arguments use the reference layout; they are converted once to the
B200 layout on the device and cached per tensor (keyed on storage pointer,
shape and version counter).  The math runs on tcgen05 tensor cores: ternary
weights are exact in 16-bit floats, activations enter as bf16 (bf16 input) or
fp16 (fp32 input) with fp32 accumulation, the SwiGLU hidden state is rounded
to fp16 before the down projection.
"""

from __future__ import annotations

import weakref
from typing import Optional

import torch

from sb200 import _lib
from sb200 import ternary as _t

# repacked weights per packed tensor object, keyed by the object's id and
# holding a weak reference to it: an entry whose tensor died (a later tensor may
# reuse the id) is never taken for the new one, and dies with a finaliser.
# (Tensors cannot be weak-dictionary keys: the lookup compares keys with ==,
# which is elementwise for tensors.)
_cache: dict = {}


def _device_layout(packed: torch.Tensor, K: int) -> torch.Tensor:
    stamp = (packed.data_ptr(), tuple(packed.shape), packed._version, K, packed.device)
    key = id(packed)
    hit = _cache.get(key)
    if hit is not None and hit[0]() is packed and hit[1] == stamp:
        return hit[2]
    out = _t.repack_reference(packed.contiguous(), K)
    if hit is None or hit[0]() is not packed:
        weakref.finalize(packed, _cache.pop, key, None)
    _cache[key] = (weakref.ref(packed), stamp, out)
    return out


def pack_ternary(weights_int8: torch.Tensor) -> torch.Tensor:
    """Host packer, bit-identical to pack_ternary_impl (ternary_torch_ext.cu:197-231)."""
    if not (isinstance(weights_int8, torch.Tensor) and weights_int8.device.type == "cpu"
            and weights_int8.dtype == torch.int8):
        raise RuntimeError("weights must be CPU int8")
    import ctypes as C
    w = weights_int8.contiguous()
    K, N = w.shape
    out = torch.zeros((K + 15) // 16, N, dtype=torch.int32)
    _lib.check(_lib.load().sb_ternary_pack_ref(C.c_void_p(w.data_ptr()), K, N, C.c_void_p(out.data_ptr())),
               "sb_ternary_pack_ref")
    return out


def _check_cuda(t: torch.Tensor, what: str):
    if not (isinstance(t, torch.Tensor) and t.is_cuda and t.is_contiguous()):
        raise RuntimeError(f"{what} must be CUDA contiguous")


def ternary_linear(input: torch.Tensor, packed_weights: torch.Tensor, scale: torch.Tensor,
                   bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    _check_cuda(input, "input")
    _check_cuda(packed_weights, "packed_weights")
    _check_cuda(scale, "scale")
    K = input.shape[1]
    N = packed_weights.shape[1]
    if packed_weights.shape[0] != (K + 15) // 16:
        raise RuntimeError(f"packed_weights rows {packed_weights.shape[0]} do not match in_dim {K}")
    w = _device_layout(packed_weights, K)
    b = bias.float().contiguous() if bias is not None else None
    return _t.linear(input, w, scale.float().contiguous(), b, K, N)


def ternary_gated_mlp(input: torch.Tensor, gate_packed: torch.Tensor, up_packed: torch.Tensor,
                      down_packed: torch.Tensor, gate_scale: torch.Tensor, up_scale: torch.Tensor,
                      down_scale: torch.Tensor) -> torch.Tensor:
    _check_cuda(input, "input")
    H = input.shape[1]
    I = gate_packed.shape[1]
    out_dim = down_packed.shape[1]
    if out_dim != H:
        raise RuntimeError(f"down projection out_dim {out_dim} must equal in_dim {H}")
    g = _device_layout(gate_packed, H)
    u = _device_layout(up_packed, H)
    d = _device_layout(down_packed, I)
    return _t.gated_mlp(input, g, u, d, gate_scale.float().contiguous(), up_scale.float().contiguous(),
                        down_scale.float().contiguous(), H, I)
