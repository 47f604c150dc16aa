"""Torch-facing wrappers of the ternary C-ABI entry points.

Weights live on the device in the B200 layout: uint32 [N, KW], KW =
ceil(K/64)*4, one word per 16 consecutive K of an output row; element 2j+e of
a word (e = 0, 1) is stored as the biased code value+1 in bits 16e+p_j ..
16e+p_j+1 with p_j = TERN_POS[j] (the order in which the kernels can expand
most pairs without a shift), and padding holds code 1 (value 0).  ``pack_device`` builds it on the host from int8 ternary
matrices in the PyTorch [out, in] layout; ``repack_reference`` converts the
reference extension's packed layout (int32 [ceil(K/16), N],
cuda/v5/ternary_torch_ext.cu:197-231) on the device.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib


# bit position of pair j in each 16-bit half (csrc/ternary_gemm.cuh tern_pos)
TERN_POS = (0, 2, 4, 8, 10, 12, 6, 14)


def row_words(K: int) -> int:
    return (K + 63) // 64 * 4


def pack_device(T: np.ndarray) -> np.ndarray:
    """int8 ternary [N, K] ({-1,0,+1}) -> uint32 [N, ceil(K/64)*4] device layout."""
    T = np.asarray(T)
    N, K = T.shape
    KW = row_words(K)
    pad = np.zeros((N, KW * 16), np.int8)
    pad[:, :K] = T
    code = (pad.reshape(N, KW, 8, 2).astype(np.int64) + 1).astype(np.uint32)  # [n, word, j, e]
    p = np.array(TERN_POS, dtype=np.uint32)[None, None, :]
    w = (code[..., 0] << p) | (code[..., 1] << (16 + p))
    return np.bitwise_or.reduce(w, axis=2).astype(np.uint32)


def pack_device_torch(T: torch.Tensor) -> torch.Tensor:
    """Same layout as ``pack_device`` with torch ops on any device:
    int8 [N, K] -> int32 [N, ceil(K/64)*4] (the uint32 words viewed as int32)."""
    N, K = T.shape
    KW = row_words(K)
    pad = torch.zeros(N, KW * 16, dtype=torch.int8, device=T.device)
    pad[:, :K] = T
    code = pad.view(N, KW, 8, 2).to(torch.int64) + 1
    p = torch.tensor(TERN_POS, device=T.device, dtype=torch.int64).view(1, 1, 8)
    w = (code[..., 0] << p) | (code[..., 1] << (16 + p))
    words = w.sum(dim=2)  # the bit fields of the 8 pairs are disjoint
    return torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)


def _stream(dev) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _ws(nbytes: int, device) -> tuple:
    buf = torch.empty(nbytes + 1024, dtype=torch.uint8, device=device)
    base = buf.data_ptr()
    aligned = (base + 1023) // 1024 * 1024
    return buf, aligned, buf.numel() - (aligned - base)


def repack_reference(packed: torch.Tensor, K: int) -> torch.Tensor:
    """Reference-layout packed int32 [ceil(K/16), N] (CUDA) -> device layout (CUDA)."""
    lib = _lib.load()
    if not packed.is_cuda:
        raise RuntimeError("packed weights must be a CUDA tensor")
    packed = packed.contiguous()
    N = packed.shape[1]
    out = torch.empty(N, row_words(K), dtype=torch.int32, device=packed.device)
    with torch.cuda.device(packed.device):
        _lib.check(lib.sb_ternary_repack(C.c_void_p(packed.data_ptr()), K, N, C.c_void_p(out.data_ptr()),
                                         _stream(packed.device)), "sb_ternary_repack")
    return out


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return _lib.SB_F32
    if t.dtype == torch.bfloat16:
        return _lib.SB_BF16
    raise RuntimeError(f"activation dtype {t.dtype} must be float32 or bfloat16")


def gated_mlp(x: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
              gate_scale: torch.Tensor, up_scale: torch.Tensor, down_scale: torch.Tensor,
              hidden: int, inter: int) -> torch.Tensor:
    """One expert: y fp32 [M, H]; weights already in the device layout."""
    lib = _lib.load()
    M = x.shape[0]
    y = torch.empty(M, hidden, dtype=torch.float32, device=x.device)
    need = int(lib.sb_ternary_gated_mlp_workspace_bytes(M, hidden, inter))
    buf, ws, wsb = _ws(need, x.device)
    with torch.cuda.device(x.device):
        rc = lib.sb_ternary_gated_mlp(
            C.c_void_p(x.data_ptr()), _dtype_code(x), M, hidden, inter,
            C.c_void_p(gate.data_ptr()), C.c_void_p(up.data_ptr()), C.c_void_p(down.data_ptr()),
            C.c_void_p(gate_scale.data_ptr()), C.c_void_p(up_scale.data_ptr()),
            C.c_void_p(down_scale.data_ptr()), C.c_void_p(y.data_ptr()), C.c_void_p(ws), wsb,
            _stream(x.device))
    _lib.check(rc, "sb_ternary_gated_mlp")
    return y


def linear(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor, bias: Optional[torch.Tensor],
           K: int, N: int) -> torch.Tensor:
    lib = _lib.load()
    M = x.shape[0]
    y = torch.empty(M, N, dtype=torch.float32, device=x.device)
    need = int(lib.sb_ternary_linear_workspace_bytes(M, K, N))
    buf, ws, wsb = _ws(need, x.device)
    with torch.cuda.device(x.device):
        rc = lib.sb_ternary_linear(C.c_void_p(x.data_ptr()), _dtype_code(x), M, K, N,
                                   C.c_void_p(w.data_ptr()), C.c_void_p(scale.data_ptr()),
                                   C.c_void_p(bias.data_ptr()) if bias is not None else None,
                                   C.c_void_p(y.data_ptr()), C.c_void_p(ws), wsb, _stream(x.device))
    _lib.check(rc, "sb_ternary_linear")
    return y


class TernaryExperts:
    """E ternary SwiGLU experts resident on one device, in the B200 layout.

    ``experts`` is a sequence of containers with the reference fields
    (python/real_model_demo.py:85-98): gate_ternary [I,H], up_ternary [I,H],
    down_ternary [H,I] (values in {-1,0,+1}) and gate_scale [I], up_scale [I],
    down_scale [H]; dicts or attribute objects both work.
    """

    def __init__(self, experts: Sequence, device):
        def get(e, k):
            return e[k] if isinstance(e, dict) else getattr(e, k)

        self.device = torch.device(device)
        self.E = len(experts)
        g0 = np.asarray(get(experts[0], "gate_ternary"))
        self.I, self.H = g0.shape
        gate = np.concatenate([pack_device(np.asarray(get(e, "gate_ternary"), np.int8)) for e in experts])
        up = np.concatenate([pack_device(np.asarray(get(e, "up_ternary"), np.int8)) for e in experts])
        down = np.concatenate([pack_device(np.asarray(get(e, "down_ternary"), np.int8)) for e in experts])
        to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(self.device)
        self.gate = to(gate.view(np.int32))
        self.up = to(up.view(np.int32))
        self.down = to(down.view(np.int32))
        self.gate_scale = to(np.stack([np.asarray(get(e, "gate_scale"), np.float32) for e in experts]))
        self.up_scale = to(np.stack([np.asarray(get(e, "up_scale"), np.float32) for e in experts]))
        self.down_scale = to(np.stack([np.asarray(get(e, "down_scale"), np.float32) for e in experts]))
        self._ws = None

    @classmethod
    def from_packed_modules(cls, modules: Sequence, device) -> "TernaryExperts":
        """Group expert modules that hold the reference packed layout
        (``CUDATernaryExpertModule``: gate_packed / up_packed / down_packed from
        ``pack_ternary`` and per-channel gate_s / up_s / down_s,
        python/ternary_expert_ext_bridge.py:93-129) into one device block,
        repacked on the device."""
        self = cls.__new__(cls)
        self.device = torch.device(device)
        self.E = len(modules)
        m0 = modules[0]
        self.H, self.I = int(m0._in_dim), int(m0._inter_dim)
        for m in modules:
            if (int(m._in_dim), int(m._inter_dim), int(m._out_dim)) != (self.H, self.I, self.H):
                raise RuntimeError("grouped experts need equal shapes with out_dim == in_dim")
        dev = self.device
        self.gate = torch.cat([repack_reference(m.gate_packed.to(dev), self.H) for m in modules])
        self.up = torch.cat([repack_reference(m.up_packed.to(dev), self.H) for m in modules])
        self.down = torch.cat([repack_reference(m.down_packed.to(dev), self.I) for m in modules])
        self.gate_scale = torch.stack([m.gate_s.to(dev, torch.float32) for m in modules]).contiguous()
        self.up_scale = torch.stack([m.up_s.to(dev, torch.float32) for m in modules]).contiguous()
        self.down_scale = torch.stack([m.down_s.to(dev, torch.float32) for m in modules]).contiguous()
        self._ws = None
        return self

    @classmethod
    def random(cls, n_experts: int, hidden: int, inter: int, seed: int, device) -> "TernaryExperts":
        """Random experts built on the device: T uniform over {-1,0,+1}, one
        scale c/sqrt(fan_in) per matrix with c ~ U[0.5, 1.5) (the recipe of
        sb200.synth.ternary_experts, drawn from a device generator)."""
        self = cls.__new__(cls)
        self.device = torch.device(device)
        self.E, self.H, self.I = n_experts, hidden, inter
        g = torch.Generator(device=self.device).manual_seed(seed)
        rng = np.random.default_rng(seed)

        def mats(rows, cols):
            out = []
            for _ in range(n_experts):
                t = torch.randint(-1, 2, (rows, cols), generator=g, device=self.device, dtype=torch.int8)
                out.append(pack_device_torch(t))
            return torch.cat(out)

        self.gate = mats(inter, hidden)
        self.up = mats(inter, hidden)
        self.down = mats(hidden, inter)

        def scales(n, fan_in):
            c = rng.uniform(0.5, 1.5, size=(n_experts, 1)) / np.sqrt(fan_in)
            return torch.from_numpy(np.repeat(c, n, axis=1).astype(np.float32)).to(self.device)

        self.gate_scale = scales(inter, hidden)
        self.up_scale = scales(inter, hidden)
        self.down_scale = scales(hidden, inter)
        self._ws = None
        return self

    def memory_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.gate, self.up, self.down, self.gate_scale,
                                                            self.up_scale, self.down_scale))

    def workspace_bytes(self, B: int, k: int) -> int:
        return int(_lib.load().sb_ternary_moe_workspace_bytes(B, self.H, self.I, self.E, k))

    def forward(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                out_dtype=torch.float32, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """out[t] = sum_j weights[t,j] * expert_{ids[t,j]}(x[t])."""
        lib = _lib.load()
        if not x.is_cuda:
            raise RuntimeError("activations must be CUDA tensors (there is no CPU path)")
        x = x.contiguous()
        ids = ids.to(torch.int32).contiguous()
        weights = weights.to(torch.float32).contiguous()
        B, k = ids.shape
        if out is None:
            out = torch.empty(B, self.H, dtype=out_dtype, device=x.device)
        need = self.workspace_bytes(B, k)
        if self._ws is None or self._ws[0].numel() < need + 1024:
            self._ws = _ws(need, x.device)
        buf, ws, wsb = self._ws
        with torch.cuda.device(x.device):
            rc = lib.sb_ternary_moe_swiglu(
                C.c_void_p(x.data_ptr()), _dtype_code(x), B, self.H, self.I, self.E, k,
                C.c_void_p(ids.data_ptr()), C.c_void_p(weights.data_ptr()),
                C.c_void_p(self.gate.data_ptr()), C.c_void_p(self.up.data_ptr()),
                C.c_void_p(self.down.data_ptr()), C.c_void_p(self.gate_scale.data_ptr()),
                C.c_void_p(self.up_scale.data_ptr()), C.c_void_p(self.down_scale.data_ptr()),
                C.c_void_p(out.data_ptr()),
                _lib.SB_BF16 if out.dtype == torch.bfloat16 else _lib.SB_F32,
                C.c_void_p(ws), wsb, _stream(x.device))
        _lib.check(rc, "sb_ternary_moe_swiglu")
        return out
