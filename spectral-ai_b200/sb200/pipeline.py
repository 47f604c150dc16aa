"""Torch-facing wrappers of the MoE pipeline stage kernels (sb_softmax_topk,
sb_apply_calibration, sb_scatter_by_expert, sb_weighted_combine).

They replace the stage kernels of the reference's tri-core pipeline
(cuda/async_pipeline.cu:79-230) and the Python stage loops of
python/async_pipeline_bridge.py:89-150.  Every call runs on the current CUDA
stream of its input's device; there is no CPU path.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional, Tuple

import torch

from . import _lib


def _stream(dev) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (there is no CPU path)")


def _ptr(t: Optional[torch.Tensor]):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def softmax_topk(logits: torch.Tensor, k: int, cal_w: Optional[torch.Tensor] = None,
                 cal_b: Optional[torch.Tensor] = None, apply_softmax: bool = True,
                 want_probs: bool = False) -> Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]]:
    """(topk_ids int32 [B,k], topk_weights f32 [B,k], probs f32 [B,E] or None).

    logits [B,E] f32; optional calibration cal_w [E,E] (nn.Linear layout),
    cal_b [E]; softmax over E when apply_softmax; top-k by value, lower expert
    index first among equal values."""
    _cuda(logits, "logits")
    x = logits.float().contiguous()
    B, E = x.shape
    dev = x.device
    ids = torch.empty(B, k, dtype=torch.int32, device=dev)
    wts = torch.empty(B, k, dtype=torch.float32, device=dev)
    probs = torch.empty(B, E, dtype=torch.float32, device=dev) if want_probs else None
    cw = cal_w.float().contiguous() if cal_w is not None else None
    cb = cal_b.float().contiguous() if cal_b is not None else None
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sb_softmax_topk(_ptr(x), B, E, int(k), _ptr(cw), _ptr(cb), int(bool(apply_softmax)), _ptr(probs),
                                 _ptr(ids), _ptr(wts), _stream(dev))
    _lib.check(rc, "sb_softmax_topk")
    return ids, wts, probs


def apply_calibration(raw: torch.Tensor, cal_w: torch.Tensor, cal_b: torch.Tensor) -> torch.Tensor:
    """raw [B,E] W^T + b (the pipeline's Linear(E,E) calibration)."""
    _cuda(raw, "raw")
    x = raw.float().contiguous()
    B, E = x.shape
    out = torch.empty_like(x)
    cw, cb = cal_w.float().contiguous(), cal_b.float().contiguous()
    lib = _lib.load()
    with torch.cuda.device(x.device):
        rc = lib.sb_apply_calibration(_ptr(x), B, E, _ptr(cw), _ptr(cb), _ptr(out), _stream(x.device))
    _lib.check(rc, "sb_apply_calibration")
    return out


def scatter_by_expert(ids: torch.Tensor, n_experts: int, max_tokens_per_expert: Optional[int] = None,
                      store_entry: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """(dispatch_indices int32 [E, max], expert_counts int32 [E]) of routing ids
    [B,k]: expert e's first min(count, max) entries in token order, as the
    token index t (or the entry index t*k + j with ``store_entry``).  Counts
    are not clamped; max defaults to B (nothing dropped)."""
    _cuda(ids, "ids")
    x = ids.to(torch.int32).contiguous()
    B, k = x.shape
    mx = B if max_tokens_per_expert is None else int(max_tokens_per_expert)
    disp = torch.empty(n_experts, max(mx, 0), dtype=torch.int32, device=x.device)
    counts = torch.empty(n_experts, dtype=torch.int32, device=x.device)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        rc = lib.sb_scatter_by_expert(_ptr(x), B, k, int(n_experts), mx, int(bool(store_entry)), _ptr(disp),
                                      _ptr(counts), _stream(x.device))
    _lib.check(rc, "sb_scatter_by_expert")
    return disp, counts


def weighted_combine(expert_outputs: torch.Tensor, weights: torch.Tensor,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out [B,H] = sum_j weights[t,j] * expert_outputs[t,j,:] (fp32)."""
    _cuda(expert_outputs, "expert_outputs")
    eo = expert_outputs.float().contiguous()
    B, k, H = eo.shape
    w = weights.float().contiguous()
    if out is None:
        out = torch.empty(B, H, dtype=torch.float32, device=eo.device)
    lib = _lib.load()
    with torch.cuda.device(eo.device):
        rc = lib.sb_weighted_combine(_ptr(eo), _ptr(w), B, H, k, _ptr(out), _stream(eo.device))
    _lib.check(rc, "sb_weighted_combine")
    return out
