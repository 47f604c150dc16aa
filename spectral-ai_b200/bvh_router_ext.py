"""Drop-in ``bvh_router_ext`` (the reference's torch extension of the legacy
ray-sphere tree router, cuda/v5/bvh_torch_ext.cu:270-371) backed by the B200
kernel (sb_tree_* of libspectral_b200.so).

  upload_tree(centers[85,3], radii[85], portals[85,12], snell_w[85,64], snell_b[85])
      CPU contiguous float32 tensors, as the reference checks (:276-286);
  route(origins[B,3], directions[B,3], spectral[B,64])
      CUDA contiguous float32; returns (expert_ids int32 [B], scores f32 [B,64],
      confidence f32 [B], path int32 [B,3]), asynchronous on the current stream;
  route_sync(...) the same, then a device synchronize.
The tree lives per device (one per CUDA device the calls touch), uploaded to
every device already in use; the reference keeps one tree in __constant__
memory.  The reference caps a batch at 1024 rays; this one does not.
"""

from __future__ import annotations

import ctypes as C
from typing import Dict, Tuple

import torch

from sb200 import _lib

_trees: Dict[int, C.c_void_p] = {}
_params = None


def _check_cpu(t: torch.Tensor, name: str, shape) -> None:
    if not (isinstance(t, torch.Tensor) and t.device.type == "cpu" and t.is_contiguous()
            and t.dtype == torch.float32 and tuple(t.shape) == tuple(shape)):
        raise RuntimeError(f"{name}: CPU contiguous float32 {list(shape)}")


def _tree(device_index: int) -> C.c_void_p:
    lib = _lib.load()
    h = _trees.get(device_index)
    if h is None:
        h = C.c_void_p()
        _lib.check(lib.sb_tree_create(device_index, C.byref(h)), "sb_tree_create")
        _trees[device_index] = h
        if _params is not None:
            _upload(h)
    return h


def _upload(h: C.c_void_p) -> None:
    lib = _lib.load()
    ptrs = [C.c_void_p(t.data_ptr()) for t in _params]
    _lib.check(lib.sb_tree_upload(h, *ptrs), "sb_tree_upload")


def upload_tree(centers: torch.Tensor, radii: torch.Tensor, portals: torch.Tensor, snell_w: torch.Tensor,
                snell_b: torch.Tensor) -> None:
    global _params
    _check_cpu(centers, "centers", (85, 3))
    _check_cpu(radii, "radii", (85,))
    _check_cpu(portals, "portals", (85, 12))
    _check_cpu(snell_w, "snell_w", (85, 64))
    _check_cpu(snell_b, "snell_b", (85,))
    _params = tuple(t.clone() for t in (centers, radii, portals, snell_w, snell_b))
    if not _trees:
        _tree(torch.cuda.current_device())
    for h in _trees.values():
        _upload(h)


def route(ray_origins: torch.Tensor, ray_directions: torch.Tensor,
          ray_spectral: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    for t, name, w in ((ray_origins, "ray_origins", 3), (ray_directions, "ray_directions", 3),
                       (ray_spectral, "ray_spectral", 64)):
        if not (isinstance(t, torch.Tensor) and t.is_cuda and t.is_contiguous() and t.dtype == torch.float32
                and t.dim() == 2 and t.shape[1] == w):
            raise RuntimeError(f"{name}: CUDA contiguous float32 [batch, {w}]")
    if _params is None:
        raise RuntimeError("call upload_tree first")
    B = ray_origins.shape[0]
    if B <= 0 or ray_directions.shape[0] != B or ray_spectral.shape[0] != B:
        raise RuntimeError(f"batch_size must be >= 1 and equal for all inputs, got {B}")
    dev = ray_origins.device
    h = _tree(dev.index if dev.index is not None else torch.cuda.current_device())
    expert = torch.empty(B, dtype=torch.int32, device=dev)
    scores = torch.empty(B, 64, dtype=torch.float32, device=dev)
    conf = torch.empty(B, dtype=torch.float32, device=dev)
    path = torch.empty(B, 3, dtype=torch.int32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sb_tree_route(h, C.c_void_p(ray_origins.data_ptr()), C.c_void_p(ray_directions.data_ptr()), B,
                               C.c_void_p(expert.data_ptr()), C.c_void_p(scores.data_ptr()),
                               C.c_void_p(path.data_ptr()), C.c_void_p(conf.data_ptr()),
                               C.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(rc, "sb_tree_route")
    return expert, scores, conf, path


def route_sync(ray_origins: torch.Tensor, ray_directions: torch.Tensor, ray_spectral: torch.Tensor):
    out = route(ray_origins, ray_directions, ray_spectral)
    torch.cuda.synchronize(ray_origins.device)
    return out
