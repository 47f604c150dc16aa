"""Drop-in ``optix_training_ext`` (the reference's OptiX RT-core router
extension, cuda/v5/optix_training_ext.cu) served by the CUDA kernels of
libspectral_b200.so (sb_gas_*): no OptiX, RT cores or PTX programs.

Same functions and argument checks:
  initialize(ptx_raygen, ptx_hitgroup)      accepts any paths (there is no PTX)
  build_gas(centers[N,3], radii[N], use_triangles=False)   CPU float32
  route(positions[B,3], directions[B,3]) -> (expert_ids int32 [B], distances f32 [B])
  route_topk(positions, directions, top_k=8) -> (topk_ids int32 [B,k], topk_dists f32 [B,k])
  route_async(...), sync(), is_ready(), gas_size(), num_experts(), shutdown(),
  benchmark(...), is_coopvec_supported(), upload_calibration_affine/linear,
  disable_calibration(), has_calibration()
Routing semantics follow the reference's device programs
(cuda/optix_router_raygen.cu, cuda/optix_router_hitgroup.cu): the closest hit
in t in [0.001, 1000] names the expert (-1 and 1e30 on a miss); top-k traces a
fan of k rays.  Boxes (use_triangles=False) are hit at their entry point —
the reference's intersection program reports every box at the ray's tmin,
which leaves its choice to the RT traversal order.  The calibration uploads
are stored and checked as in the reference; like the reference's programs,
routing does not read them.
"""

from __future__ import annotations

import ctypes as C
import time
from typing import Optional, Tuple

import torch

from sb200 import _lib

_state = {"init": False, "gas": None, "dev": None, "n": 0, "bytes": 0, "cal": None}


def _check(t: torch.Tensor, name: str, cuda: bool) -> None:
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} must be a tensor")
    if cuda and not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not cuda and t.is_cuda:
        raise RuntimeError(f"{name} must be a CPU tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} has wrong dtype")


def initialize(ptx_raygen: str = "", ptx_hitgroup: str = "") -> bool:
    _state["init"] = True
    return True


def build_gas(centers: torch.Tensor, radii: torch.Tensor, use_triangles: bool = False) -> bool:
    if not _state["init"]:
        raise RuntimeError("Call initialize() first")
    _check(centers, "centers", cuda=False)
    _check(radii, "radii", cuda=False)
    if centers.dim() != 2 or centers.shape[1] != 3:
        raise RuntimeError("centers must be (N, 3)")
    n = centers.shape[0]
    if radii.dim() != 1 or radii.shape[0] != n:
        raise RuntimeError("radii must be (N,)")
    lib = _lib.load()
    dev = torch.cuda.current_device()
    if _state["gas"] is None or _state["dev"] != dev:
        h = C.c_void_p()
        _lib.check(lib.sb_gas_create(dev, C.byref(h)), "sb_gas_create")
        _state["gas"], _state["dev"] = h, dev
    _lib.check(lib.sb_gas_build(_state["gas"], C.c_void_p(centers.data_ptr()), C.c_void_p(radii.data_ptr()), n,
                                int(bool(use_triangles))), "sb_gas_build")
    _state["n"] = n
    _state["bytes"] = n * 16
    return True


def is_ready() -> bool:
    return bool(_state["init"] and _state["gas"] is not None and _state["n"] > 0)


def gas_size() -> int:
    return int(_state["bytes"])


def num_experts() -> int:
    return int(_state["n"])


def _route(positions: torch.Tensor, directions: torch.Tensor, top_k: int, sync: bool):
    if not is_ready():
        raise RuntimeError("Router not ready. Call initialize() + build_gas() first.")
    _check(positions, "positions", cuda=True)
    _check(directions, "directions", cuda=True)
    if positions.dim() != 2 or positions.shape[1] != 3:
        raise RuntimeError("positions must be (B, 3)")
    if directions.dim() != 2 or directions.shape[1] != 3 or directions.shape[0] != positions.shape[0]:
        raise RuntimeError("directions must be (B, 3)")
    B, dev = positions.shape[0], positions.device
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    dists = torch.empty(B, dtype=torch.float32, device=dev)
    tids: Optional[torch.Tensor] = None
    tdists: Optional[torch.Tensor] = None
    if top_k > 1:
        tids = torch.empty(B, top_k, dtype=torch.int32, device=dev)
        tdists = torch.empty(B, top_k, dtype=torch.float32, device=dev)
    lib = _lib.load()
    P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
    with torch.cuda.device(dev):
        rc = lib.sb_gas_route(_state["gas"], P(positions), P(directions), B, int(top_k), P(ids), P(dists), P(tids),
                              P(tdists), C.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(rc, "sb_gas_route")
    if sync:
        torch.cuda.current_stream(dev).synchronize()
    return ids, dists, tids, tdists


def route(positions: torch.Tensor, directions: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    ids, dists, _, _ = _route(positions, directions, 1, True)
    return ids, dists


def route_topk(positions: torch.Tensor, directions: torch.Tensor, top_k: int = 8) -> Tuple[torch.Tensor, torch.Tensor]:
    if top_k < 1:
        raise RuntimeError("top_k must be >= 1")
    ids, dists, tids, tdists = _route(positions, directions, int(top_k), True)
    if top_k == 1:
        return ids.view(-1, 1), dists.view(-1, 1)
    return tids, tdists


def route_async(positions: torch.Tensor, directions: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    ids, dists, _, _ = _route(positions, directions, 1, False)
    return ids, dists


def sync() -> None:
    if _state["gas"] is not None:
        torch.cuda.current_stream().synchronize()


def benchmark(num_experts: int = 64, batch_size: int = 256, num_warmup: int = 10, num_iters: int = 100,
              ptx_raygen: str = "", ptx_hitgroup: str = "") -> bool:
    """Routes random queries against random spheres in both geometry modes and
    prints the time per batch (host clock around a synchronize)."""
    g = torch.Generator().manual_seed(0)
    centers = torch.randn(num_experts, 3, generator=g) * 3.0
    radii = torch.rand(num_experts, generator=g) + 0.5
    pos = torch.randn(batch_size, 3, generator=g).cuda()
    dirs = torch.nn.functional.normalize(torch.randn(batch_size, 3, generator=g), dim=1).cuda()
    initialize()
    for tris in (False, True):
        build_gas(centers, radii, tris)
        for _ in range(num_warmup):
            route(pos, dirs)
        t0 = time.perf_counter()
        for _ in range(num_iters):
            route(pos, dirs)
        us = (time.perf_counter() - t0) / num_iters * 1e6
        print(f"  {'triangles' if tris else 'boxes'}: {us:.1f} us per batch of {batch_size}")
    return True


def shutdown() -> None:
    if _state["gas"] is not None:
        _lib.load().sb_gas_destroy(_state["gas"])
    _state.update(init=False, gas=None, dev=None, n=0, bytes=0, cal=None)


def is_coopvec_supported() -> bool:
    return False   # no OptiX cooperative vectors on this path


def upload_calibration_affine(scale: torch.Tensor, bias: torch.Tensor) -> bool:
    if not _state["init"]:
        raise RuntimeError("Call initialize() first")
    _check(scale, "scale", cuda=False)
    _check(bias, "bias", cuda=False)
    if scale.dim() != 1 or bias.dim() != 1 or scale.shape[0] != bias.shape[0]:
        raise RuntimeError("scale and bias must be 1D of the same size")
    _state["cal"] = ("affine", scale.clone(), bias.clone())
    return True


def upload_calibration_linear(W: torch.Tensor, bias: torch.Tensor) -> bool:
    if not _state["init"]:
        raise RuntimeError("Call initialize() first")
    _check(W, "W", cuda=False)
    _check(bias, "bias", cuda=False)
    if W.dim() != 2 or bias.dim() != 1 or W.shape[0] != bias.shape[0]:
        raise RuntimeError("W rows must match bias size")
    _state["cal"] = ("linear", W.clone(), bias.clone())
    return True


def disable_calibration() -> bool:
    if not _state["init"]:
        return False
    _state["cal"] = None
    return True


def has_calibration() -> bool:
    return bool(_state["init"] and _state["cal"] is not None)
