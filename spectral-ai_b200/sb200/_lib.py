"""ctypes binding of libspectral_b200.so (the C ABI in include/spectral_b200.h).

The library is loaded from this directory (built in-tree by
``spectral-ai_b200/build.py``).  There is no fallback: if the library is
missing or a call fails, a ``RuntimeError`` carrying the library's own error
message is raised.
"""

from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libspectral_b200.so"

SB_OK = 0
SB_ERR = {
    -1: "SB_ERR_INVALID", -2: "SB_ERR_CUDA", -3: "SB_ERR_UNSUPPORTED",
    -4: "SB_ERR_DEVICE_TIMEOUT", -5: "SB_ERR_NOMEM", -6: "SB_ERR_WORKSPACE",
}
SB_F32, SB_BF16, SB_F16 = 0, 1, 2
SB_SELECT_HARD, SB_SELECT_SOFT = 0, 1
SB_PREC_FAST, SB_PREC_EXACT = 0, 1
SB_MAX_LEVELS = 8

FP = C.POINTER(C.c_float)


class RouterDesc(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("spectral", C.c_int32), ("n_levels", C.c_int32),
                ("branching", C.c_int32 * SB_MAX_LEVELS)]


class RouterWeights(C.Structure):
    _fields_ = [("to3d_w", C.c_void_p), ("to3d_b", C.c_void_p),
                ("enc1_w", C.c_void_p), ("enc1_b", C.c_void_p),
                ("enc2_w", C.c_void_p), ("enc2_b", C.c_void_p),
                ("centers", C.c_void_p * SB_MAX_LEVELS),
                ("refract_w", C.c_void_p * SB_MAX_LEVELS),
                ("refract_b", C.c_void_p * SB_MAX_LEVELS),
                ("portals", C.c_void_p * SB_MAX_LEVELS),
                ("temperature", C.c_float)]


class RouterOutputs(C.Structure):
    _fields_ = [("topk_ids", C.c_void_p), ("topk_weights", C.c_void_p),
                ("expert_id", C.c_void_p), ("expert_probs", C.c_void_p),
                ("route_path", C.c_void_p), ("confidence", C.c_void_p)]


class EnhDesc(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("feature", C.c_int32), ("branching", C.c_int32 * 3)]


class EnhLevel(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("centers", "to3d_w", "to3d_b", "feat0_w", "feat0_b",
                                          "feat2_w", "feat2_b", "head_w", "head_b")]


class EnhWeights(C.Structure):
    _fields_ = ([(n, C.c_void_p) for n in ("in0_w", "in0_b", "in2_w", "in2_b", "ln_w", "ln_b")]
                + [("level", EnhLevel * 3)]
                + [(n, C.c_void_p) for n in ("eh0_w", "eh0_b", "eh2_w", "eh2_b")]
                + [("temperature", C.c_float)])


class EnhOutputs(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("logits", "expert_probs", "expert_ids", "geo_dist", "branch_bonus",
                                          "router_probs", "topk_weights", "topk_ids")]


SB_GATE_SOFTMAX, SB_GATE_TOPK_SOFTMAX, SB_GATE_HYBRID = 0, 1, 2


class EpDesc(C.Structure):
    _fields_ = [("world", C.c_int32), ("rank", C.c_int32), ("n_experts", C.c_int32), ("top_k", C.c_int32),
                ("max_tokens", C.c_int64), ("hidden", C.c_int64), ("intermediate", C.c_int64),
                ("timeout_ms", C.c_int32)]


SB_EP_HANDLE_BYTES = 128

# (name, restype, argtypes) of every symbol the header declares
SIGNATURES = [
    ("sb_abi_version", C.c_int, []),
    ("sb_last_error", C.c_int, [C.c_char_p, C.c_size_t]),
    ("sb_device_status", C.c_int, [C.c_int]),
    ("sb_profile_enable", C.c_int, [C.c_int]),
    ("sb_profile_count", C.c_int, []),
    ("sb_profile_entry", C.c_int, [C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_int64),
                                   C.POINTER(C.c_double)]),
    ("sb_router_create", C.c_int, [C.POINTER(RouterDesc), C.c_int, C.POINTER(C.c_void_p)]),
    ("sb_router_upload", C.c_int, [C.c_void_p, C.POINTER(RouterWeights)]),
    ("sb_router_workspace_bytes", C.c_size_t, [C.c_void_p, C.c_int64, C.c_int]),
    ("sb_router_forward", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int, C.c_int64, C.c_int, C.c_int, C.c_int,
      C.POINTER(RouterOutputs), C.c_void_p, C.c_size_t, C.c_void_p]),
    ("sb_router_destroy", C.c_int, [C.c_void_p]),
    ("sb_router_forward_noalloc", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int, C.c_int64, C.c_int, C.c_int, C.c_int,
      C.POINTER(RouterOutputs), C.c_void_p]),
    ("sb_ternary_pack_ref", C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p]),
    ("sb_ternary_matrix_bytes", C.c_size_t, [C.c_int64, C.c_int64]),
    ("sb_ternary_repack", C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p]),
    ("sb_ternary_gated_mlp", C.c_int,
     [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_int64,
      C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    ("sb_ternary_gated_mlp_workspace_bytes", C.c_size_t, [C.c_int64, C.c_int64, C.c_int64]),
    ("sb_ternary_linear", C.c_int,
     [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p,
      C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    ("sb_ternary_linear_workspace_bytes", C.c_size_t, [C.c_int64, C.c_int64, C.c_int64]),
    ("sb_ternary_moe_swiglu", C.c_int,
     [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_int64, C.c_int32, C.c_int32,
      C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
      C.c_void_p, C.c_size_t, C.c_void_p]),
    ("sb_ternary_moe_workspace_bytes", C.c_size_t,
     [C.c_int64, C.c_int64, C.c_int64, C.c_int32, C.c_int32]),
    ("sb_enh_create", C.c_int, [C.POINTER(EnhDesc), C.c_int, C.POINTER(C.c_void_p)]),
    ("sb_enh_upload", C.c_int, [C.c_void_p, C.POINTER(EnhWeights)]),
    ("sb_enh_workspace_bytes", C.c_size_t, [C.c_void_p, C.c_int64, C.c_int]),
    ("sb_enh_forward", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
      C.POINTER(EnhOutputs), C.c_void_p, C.c_size_t, C.c_void_p]),
    ("sb_enh_set_dense_gate", C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]),
    ("sb_enh_forward_hybrid", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
      C.POINTER(EnhOutputs), C.c_void_p, C.c_size_t, C.c_void_p]),
    ("sb_enh_destroy", C.c_int, [C.c_void_p]),
    ("sb_softmax_topk", C.c_int,
     [C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
      C.c_void_p, C.c_void_p]),
    ("sb_apply_calibration", C.c_int,
     [C.c_void_p, C.c_int64, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("sb_scatter_by_expert", C.c_int,
     [C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("sb_weighted_combine", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    ("sb_tree_create", C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    ("sb_tree_upload", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("sb_tree_route", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p]),
    ("sb_tree_destroy", C.c_int, [C.c_void_p]),
    ("bvh_upload_tree", C.c_int, [C.c_void_p] * 5),
    ("bvh_alloc_buffers", C.c_int, [C.c_int]),
    ("bvh_free_buffers", None, []),
    ("bvh_route_batch", C.c_int, [C.c_void_p] * 7 + [C.c_int, C.c_int]),
    ("bvh_get_batch_capacity", C.c_int, []),
    ("bvh_get_num_nodes", C.c_int, []),
    ("bvh_get_num_experts", C.c_int, []),
    ("bvh_get_spec_dim", C.c_int, []),
    ("sb_gas_create", C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    ("sb_gas_build", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int]),
    ("sb_gas_route", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p]),
    ("sb_gas_destroy", C.c_int, [C.c_void_p]),
    ("sb_ep_create", C.c_int, [C.POINTER(EpDesc), C.POINTER(C.c_void_p)]),
    ("sb_ep_export", C.c_int, [C.c_void_p, C.c_void_p]),
    ("sb_ep_connect", C.c_int, [C.c_void_p, C.c_void_p]),
    ("sb_ep_connect_nccl", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    ("sb_ep_workspace_bytes", C.c_size_t, [C.c_void_p]),
    ("sb_ep_set_placement", C.c_int, [C.c_void_p, C.c_void_p]),
    ("sb_ep_forward", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]),
    ("sb_ep_status", C.c_int, [C.c_void_p]),
    ("sb_ep_inject_stale_wait", C.c_int, [C.c_void_p, C.c_void_p]),
    ("sb_ep_destroy", C.c_int, [C.c_void_p]),
    ("sb_nccl_unique_id", C.c_int, [C.c_void_p]),
    ("sb_nccl_comm_init", C.c_int, [C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_void_p)]),
    ("sb_nccl_comm_destroy", C.c_int, [C.c_void_p]),
]

_lib = None
_lock = threading.Lock()


def load() -> C.CDLL:
    """Loads the library once; raises RuntimeError if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"libspectral_b200.so not found at {LIB_PATH}; build it with "
                    "`python spectral-ai_b200/build.py` (there is no CPU fallback)")
            lib = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
            for name, res, args in SIGNATURES:
                f = getattr(lib, name, None)
                if f is None:
                    continue
                f.restype = res
                f.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(2048)
    load().sb_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != SB_OK:
        raise RuntimeError(f"{what}: {SB_ERR.get(rc, rc)}: {last_error()}")


def profile_enable(on: bool = True) -> None:
    load().sb_profile_enable(1 if on else 0)


def profile_read():
    """{kernel name: (launches, total_ms)} of the library's event profiler."""
    lib = load()
    out = {}
    for i in range(lib.sb_profile_count()):
        name = C.create_string_buffer(128)
        n = C.c_int64()
        ms = C.c_double()
        check(lib.sb_profile_entry(i, name, 128, C.byref(n), C.byref(ms)), "sb_profile_entry")
        out[name.value.decode()] = (int(n.value), float(ms.value))
    return out


def exported_symbols():
    return [name for name, _, _ in SIGNATURES]
