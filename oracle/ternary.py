"""CPU restatement of the ternary expert SwiGLU (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg use this module; the product path never does.

Restated from the reference:
  * ``pack_ternary``      cuda/v5/ternary_torch_ext.cu:197-231
        2-bit codes 00 = 0, 01 = +1, 10 = -1, sixteen per uint32 along the
        input (K) dimension: bit pair i of word [pr, c] holds row pr*16+i.
  * code decode           cuda/v5/ternary_torch_ext.cu:38-53
        sign = (code == 1) - (code >> 1)  (so the unused code 11 reads -1)
  * ``ternary_linear``    cuda/v5/ternary_torch_ext.cu:68-107
  * ``ternary_gated_mlp`` cuda/v5/ternary_torch_ext.cu:123-191 and the PyTorch
    fallback ``TernaryExpertModule.forward_hidden`` python/real_model_demo.py:379-398
        g = s_g * (T_g x); u = s_u * (T_u x); h = silu(g) * u; y = s_d * (T_d h)
  * top-k combine         python/olmoe_extract.py:126-157
        out[t] = sum_k w[t,k] * expert_{ids[t,k]}(x[t])
  * per-matrix quantizer  python/micro_expert.py:185-203 and per-row
    quantizer python/real_model_demo.py:100-127

Accumulations run in float64: with bf16 (or integer) activations every
ternary sum is exact there, so the oracle's pre-scale accumulators are the
exact values the CUDA path is measured against.

The int8-activation path (no reference counterpart; the reference keeps fp32
activations) quantizes each token row symmetrically to int8 with scale
absmax/127 and accumulates ternary x int8 in int64.
"""

from __future__ import annotations

import numpy as np

TERN_PACK = 16


def pack_ternary(w_int8: np.ndarray) -> np.ndarray:
    """int8 [K, N] in {-1,0,+1} -> int32 [ceil(K/16), N] (reference layout)."""
    w = np.asarray(w_int8)
    K, N = w.shape
    P = (K + TERN_PACK - 1) // TERN_PACK
    codes = np.zeros((P * TERN_PACK, N), np.uint32)
    codes[:K][w > 0] = 1
    codes[:K][w < 0] = 2
    codes = codes.reshape(P, TERN_PACK, N)
    shifts = (2 * np.arange(TERN_PACK, dtype=np.uint32))[None, :, None]
    packed = np.bitwise_or.reduce(codes << shifts, axis=1)
    return packed.astype(np.uint32).view(np.int32)


def unpack_ternary(packed: np.ndarray, K: int) -> np.ndarray:
    """int32 [ceil(K/16), N] -> int8 [K, N] with the reference decode rule."""
    p = np.asarray(packed).view(np.uint32)
    P, N = p.shape
    shifts = (2 * np.arange(TERN_PACK, dtype=np.uint32))[None, :, None]
    codes = (p[:, None, :] >> shifts) & np.uint32(3)
    sign = (codes == 1).astype(np.int8) - (codes >> 1).astype(np.int8)
    return sign.reshape(P * TERN_PACK, N)[:K]


def silu(g: np.ndarray) -> np.ndarray:
    return g / (1.0 + np.exp(-g))


def ternary_linear(x, packed, scale, bias=None):
    """y = scale * (x @ T) + bias for the reference [ceil(K/16), N] layout."""
    x = np.asarray(x, np.float64)
    T = unpack_ternary(packed, x.shape[1]).astype(np.float64)
    y = (x @ T) * np.asarray(scale, np.float64)
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return y


def gated_mlp_accumulators(x, T_gate, T_up, T_down, s_gate, s_up):
    """Exact pre-scale accumulators and the hidden state.

    x [M,H] (values exactly representable in fp64), T_gate/T_up int8 [I,H],
    T_down int8 [H,I] (PyTorch [out, in] layout).  Returns (acc_g, acc_u, h).
    """
    x = np.asarray(x, np.float64)
    acc_g = x @ T_gate.astype(np.float64).T
    acc_u = x @ T_up.astype(np.float64).T
    g = acc_g * np.asarray(s_gate, np.float64)
    u = acc_u * np.asarray(s_up, np.float64)
    h = silu(g) * u
    return acc_g, acc_u, h


def gated_mlp(x, T_gate, T_up, T_down, s_gate, s_up, s_down):
    """Expert forward in the PyTorch [out, in] weight layout, float64."""
    _, _, h = gated_mlp_accumulators(x, T_gate, T_up, T_down, s_gate, s_up)
    return (h @ T_down.astype(np.float64).T) * np.asarray(s_down, np.float64)


def gated_mlp_packed(x, gate_packed, up_packed, down_packed, gs, us, ds):
    """``ternary_gated_mlp`` with reference-layout packed weights."""
    x = np.asarray(x, np.float64)
    H = x.shape[1]
    I = np.asarray(gate_packed).shape[1]
    Tg = unpack_ternary(gate_packed, H).T
    Tu = unpack_ternary(up_packed, H).T
    Td = unpack_ternary(down_packed, I).T
    return gated_mlp(x, Tg, Tu, Td, gs, us, ds)


def gated_mlp_f32(x, T_gate, T_up, T_down, s_gate, s_up, s_down):
    """fp32 restatement of TernaryExpertModule.forward_hidden (real_model_demo.py:379-398),
    including its per-call dequantization W = T * s; used to time the CPU path."""
    x = np.asarray(x, np.float32)
    gw = T_gate.astype(np.float32) * np.asarray(s_gate, np.float32)[:, None]
    uw = T_up.astype(np.float32) * np.asarray(s_up, np.float32)[:, None]
    dw = T_down.astype(np.float32) * np.asarray(s_down, np.float32)[:, None]
    g = x @ gw.T
    h = (g / (np.float32(1) + np.exp(-g))) * (x @ uw.T)
    return h @ dw.T


def moe_combine(x, ids, weights, experts, fp32: bool = False):
    """out[t] = sum_k weights[t,k] * expert_{ids[t,k]}(x[t]) (float64, or fp32 with ``fp32``).

    ``experts`` is a list of dicts in the container layout of
    python/real_model_demo.py:85-98.
    """
    dt = np.float32 if fp32 else np.float64
    x = np.asarray(x, dt)
    ids = np.asarray(ids)
    weights = np.asarray(weights, dt)
    out = np.zeros_like(x)
    f = gated_mlp_f32 if fp32 else gated_mlp
    for e in np.unique(ids):
        rows, slots = np.nonzero(ids == e)
        ex = experts[int(e)]
        y = f(x[rows], ex["gate_ternary"], ex["up_ternary"], ex["down_ternary"],
              ex["gate_scale"], ex["up_scale"], ex["down_scale"])
        np.add.at(out, rows, weights[rows, slots][:, None] * y)
    return out


def quantize_int8_rows(x):
    """Symmetric per-row int8: q = rint(x / s), s = absmax / 127 (s = 1 for zero rows)."""
    x = np.asarray(x, np.float32)
    amax = np.abs(x).max(axis=1)
    s = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(x / s[:, None]), -127, 127).astype(np.int8)
    return q, s


def int8_accumulate(q, T):
    """Exact int64 ternary x int8 accumulator: q [M,K] int8, T [N,K] int8 -> [M,N]."""
    return q.astype(np.int64) @ T.astype(np.int64).T


def quantize_ternary_per_matrix(w):
    """python/micro_expert.py:185-203: threshold = mean|w|, scale = mean|w| over non-zeros."""
    w = np.asarray(w, np.float32)
    thr = np.abs(w).mean()
    t = np.zeros(w.shape, np.int8)
    t[w > thr] = 1
    t[w < -thr] = -1
    mask = t != 0
    scale = np.float32(np.abs(w)[mask].mean()) if mask.any() else np.float32(1.0)
    return t, scale


def quantize_ternary_per_row(w):
    """python/real_model_demo.py:100-127: global threshold, per-row non-zero mean scale."""
    w = np.asarray(w, np.float32)
    thr = np.abs(w).mean()
    t = np.zeros(w.shape, np.int8)
    t[w > thr] = 1
    t[w < -thr] = -1
    mask = t != 0
    scale = np.ones(w.shape[0], np.float32)
    for i in range(w.shape[0]):
        if mask[i].any():
            scale[i] = np.abs(w[i])[mask[i]].mean()
    return t, scale
