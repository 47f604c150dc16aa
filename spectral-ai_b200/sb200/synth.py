"""Seeded synthetic inputs and random-init weights for the router and the
ternary expert layer.

There are no trained checkpoints or datasets for this path, so every workload
is generated from a fixed recipe.  The recipe is written once here and shared
by the golden-fixture script, the tests and the benchmark, so that no part of
the code depends on matching another RNG stream by accident.

Router recipe (state_dict names follow ``BVHRouter``, python/bvh_router.py:227-255):
  * Weights use a generator seeded with ``WEIGHT_STREAM + seed``.
  * Linears whose in_features is the hidden size (``to_3d``, ``spectral.net.0``,
    ``spectral.net.2``) get W ~ N(0, 1/H); the refraction Linears (in = S) get
    W ~ N(0, 1/S); biases are 0; centers ~ U[-1, 1]^3; log_radii = 0; portals
    are the identity; temperature = 1.0.  Draw order is fixed (see
    ``router_weights``).
  * ``perturb=True`` additionally draws non-zero biases, non-identity portals
    and a temperature != 1 so that every term of the forward is exercised.

Ternary recipe (ternary SwiGLU, python/real_model_demo.py:85-98 container):
  * T in {-1, 0, +1} with P = 1/3 each, one fp32 scale per expert matrix
    (``c / sqrt(fan_in)`` with c ~ U[0.5, 1.5)), broadcast to the per-channel
    scale vectors the reference kernel API takes.
Inputs (``hidden_states``) use a generator seeded with ``seed`` itself, so equal
seeds never give correlated router weights and inputs.
Routing recipe (MoE layer): each token picks ``k`` distinct experts by
Gumbel-top-k over Zipf(1.1) probabilities on a seeded expert permutation;
weights are the softmax of N(0, 1) logits.
"""

from __future__ import annotations

import math
from typing import Dict, List, Sequence

import numpy as np
import torch


WEIGHT_STREAM = 0x5B200000


def level_sizes(branching: Sequence[int]) -> List[int]:
    """Number of nodes on each level: level l has prod(branching[:l+1]) nodes."""
    out, n = [], 1
    for b in branching:
        n *= int(b)
        out.append(n)
    return out


def router_weights(hidden: int, spectral: int, branching: Sequence[int] = (4, 4, 4),
                   seed: int = 0, perturb: bool = False,
                   temperature: float = 1.0) -> Dict[str, np.ndarray]:
    """fp32 router parameters keyed by ``BVHRouter`` state_dict names."""
    # weights draw from their own stream: with the same seed as the inputs the
    # first weight rows would equal the first input rows
    g = torch.Generator().manual_seed(WEIGHT_STREAM + seed)
    H, S = hidden, spectral
    sizes = level_sizes(branching)
    L = len(sizes)
    w: Dict[str, np.ndarray] = {}

    def randn(*shape, std):
        return (torch.randn(*shape, generator=g) * std).numpy().astype(np.float32)

    w["to_3d.weight"] = randn(3, H, std=1.0 / math.sqrt(H))
    w["spectral.net.0.weight"] = randn(H, H, std=1.0 / math.sqrt(H))
    w["spectral.net.2.weight"] = randn(S, H, std=1.0 / math.sqrt(H))
    for l in range(L):
        w[f"refract{l + 1}.W_dispersion.weight"] = randn(sizes[l], S, std=1.0 / math.sqrt(S))
    for l in range(L):
        c = torch.rand(sizes[l], 3, generator=g) * 2.0 - 1.0
        w[f"level{l + 1}.centers"] = c.numpy().astype(np.float32)
    if perturb:
        w["to_3d.bias"] = randn(3, std=0.1)
        w["spectral.net.0.bias"] = randn(H, std=0.1)
        w["spectral.net.2.bias"] = randn(S, std=0.1)
        for l in range(L):
            w[f"refract{l + 1}.W_dispersion.bias"] = randn(sizes[l], std=0.5)
        for l in range(L - 1):
            eye = np.zeros((sizes[l], 3, 4), np.float32)
            for i in range(3):
                eye[:, i, i] = 1.0
            w[f"portal{l + 1}.transform"] = eye + randn(sizes[l], 3, 4, std=0.2)
    else:
        w["to_3d.bias"] = np.zeros(3, np.float32)
        w["spectral.net.0.bias"] = np.zeros(H, np.float32)
        w["spectral.net.2.bias"] = np.zeros(S, np.float32)
        for l in range(L):
            w[f"refract{l + 1}.W_dispersion.bias"] = np.zeros(sizes[l], np.float32)
        for l in range(L - 1):
            eye = np.zeros((sizes[l], 3, 4), np.float32)
            for i in range(3):
                eye[:, i, i] = 1.0
            w[f"portal{l + 1}.transform"] = eye
    for l in range(L):
        w[f"level{l + 1}.log_radii"] = np.zeros(sizes[l], np.float32)
    w["temperature"] = np.array(temperature, np.float32)
    w["expert_counts"] = np.zeros(sizes[-1], np.float32)
    return w


def enhanced_router_weights(hidden: int = 2048, branching: Sequence[int] = (4, 4, 4), feature_dim: int = 128,
                            seed: int = 0, perturb: bool = True,
                            temperature: float = 1.0) -> Dict[str, np.ndarray]:
    """fp32 parameters keyed by ``EnhancedBVHRouter`` state_dict names
    (python/olmoe_bvh_distill.py:422-516, spectral_mode off): Linear weights
    N(0, 1/in), centers N(0, 0.3^2); with ``perturb`` the biases, the LayerNorm
    affine and log-radii move off their initial values too."""
    g = torch.Generator().manual_seed(WEIGHT_STREAM + 0x1000 + seed)
    n1, n2, n3 = branching
    F = feature_dim
    w: Dict[str, np.ndarray] = {}

    def randn(*shape, std):
        return (torch.randn(*shape, generator=g) * std).numpy().astype(np.float32)

    def linear(name, n_in, n_out):
        w[name + ".weight"] = randn(n_out, n_in, std=1.0 / math.sqrt(n_in))
        w[name + ".bias"] = randn(n_out, std=0.1) if perturb else np.zeros(n_out, np.float32)

    w["temperature"] = np.array(temperature, np.float32)
    w["expert_counts"] = np.zeros(n1 * n2 * n3, np.float32)
    linear("input_proj.0", hidden, 512)
    linear("input_proj.2", 512, 256)
    if perturb:
        w["input_proj.3.weight"] = (1.0 + randn(256, std=0.1)).astype(np.float32)
        w["input_proj.3.bias"] = randn(256, std=0.1)
    else:
        w["input_proj.3.weight"] = np.ones(256, np.float32)
        w["input_proj.3.bias"] = np.zeros(256, np.float32)
    for l, (n_in, k) in enumerate(((256, n1), (F, n2), (F, n3)), start=1):
        w[f"level{l}.centers"] = randn(k, 3, std=0.3)
        w[f"level{l}.log_radii"] = randn(k, std=0.1) if perturb else np.zeros(k, np.float32)
        linear(f"level{l}.to_3d", n_in, 3)
        linear(f"level{l}.feature_net.0", n_in, F)
        linear(f"level{l}.feature_net.2", F, F)
        linear(f"level{l}.route_head", F + 3, k)
    linear("expert_head.0", F + n1 + n2 + n3, 256)
    linear("expert_head.2", 256, n1 * n2 * n3)
    return w


def dense_gate_weight(n_experts: int, hidden: int, seed: int = 0, gain: float = 2.0) -> np.ndarray:
    """A layer's dense top-k gate ``nn.Linear(hidden, n_experts, bias=False)``
    weight for the hybrid pre-filter: N(0, gain^2 / hidden), so unit-RMS
    tokens get logits of standard deviation ``gain``."""
    g = torch.Generator().manual_seed(WEIGHT_STREAM + 0x2000 + seed)
    return (torch.randn(n_experts, hidden, generator=g) * (gain / math.sqrt(hidden))).numpy().astype(np.float32)


def mlp_experts(n_experts: int, hidden: int, inner: int, seed: int = 0) -> List[Dict[str, np.ndarray]]:
    """State dicts of small dense experts ``Sequential(Linear(hidden, inner),
    GELU(), Linear(inner, hidden))`` (keys 0.weight, 0.bias, 2.weight,
    2.bias; N(0, 1/in) weights, N(0, 0.1^2) biases) for pipeline tests."""
    g = torch.Generator().manual_seed(WEIGHT_STREAM + 0x3000 + seed)
    out = []
    for _ in range(n_experts):
        out.append({"0.weight": (torch.randn(inner, hidden, generator=g) / math.sqrt(hidden)).numpy(),
                    "0.bias": (torch.randn(inner, generator=g) * 0.1).numpy(),
                    "2.weight": (torch.randn(hidden, inner, generator=g) / math.sqrt(inner)).numpy(),
                    "2.bias": (torch.randn(hidden, generator=g) * 0.1).numpy()})
    return out


def calibration_linear(n_experts: int, seed: int = 0) -> Dict[str, np.ndarray]:
    """A Linear(E, E) calibration state (weight = I + N(0, 0.05^2), bias N(0, 0.1^2))."""
    g = torch.Generator().manual_seed(WEIGHT_STREAM + 0x4000 + seed)
    w = torch.eye(n_experts) + torch.randn(n_experts, n_experts, generator=g) * 0.05
    return {"weight": w.numpy().astype(np.float32), "bias": (torch.randn(n_experts, generator=g) * 0.1).numpy()}


def legacy_tree(seed: int = 0) -> Dict[str, np.ndarray]:
    """Parameters of the legacy 85-node ray-sphere tree (root, 4, 16, 64 leaves)
    in the layout bvh_upload_tree takes: centers [85,3] (children scattered
    around their parent at shrinking scale), radii [85] in [0.2, 0.5), portals
    [85,12] (3x4 identity plus N(0, 0.05^2) and a small translation),
    snell_w [85,64] N(0, 1/64), snell_b [85] N(0, 0.1^2)."""
    g = torch.Generator().manual_seed(WEIGHT_STREAM + 0x5000 + seed)
    c = np.zeros((85, 3), np.float32)
    for n in range(1, 85):
        parent = (n - 1) // 4
        depth = 1 if n < 5 else (2 if n < 21 else 3)
        c[n] = c[parent] + (torch.randn(3, generator=g) * (1.2 / depth)).numpy()
    radii = (0.2 + 0.3 * torch.rand(85, generator=g)).numpy().astype(np.float32)
    eye = np.concatenate([np.eye(3, dtype=np.float32), np.zeros((3, 1), np.float32)], axis=1)
    portals = (eye[None] + (torch.randn(85, 3, 4, generator=g) * 0.05).numpy()).astype(np.float32)
    return {"centers": c, "radii": radii, "portals": portals.reshape(85, 12),
            "snell_w": (torch.randn(85, 64, generator=g) / 8.0).numpy().astype(np.float32),
            "snell_b": (torch.randn(85, generator=g) * 0.1).numpy().astype(np.float32)}


def rays(batch: int, seed: int):
    """Ray origins N(0, 0.5^2) and unit directions [B,3], fp32."""
    g = torch.Generator().manual_seed(seed)
    o = torch.randn(batch, 3, generator=g) * 0.5
    d = torch.randn(batch, 3, generator=g)
    d = d / d.norm(dim=1, keepdim=True)
    return o.numpy().astype(np.float32), d.numpy().astype(np.float32)


def unit_rms_rows(x: torch.Tensor) -> torch.Tensor:
    """Divide each row by its root-mean-square (fp32)."""
    rms = x.float().pow(2).mean(dim=-1, keepdim=True).sqrt()
    return x.float() / rms


def hidden_states(batch: int, hidden: int, seed: int, dtype=torch.float32,
                  device="cpu") -> torch.Tensor:
    """Unit-RMS Gaussian rows; generated on ``device`` with a seeded generator."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(batch, hidden, generator=g, device=device, dtype=torch.float32)
    return unit_rms_rows(x).to(dtype)


def ternary_experts(n_experts: int, hidden: int, inter: int, seed: int = 2):
    """Ternary SwiGLU experts in the reference container layout.

    Returns a list of dicts with ``gate_ternary [I,H]``, ``up_ternary [I,H]``,
    ``down_ternary [H,I]`` (int8) and per-channel fp32 scale vectors holding one
    constant per matrix.
    """
    rng = np.random.default_rng(seed)
    out = []
    for e in range(n_experts):
        d = {"expert_id": e}
        for name, shape, fan_in in (("gate", (inter, hidden), hidden),
                                    ("up", (inter, hidden), hidden),
                                    ("down", (hidden, inter), inter)):
            t = rng.integers(-1, 2, size=shape, dtype=np.int8)
            c = rng.uniform(0.5, 1.5)
            d[f"{name}_ternary"] = t
            d[f"{name}_scale"] = np.full(shape[0], c / math.sqrt(fan_in), np.float32)
        out.append(d)
    return out


def zipf_routing(n_tokens: int, n_experts: int, k: int, seed: int, alpha: float = 1.1):
    """Top-k expert ids (int32 [B,k], distinct per row) and weights (fp32 [B,k]).

    Experts are ranked by a seeded permutation and drawn without replacement
    with Zipf(alpha) probabilities through the Gumbel-top-k trick; weights are
    softmax(N(0,1)) over the k slots.
    """
    rng = np.random.default_rng(seed)
    perm = rng.permutation(n_experts)
    p = 1.0 / np.arange(1, n_experts + 1, dtype=np.float64) ** alpha
    logp = np.log(p / p.sum())
    keys = logp[None, :] + rng.gumbel(size=(n_tokens, n_experts))
    ranks = np.argsort(-keys, axis=1, kind="stable")[:, :k]
    ids = perm[ranks].astype(np.int32)
    logits = rng.standard_normal((n_tokens, k))
    wts = np.exp(logits - logits.max(axis=1, keepdims=True))
    wts = (wts / wts.sum(axis=1, keepdims=True)).astype(np.float32)
    return ids, wts
