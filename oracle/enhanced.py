"""CPU restatement of the EnhancedBVHRouter eval forward and the BVHGateWrapper
top-k conventions (test infrastructure only).

This module is the parity checker for the CUDA enhanced router.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import it; the product path never does.

It restates, in numpy fp32, op by op (spectral_mode off, n_rays = 1):
  * ``input_proj``  Linear(H,512) -> GELU(erf) -> Linear(512,256) -> LayerNorm(256)
                    python/olmoe_bvh_distill.py:459-465, 597
  * ``HierarchicalLevel.forward`` (eval)           olmoe_bvh_distill.py:366-419
      pos = to_3d(x); d2 = |pos - c_k|^2; geo = -d2 / (2 T^2 + 1e-8)
      f = Linear(F,F)(GELU(Linear(in,F)(x)))
      logits = route_head([f, pos]) + 0.5 geo; p = softmax(logits / max(T, 0.1))
  * ``EnhancedBVHRouter._forward_from_h``         olmoe_bvh_distill.py:518-585
      level chain h -> f1 -> f2 -> f3; geometric distances to the 64 leaves
      d1[i] + d2[j] + d3[k] with d = sqrt(d2 + 1e-8); branch bonus
      1 + 0.2 [same domain] + 0.1 [same subdomain] from the level argmaxes;
      logits = expert_head([f3, p1, p2, p3])
  * ``EnhancedBVHRouter.forward`` (eval)           olmoe_bvh_distill.py:593-632
      expert_probs = softmax(logits / max(T, 0.1)); expert_ids = argmax
  * ``BVHGateWrapper.forward``                     python/olmoe_e2e_eval.py:316-971
      logits rounded to the hidden-state dtype, then
      "softmax" (:928-938): router_probs = softmax(logits) over all experts,
        top-k of it, renormalised when norm_topk_prob;
      "topk_softmax" (:521-529): top-k of the logits, softmax over those k,
        router_probs = those k weights scattered into zeros.
  * the hybrid pre-filter gate of ``replace_gate_with_bvh(hybrid=True)``
                                                   python/olmoe_e2e_eval.py:1264-1296
      BVH top-n candidates, the dense gate's full fp32 softmax, top-k of it
      restricted to the candidates.

Parity: pinned against the reference's own outputs through the committed
fixtures tests/golden/enhanced_*.npz (tests/golden/make_golden.py imports the
reference EnhancedBVHRouter and BVHGateWrapper).
"""

from __future__ import annotations

from typing import Dict, Tuple

import numpy as np

from .router import F32, gelu_erf, linear, softmax


def layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """nn.LayerNorm: biased variance over the last axis, fp32."""
    x = x.astype(F32)
    mu = x.mean(axis=-1, keepdims=True, dtype=np.float64).astype(F32)
    xc = x - mu
    var = (xc * xc).mean(axis=-1, keepdims=True, dtype=np.float64).astype(F32)
    return (xc / np.sqrt(var + F32(eps)) * w + b).astype(F32)


def input_proj(w: Dict[str, np.ndarray], x: np.ndarray) -> np.ndarray:
    g = gelu_erf(linear(x, w["input_proj.0.weight"], w["input_proj.0.bias"]))
    p = linear(g, w["input_proj.2.weight"], w["input_proj.2.bias"])
    return layer_norm(p, w["input_proj.3.weight"], w["input_proj.3.bias"])


def hierarchical_level(w: Dict[str, np.ndarray], name: str, x: np.ndarray, T: float):
    """(probs [B,K], features [B,F], pos [B,3]) — olmoe_bvh_distill.py:366-419, eval."""
    pos = linear(x, w[f"{name}.to_3d.weight"], w[f"{name}.to_3d.bias"])
    c = w[f"{name}.centers"].astype(F32)
    diff = pos[:, None, :] - c[None, :, :]
    d2 = (diff * diff).sum(axis=-1, dtype=F32)
    geo = (-d2 / F32(2.0 * T * T + 1e-8)).astype(F32)
    h = gelu_erf(linear(x, w[f"{name}.feature_net.0.weight"], w[f"{name}.feature_net.0.bias"]))
    f = linear(h, w[f"{name}.feature_net.2.weight"], w[f"{name}.feature_net.2.bias"])
    logits = linear(np.concatenate([f, pos], axis=1), w[f"{name}.route_head.weight"],
                    w[f"{name}.route_head.bias"])
    logits = (logits + F32(0.5) * geo).astype(F32)
    probs = softmax(logits / F32(max(T, 0.1)))
    return probs, f, pos


def _leaf_distance(pos: np.ndarray, c: np.ndarray) -> np.ndarray:
    diff = pos[:, None, :] - c[None, :, :].astype(F32)
    return np.sqrt((diff * diff).sum(axis=-1, dtype=F32) + F32(1e-8)).astype(F32)


def forward_from_h(w: Dict[str, np.ndarray], h: np.ndarray, T: float):
    """logits [B,64] plus the side outputs (geometric distances [B,64], branch
    bonus [B,64], level probabilities) — olmoe_bvh_distill.py:518-585."""
    p1, f1, pos1 = hierarchical_level(w, "level1", h, T)
    p2, f2, pos2 = hierarchical_level(w, "level2", f1, T)
    p3, f3, pos3 = hierarchical_level(w, "level3", f2, T)
    n1, n2, n3 = p1.shape[1], p2.shape[1], p3.shape[1]
    d1 = _leaf_distance(pos1, w["level1.centers"])
    d2 = _leaf_distance(pos2, w["level2.centers"])
    d3 = _leaf_distance(pos3, w["level3.centers"])
    geo = ((d1[:, :, None, None] + d2[:, None, :, None]) + d3[:, None, None, :]).reshape(h.shape[0], -1)
    e = np.arange(n1 * n2 * n3)
    same1 = (e[None, :] // (n2 * n3)) == p1.argmax(axis=1)[:, None]
    same2 = ((e[None, :] % (n2 * n3)) // n3) == p2.argmax(axis=1)[:, None]
    bonus = (F32(1.0) + F32(0.2) * same1.astype(F32) + F32(0.1) * same2.astype(F32)).astype(F32)
    z = gelu_erf(linear(np.concatenate([f3, p1, p2, p3], axis=1), w["expert_head.0.weight"],
                        w["expert_head.0.bias"]))
    logits = linear(z, w["expert_head.2.weight"], w["expert_head.2.bias"])
    return logits, {"geo_dist": geo.astype(F32), "branch_bonus": bonus, "p1": p1, "p2": p2, "p3": p3}


def router_forward(w: Dict[str, np.ndarray], x: np.ndarray):
    """EnhancedBVHRouter eval forward: (expert_probs [B,64], expert_ids [B], logits, side)."""
    T = float(np.asarray(w["temperature"]))
    h = input_proj(w, x.astype(F32))
    logits, side = forward_from_h(w, h, T)
    probs = softmax(logits / F32(max(T, 0.1)))
    side["h"] = h
    return probs, probs.argmax(axis=1), logits, side


def topk_desc(v: np.ndarray, k: int) -> Tuple[np.ndarray, np.ndarray]:
    """torch.topk order: largest first, equal values toward the lower index."""
    idx = np.argsort(-v, axis=1, kind="stable")[:, :k]
    return np.take_along_axis(v, idx, axis=1), idx


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """The wrapper's ``logits.to(hidden_states.dtype)``: bf16 rounds to nearest even."""
    if dtype == "f32":
        return x.astype(F32)
    u = x.astype(F32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    return u.astype(np.uint32).view(F32)


def gate_topk(logits: np.ndarray, k: int = 8, mode: str = "softmax", norm_topk_prob: bool = False,
              dtype: str = "f32"):
    """BVHGateWrapper weights: (router_probs [B,E] f32, top-k weights [B,k] f32
    before the cast to the hidden dtype, top-k ids [B,k])."""
    lg = round_to(logits, dtype)
    if mode == "softmax":
        probs = softmax(lg)
        wts, ids = topk_desc(probs, k)
        if norm_topk_prob:
            wts = (wts / wts.sum(axis=1, keepdims=True)).astype(F32)
        return probs, wts, ids
    if mode == "topk_softmax":
        vals, ids = topk_desc(lg, k)
        wts = softmax(vals)
        probs = np.zeros_like(lg, dtype=F32)
        np.put_along_axis(probs, ids, wts, axis=1)
        return probs, wts, ids
    raise ValueError(f"weight mode {mode!r} is not restated")


def dense_gate_logits(x: np.ndarray, w_gate: np.ndarray, dtype: str = "f32") -> np.ndarray:
    """full_logits = F.linear(h2d, W_gate) in the hidden dtype
    (python/olmoe_e2e_eval.py:1278): fp32 products accumulated in float64 here,
    then rounded to the hidden dtype (bf16: round-to-nearest-even)."""
    acc = (np.asarray(x, np.float64) @ np.asarray(w_gate, np.float64).T).astype(F32)
    return round_to(acc, dtype)


def hybrid_gate(bvh_probs: np.ndarray, full_logits: np.ndarray, n_candidates: int, k: int = 8,
                norm_topk_prob: bool = False):
    """The hybrid pre-filter of replace_gate_with_bvh(hybrid=True),
    python/olmoe_e2e_eval.py:1264-1296:
      candidate_ids = topk(bvh_probs, n_candidates)
      full_probs    = softmax(full_logits, fp32) over all experts
      top-k of full_probs gathered at the candidates, mapped back to expert
      ids, renormalised when norm_topk_prob.
    Returns (full_probs [B,E], top-k weights [B,k] f32 before the cast to the
    hidden dtype, top-k ids [B,k])."""
    _, cand = topk_desc(np.asarray(bvh_probs, F32), n_candidates)
    full = softmax(np.asarray(full_logits, F32))
    cprob = np.take_along_axis(full, cand, axis=1)
    vals, local = topk_desc(cprob, k)
    ids = np.take_along_axis(cand, local, axis=1)
    if norm_topk_prob:
        vals = (vals / vals.sum(axis=1, keepdims=True)).astype(F32)
    return full, vals, ids
