"""Drop-in module surface checks that need no GPU."""

from __future__ import annotations

import pytest
import torch

from conftest import load_golden


def test_state_dict_keys_match_reference():
    """A reference checkpoint loads unchanged: same keys and shapes (bvh_router.py:227-255)."""
    from bvh_router import BVHRouter, RouterConfig
    g = load_golden("router_small")
    ref_keys = {k[2:]: g[k].shape for k in g if k.startswith("w/")}
    r = BVHRouter(RouterConfig(embed_dim=64, spectral_dim=16))
    mine = {k: tuple(v.shape) for k, v in r.state_dict().items()}
    assert set(mine) == set(ref_keys)
    for k, shp in ref_keys.items():
        assert mine[k] == tuple(shp), k
    r.load_state_dict({k: torch.from_numpy(g["w/" + k]) for k in ref_keys})


def test_config_totals():
    from bvh_router import RouterConfig
    cfg = RouterConfig(n_level1=3, n_level2=5, n_level3=2)
    assert (cfg.total_l1, cfg.total_l2, cfg.total_l3, cfg.n_experts) == (3, 15, 30, 30)
    deep = RouterConfig(embed_dim=4096, spectral_dim=256, branching=(4,) * 6)
    assert deep.n_experts == 4096 and deep.n_levels == 6


def test_cpu_input_fails_loudly():
    from bvh_router import BVHRouter, RouterConfig
    r = BVHRouter(RouterConfig(embed_dim=64, spectral_dim=16)).eval()
    with pytest.raises(RuntimeError, match="CUDA"):
        r(torch.randn(4, 64))


def test_training_gumbel_forward_is_not_offered():
    from bvh_router import BVHRouter, RouterConfig
    r = BVHRouter(RouterConfig(embed_dim=64, spectral_dim=16)).train()
    with pytest.raises(NotImplementedError):
        r(torch.randn(4, 64))


def test_anneal_and_balance_bookkeeping():
    from bvh_router import BVHRouter, RouterConfig
    r = BVHRouter(RouterConfig(embed_dim=64, spectral_dim=16))
    r.anneal_temperature()
    assert abs(r.temperature.item() - 0.95) < 1e-6
    assert r.load_balancing_loss().item() == 0.0


def test_facade_and_hybrid_router_surface():
    import spectral_ai
    from bvh_router_bridge import HybridBVHRouter
    for name in ("BVHRouter", "RouterConfig", "RoutingResult", "HybridBVHRouter", "BVHMoELayer"):
        assert hasattr(spectral_ai, name)
    h = HybridBVHRouter(spectral_ai.RouterConfig(embed_dim=64, spectral_dim=16))
    assert all(k.startswith("pytorch_router.") for k in h.state_dict())
    h.anneal_temperature()
    assert h.load_balancing_loss().item() == 0.0
