"""The MoE layer (BVH router top-k -> grouped ternary SwiGLU) and its host pipeline (needs a B200).

The router is pinned to the oracle by test_router_gpu.py; here the layer output is
checked against the oracle's MoE combine fed with the GPU router's own ids and
weights (so the ternary contract, 1e-3 row-normwise, applies), and the host
pipeline against direct layer calls bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ternary as otern
from parity import ternary_errors

pytestmark = pytest.mark.gpu


def make_layer(device, E=16, H=256, I=128, seed=3):
    from bvh_router import BVHRouter, RouterConfig
    from sb200 import synth
    from sb200.moe import BVHMoELayer
    from sb200.ternary import TernaryExperts
    br = (2, 2, 4)
    w = synth.router_weights(H, 32, br, seed=seed, perturb=True)
    r = BVHRouter(RouterConfig(embed_dim=H, spectral_dim=32, branching=br))
    r.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()})
    r = r.to(device).eval()
    experts = synth.ternary_experts(E, H, I, seed=seed + 1)
    return BVHMoELayer(r, TernaryExperts(experts, device), top_k=4), experts


@pytest.mark.parametrize("B", [1, 37, 600])
def test_layer_matches_oracle_combine(cuda_device, B):
    from sb200 import synth
    layer, experts = make_layer(cuda_device)
    x = synth.hidden_states(B, 256, seed=B, dtype=torch.bfloat16, device=cuda_device)
    y = layer(x, out_dtype=torch.float32)
    ids, w = layer.route(x)
    assert y.shape == (B, 256) and y.dtype == torch.float32
    ref = otern.moe_combine(x.float().cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), experts)
    norm, elem = ternary_errors(y.cpu().numpy(), ref)
    assert norm <= 1e-3 and elem <= 5e-3, (norm, elem)


def test_host_pipeline_equals_direct_calls(cuda_device):
    from sb200 import synth
    from sb200.moe import HostPipeline
    layer, _ = make_layer(cuda_device)
    B, n = 300, 5
    xs = [synth.hidden_states(B, 256, seed=100 + i, dtype=torch.bfloat16) for i in range(n)]
    direct = [layer(x.to(cuda_device)).cpu() for x in xs]
    pipe = HostPipeline(layer, B, 256, dtype=torch.bfloat16, device=cuda_device)
    hx = [x.pin_memory() for x in xs]
    hy = [torch.empty(B, 256, dtype=torch.bfloat16).pin_memory() for _ in range(n)]
    pipe.run(hx, hy)
    torch.cuda.current_stream(cuda_device).synchronize()
    for a, b in zip(direct, hy):
        assert torch.equal(a, b)


@pytest.mark.parametrize("B", [37, 4096])
def test_graphed_layer_replays_the_eager_layer(cuda_device, B):
    """GraphedLayer (the layer captured into one CUDA graph) gives the eager
    layer's bits, picks up new input data in the same buffer, and feeds the
    host pipeline."""
    from sb200 import synth
    from sb200.moe import GraphedLayer, HostPipeline
    layer, _ = make_layer(cuda_device)
    g = GraphedLayer(layer)
    x = synth.hidden_states(B, 256, seed=B + 1, dtype=torch.bfloat16, device=cuda_device)
    out = torch.empty(B, 256, dtype=torch.bfloat16, device=cuda_device)
    g(x, out)
    assert torch.equal(out, layer(x))
    x.copy_(synth.hidden_states(B, 256, seed=B + 2, dtype=torch.bfloat16, device=cuda_device))
    g(x, out)
    assert torch.equal(out, layer(x))
    assert len(g._graphs) == 1
    pipe = HostPipeline(g, B, 256, dtype=torch.bfloat16, device=cuda_device)
    xs = [synth.hidden_states(B, 256, seed=50 + i, dtype=torch.bfloat16).pin_memory() for i in range(4)]
    ys = [torch.empty(B, 256, dtype=torch.bfloat16).pin_memory() for _ in range(4)]
    pipe.run(xs, ys)
    torch.cuda.synchronize()
    for xh, yh in zip(xs, ys):
        assert torch.equal(yh, layer(xh.to(cuda_device)).cpu())
