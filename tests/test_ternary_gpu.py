"""Ternary SwiGLU kernels against the CPU oracle (needs a B200).

Contract: outputs after the fp32 scales within 1e-3 relative.

* fp32 inputs (the reference API's dtype) take the fp32-faithful form: x and
  the SwiGLU hidden state h enter the tensor cores as bf16 hi/lo pairs (each
  value to 2^-16, with fp32's exponent range), accumulation fp32.  Held to
  1e-4 row-normwise and, elementwise, 1e-3 relative to |y_ref| + 0.1 rms(row):
  1e-3 relative for every output of at least a tenth of its row's RMS, and
  1e-4 of the row RMS absolutely for smaller ones (no elementwise bound can be
  purely relative: any two fp32 summation orders, the reference's own CPU and
  GPU paths included, differ by far more than 1e-3 of an output that cancels
  to near zero).
* bf16 inputs (the MoE layer's hot path) keep bf16 activations and round h to
  fp16 (2^-11) before the down projection: 1e-3 row-normwise and 2e-3
  elementwise relative to |y_ref| + rms(row).  An |h| beyond fp16's 65504
  turns the output non-finite, which the layer reports through the device
  status word.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import ternary as otern
from parity import ternary_errors

pytestmark = pytest.mark.gpu

NORM_TOL = 1e-3
ELEM_TOL = 2e-3
FP32_NORM_TOL = 1e-4
FP32_ELEM_TOL = 1e-3
FP32_FLOOR = 0.1

# the grouped GEMM engines (SB_TERNARY_ENGINE): CTA pairs (default), one CTA
# with the weights in TMEM, one CTA with the weights in shared memory
ENGINES = ["pair", "ts", "ss"]


@pytest.fixture
def engine(request, monkeypatch):
    monkeypatch.setenv("SB_TERNARY_ENGINE", request.param)
    return request.param


def experts_from_golden(g, prefix, n):
    keys = ("gate_ternary", "up_ternary", "down_ternary", "gate_scale", "up_scale", "down_scale")
    return [{k: g[f"{prefix}{e}/{k}"] for k in keys} for e in range(n)]


def assert_close(got, ref, what):
    norm, elem = ternary_errors(got, ref)
    print(f"{what}: normwise {norm:.3e} elementwise {elem:.3e}")
    assert norm <= NORM_TOL, f"{what}: normwise {norm}"
    assert elem <= ELEM_TOL, f"{what}: elementwise {elem}"


def assert_fp32_faithful(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    d = np.abs(got - ref)
    rms = np.sqrt((ref * ref).mean(axis=1, keepdims=True)) + 1e-30
    norm = float((np.sqrt((d * d).sum(axis=1)) / (np.sqrt((ref * ref).sum(axis=1)) + 1e-30)).max())
    elem = float((d / (np.abs(ref) + FP32_FLOOR * rms)).max())
    print(f"{what}: normwise {norm:.3e} elementwise {elem:.3e}")
    assert norm <= FP32_NORM_TOL, f"{what}: normwise {norm}"
    assert elem <= FP32_ELEM_TOL, f"{what}: elementwise {elem}"


def _olmoe_expert(cuda_device, seed=21, H=2048, I=1024):
    from sb200 import synth
    ex = synth.ternary_experts(1, H, I, seed=seed)[0]
    packs = [torch.from_numpy(otern.pack_ternary(ex[f"{n}_ternary"].T.copy())).to(cuda_device)
             for n in ("gate", "up", "down")]
    s = [torch.from_numpy(ex[f"{n}_scale"]).to(cuda_device) for n in ("gate", "up", "down")]
    return ex, packs, s


def _oracle(ex, x):
    return otern.gated_mlp(np.asarray(x, np.float64), ex["gate_ternary"], ex["up_ternary"], ex["down_ternary"],
                           ex["gate_scale"], ex["up_scale"], ex["down_scale"])


@pytest.mark.parametrize("M", [1, 3, 130, 512])
def test_gated_mlp_fp32_input_is_fp32_faithful(cuda_device, M):
    from sb200 import synth
    import ternary_expert_ext as ext
    ex, packs, s = _olmoe_expert(cuda_device)
    x = synth.hidden_states(M, 2048, seed=24, device=cuda_device)          # fp32
    y = ext.ternary_gated_mlp(x, *packs, *s)
    assert_fp32_faithful(y.cpu().numpy(), _oracle(ex, x.cpu().numpy()), f"fp32 expert M={M}")


@pytest.mark.parametrize("scale", [1e3, 1e4])
def test_large_magnitude_rows(cuda_device, scale):
    """Rows scaled far past unit RMS: the fp32 path keeps fp32's range (bf16
    hi/lo terms) and its accuracy; on the bf16 path the fp16 hidden state
    overflows and the library reports the non-finite output."""
    from sb200 import _lib, synth
    from sb200.ternary import TernaryExperts
    import ternary_expert_ext as ext
    ex, packs, s = _olmoe_expert(cuda_device, seed=25)
    x = synth.hidden_states(64, 2048, seed=26, device=cuda_device) * scale
    y = ext.ternary_gated_mlp(x, *packs, *s)
    torch.cuda.synchronize()
    assert _lib.load().sb_device_status(0) == 0
    assert_fp32_faithful(y.cpu().numpy(), _oracle(ex, x.cpu().numpy()), f"rows x{scale:g} fp32")
    te = TernaryExperts([ex], cuda_device)
    ids = torch.zeros(64, 1, dtype=torch.int32, device=cuda_device)
    w = torch.ones(64, 1, device=cuda_device)
    yb = te.forward(x.bfloat16(), ids, w)
    torch.cuda.synchronize()
    assert not torch.isfinite(yb).all()
    assert _lib.load().sb_device_status(0) == -1
    assert "non-finite" in _lib.last_error()


def _reference_extension():
    import glob
    import importlib.util
    from pathlib import Path
    so = glob.glob(str(Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "ternary_expert_ext_ref*.so"))
    if not so:
        return None
    spec = importlib.util.spec_from_file_location("ternary_expert_ext_ref", so[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("M", [1, 3, 130, 512])
def test_gated_mlp_matches_reference_kernel(cuda_device, M):
    """The reference's own ternary_gated_mlp kernel (cuda/v5/ternary_torch_ext.cu,
    compiled from its source into oracle/_ref) run on this GPU on the same
    packed weights and fp32 tokens: the drop-in agrees with it to the fp32
    contract, and both agree with the float64 oracle."""
    ref = _reference_extension()
    if ref is None:
        pytest.skip("reference extension not built (oracle/build_ref.py)")
    from sb200 import synth
    import ternary_expert_ext as ext
    ex = synth.ternary_experts(1, 2048, 1024, seed=27)[0]
    packs = [ref.pack_ternary(torch.from_numpy(ex[f"{n}_ternary"].T.copy())).to(cuda_device)
             for n in ("gate", "up", "down")]
    s = [torch.from_numpy(ex[f"{n}_scale"]).to(cuda_device) for n in ("gate", "up", "down")]
    x = synth.hidden_states(M, 2048, seed=28, device=cuda_device)
    y_ref = ref.ternary_gated_mlp(x, *packs, *s)
    y = ext.ternary_gated_mlp(x, *packs, *s)
    torch.cuda.synchronize()
    exact = _oracle(ex, x.cpu().numpy())
    assert_fp32_faithful(y_ref.cpu().numpy(), exact, f"reference kernel M={M} vs oracle")
    assert_fp32_faithful(y.cpu().numpy(), y_ref.cpu().numpy(), f"ours vs reference kernel M={M}")


def test_repack_matches_host_layout(cuda_device):
    from sb200.ternary import pack_device, repack_reference
    rng = np.random.default_rng(1)
    for K, N in [(72, 40), (2048, 1024), (1024, 2048), (37, 29)]:
        T = rng.integers(-1, 2, size=(N, K), dtype=np.int8)     # [out, in]
        ref_packed = torch.from_numpy(otern.pack_ternary(T.T.copy())).to(cuda_device)
        dev = repack_reference(ref_packed, K).cpu().numpy().view(np.uint32)
        assert np.array_equal(dev, pack_device(T))


@pytest.mark.parametrize("engine", ENGINES, indirect=True)
@pytest.mark.parametrize("xdtype", [torch.float32, torch.bfloat16])
def test_gated_mlp_matches_reference_golden(cuda_device, xdtype, engine):
    """Reference API ternary_gated_mlp on the golden expert (H=72, I=40: ragged K and N)."""
    import ternary_expert_ext as ext
    g = load_golden("ternary_small")
    gp = torch.from_numpy(otern.pack_ternary(g["e/gate_ternary"].T.copy())).to(cuda_device)
    up = torch.from_numpy(otern.pack_ternary(g["e/up_ternary"].T.copy())).to(cuda_device)
    dp = torch.from_numpy(otern.pack_ternary(g["e/down_ternary"].T.copy())).to(cuda_device)
    s = [torch.from_numpy(g[f"e/{n}_scale"]).to(cuda_device) for n in ("gate", "up", "down")]
    x = torch.from_numpy(g["e/x"]).to(xdtype).to(cuda_device)
    y = ext.ternary_gated_mlp(x, gp, up, dp, *s)
    assert y.dtype == torch.float32 and y.shape == (24, 72)
    ref = otern.gated_mlp(x.float().cpu().numpy(), g["e/gate_ternary"], g["e/up_ternary"],
                          g["e/down_ternary"], g["e/gate_scale"], g["e/up_scale"], g["e/down_scale"])
    assert_close(y.cpu().numpy(), ref, "golden expert")
    if xdtype == torch.float32:   # the reference's own output (torch fallback math)
        assert_close(y.cpu().numpy(), g["e/y"], "golden expert vs reference")


@pytest.mark.parametrize("M", [1, 3, 130, 512])
def test_gated_mlp_olmoe_shape(cuda_device, M):
    from sb200 import synth
    import ternary_expert_ext as ext
    ex = synth.ternary_experts(1, 2048, 1024, seed=21)[0]
    gp = torch.from_numpy(otern.pack_ternary(ex["gate_ternary"].T.copy())).to(cuda_device)
    up = torch.from_numpy(otern.pack_ternary(ex["up_ternary"].T.copy())).to(cuda_device)
    dp = torch.from_numpy(otern.pack_ternary(ex["down_ternary"].T.copy())).to(cuda_device)
    s = [torch.from_numpy(ex[f"{n}_scale"]).to(cuda_device) for n in ("gate", "up", "down")]
    x = synth.hidden_states(M, 2048, seed=22, dtype=torch.bfloat16, device=cuda_device)
    y = ext.ternary_gated_mlp(x, gp, up, dp, *s)
    ref = otern.gated_mlp(x.float().cpu().numpy(), ex["gate_ternary"], ex["up_ternary"],
                          ex["down_ternary"], ex["gate_scale"], ex["up_scale"], ex["down_scale"])
    assert_close(y.cpu().numpy(), ref, f"expert M={M}")
    # a second call with the same packed tensors reuses their device layout
    assert torch.equal(ext.ternary_gated_mlp(x, gp, up, dp, *s), y)


@pytest.mark.parametrize("M", [5, 200, 4096])
@pytest.mark.parametrize("xdtype", [torch.float32, torch.bfloat16])
def test_gated_mlp_equals_the_routed_single_expert(cuda_device, M, xdtype):
    """Past the few-token sizes ternary_gated_mlp reads the rows in place and
    lets the down GEMM store y (no dispatch copy, no combine); it equals the
    routed layer with one expert and weight 1 bit for bit."""
    from sb200 import synth
    from sb200 import ternary as T
    from sb200.ternary import TernaryExperts
    H, I = 2048, 1024
    te = TernaryExperts(synth.ternary_experts(1, H, I, seed=23), cuda_device)
    x = synth.hidden_states(M, H, seed=24, dtype=xdtype, device=cuda_device)
    y = T.gated_mlp(x, te.gate, te.up, te.down, te.gate_scale[0], te.up_scale[0], te.down_scale[0], H, I)
    ids = torch.zeros(M, 1, dtype=torch.int32, device=cuda_device)
    w = torch.ones(M, 1, device=cuda_device)
    y_routed = te.forward(x, ids, w, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32 and y.shape == (M, H)
    assert torch.equal(y, y_routed), f"max |diff| {(y - y_routed).abs().max()}"


def test_ternary_linear(cuda_device):
    import ternary_expert_ext as ext
    rng = np.random.default_rng(3)
    for K, N, M in [(72, 40, 5), (2048, 1024, 300), (1000, 300, 129)]:
        T = rng.integers(-1, 2, size=(K, N), dtype=np.int8)   # reference packs [in, out]
        packed = torch.from_numpy(otern.pack_ternary(T)).to(cuda_device)
        scale = torch.from_numpy(rng.uniform(0.01, 0.1, N).astype(np.float32)).to(cuda_device)
        bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to(cuda_device)
        x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(cuda_device)
        y = ext.ternary_linear(x, packed, scale, bias)
        ref = otern.ternary_linear(x.cpu().numpy(), otern.pack_ternary(T), scale.cpu().numpy(),
                                   bias.cpu().numpy())
        assert_close(y.cpu().numpy(), ref, f"linear {K}x{N}")


@pytest.mark.parametrize("engine", ENGINES, indirect=True)
def test_moe_combine_golden(cuda_device, engine):
    """Grouped MoE SwiGLU against the reference OLMoE forward_topk golden (6 experts, top-3)."""
    from sb200.ternary import TernaryExperts
    g = load_golden("ternary_small")
    experts = experts_from_golden(g, "moe/", 6)
    te = TernaryExperts(experts, cuda_device)
    x = torch.from_numpy(g["moe/x"]).to(cuda_device)
    ids = torch.from_numpy(g["moe/ids"]).to(cuda_device)
    w = torch.from_numpy(g["moe/probs"]).to(cuda_device)
    y = te.forward(x, ids, w)
    assert_close(y.cpu().numpy(), g["moe/y"], "moe golden vs reference")
    ref = otern.moe_combine(g["moe/x"], g["moe/ids"], g["moe/probs"], experts)
    assert_close(y.cpu().numpy(), ref, "moe golden vs oracle")


@pytest.mark.parametrize("engine", ENGINES, indirect=True)
def test_moe_config2_sampled(cuda_device, engine):
    """Config 2: 64 experts, 2048->1024->2048, 4096 tokens x top-8 with Zipf(1.1) loads."""
    from sb200 import synth
    from sb200.ternary import TernaryExperts
    E, H, I, B, k = 64, 2048, 1024, 4096, 8
    experts = synth.ternary_experts(E, H, I, seed=2)
    te = TernaryExperts(experts, cuda_device)
    x = synth.hidden_states(B, H, seed=2, dtype=torch.bfloat16, device=cuda_device)
    ids_np, w_np = synth.zipf_routing(B, E, k, seed=2)
    ids = torch.from_numpy(ids_np).to(cuda_device)
    w = torch.from_numpy(w_np).to(cuda_device)
    y = te.forward(x, ids, w)
    y2 = te.forward(x, ids, w)
    assert torch.equal(y, y2), "not reproducible"
    rows = np.linspace(0, B - 1, 96).astype(np.int64)
    ref = otern.moe_combine(x[rows].float().cpu().numpy(), ids_np[rows], w_np[rows], experts)
    assert_close(y.cpu().numpy()[rows], ref, "config-2 sampled rows")
    # bf16 output path
    yb = te.forward(x, ids, w, out_dtype=torch.bfloat16)
    torch.testing.assert_close(yb.float(), y, rtol=8e-3, atol=1e-5)


@pytest.mark.parametrize("B", [1, 8, 64])
def test_moe_few_token_experts(cuda_device, B):
    """Small batches through the grouped layer (the tile kernels with polling
    waits): one token, one token per expert, a Zipf mix of small and large
    experts."""
    from sb200 import synth
    from sb200.ternary import TernaryExperts
    E, H, I, k = 64, 2048, 1024, 8
    experts = synth.ternary_experts(E, H, I, seed=2)
    te = TernaryExperts(experts, cuda_device)
    x = synth.hidden_states(B, H, seed=31, dtype=torch.bfloat16, device=cuda_device)
    ids_np, w_np = synth.zipf_routing(B, E, k, seed=32)
    counts = np.bincount(ids_np.ravel(), minlength=E)
    if B == 64:
        assert (counts > 8).any() and ((counts > 0) & (counts <= 8)).any()   # small and large experts
    ids = torch.from_numpy(ids_np).to(cuda_device)
    w = torch.from_numpy(w_np).to(cuda_device)
    y = te.forward(x, ids, w)
    assert torch.equal(te.forward(x, ids, w), y)
    ref = otern.moe_combine(x.float().cpu().numpy(), ids_np, w_np, experts)
    assert_close(y.cpu().numpy(), ref, f"few-token experts B={B}")


@pytest.mark.parametrize("engine", ENGINES, indirect=True)
def test_moe_edge_cases(cuda_device, engine):
    """Experts with no tokens, one token, duplicate ids in a row, B not a tile multiple."""
    from sb200 import synth
    from sb200.ternary import TernaryExperts
    E, H, I = 5, 256, 128
    experts = synth.ternary_experts(E, H, I, seed=9)
    te = TernaryExperts(experts, cuda_device)
    B, k = 131, 2
    x = synth.hidden_states(B, H, seed=10, device=cuda_device)
    ids = torch.zeros(B, k, dtype=torch.int32)
    ids[:, 1] = 3
    ids[0, 0] = 1        # expert 1: one token; experts 2 and 4: none
    ids[1, 1] = 0        # duplicate expert in one row
    w = torch.rand(B, k)
    y = te.forward(x, ids.to(cuda_device), w.to(cuda_device))
    ref = otern.moe_combine(x.cpu().numpy(), ids.numpy(), w.numpy(), experts)
    assert_close(y.cpu().numpy(), ref, "edge cases")
    empty = te.forward(x[:0], ids[:0].to(cuda_device), w[:0].to(cuda_device))
    assert empty.shape == (0, H)


def test_bridge_module(cuda_device):
    """CUDATernaryExpertModule: reference module API and buffers."""
    from dataclasses import dataclass
    import ternary_expert_ext_bridge as bridge
    from sb200 import synth
    assert bridge.HAS_TERNARY_EXT
    ex = synth.ternary_experts(1, 256, 512, seed=4)[0]

    @dataclass
    class FakeExpert:
        expert_id: int
        gate_ternary: np.ndarray
        up_ternary: np.ndarray
        down_ternary: np.ndarray
        gate_scale: np.ndarray
        up_scale: np.ndarray
        down_scale: np.ndarray

    fe = FakeExpert(0, ex["gate_ternary"].astype(np.float32), ex["up_ternary"].astype(np.float32),
                    ex["down_ternary"].astype(np.float32), ex["gate_scale"], ex["up_scale"], ex["down_scale"])
    m = bridge.create_expert_module(fe).cuda()
    x = torch.randn(2, 8, 256, device=cuda_device)
    out = m(x)
    assert out.shape == (2, 8, 256)
    ref = otern.gated_mlp(x.reshape(16, 256).cpu().numpy(), ex["gate_ternary"], ex["up_ternary"],
                          ex["down_ternary"], ex["gate_scale"], ex["up_scale"], ex["down_scale"])
    assert_close(out.reshape(16, 256).cpu().numpy(), ref, "bridge module")
    assert m.memory_bytes() == (16 * 512 + 16 * 512 + 32 * 256) * 4 + (512 + 512 + 256) * 4
