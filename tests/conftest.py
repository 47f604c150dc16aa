"""Shared test setup: import paths, the ``gpu`` marker and golden-fixture loaders."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "spectral-ai_b200"
GOLDEN = REPO / "tests" / "golden"
for p in (str(PKG), str(REPO), str(REPO / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    """A GPU test that has not finished in 10 minutes ends the run (pytest-timeout's
    thread method, which also ends a process blocked inside a CUDA call) instead of
    holding the GPU until an outer limit."""
    try:
        import pytest_timeout  # noqa: F401
    except ImportError:
        return
    for item in items:
        if item.get_closest_marker("gpu") is not None and item.get_closest_marker("timeout") is None:
            item.add_marker(pytest.mark.timeout(600, method="thread"))


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz", allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def golden_router_case(name: str):
    """(weights dict, x fp32 [B,H], golden dict) for a router golden.

    Small cases store everything; config-0 cases are regenerated from the
    recipe in sb200/synth.py and checked against the stored checksums."""
    from sb200 import synth
    g = load_golden(name)
    if "x" in g:
        w = {k[2:]: v for k, v in g.items() if k.startswith("w/")}
        return w, g["x"], g
    H, S = int(g["H"]), int(g["S"])
    br = tuple(int(b) for b in g["branching"])
    w = synth.router_weights(H, S, br, seed=int(g["seed"]), perturb=bool(g["perturb"]),
                             temperature=float(g["temperature"]))
    x = synth.hidden_states(int(g["batch"]), H, seed=int(g["x_seed"])).numpy()
    from golden.make_golden import checksum  # same checksum routine as the generator
    assert np.allclose(checksum(x), g["x_checksum"], rtol=1e-9, atol=1e-9), "input recipe drifted"
    for k, v in w.items():
        assert np.allclose(checksum(v), g["wsum/" + k], rtol=1e-9, atol=1e-9), f"weight recipe drifted: {k}"
    return w, x, g


ROUTER_GOLDENS = ["router_small", "router_small_t05", "router_small_352", "router_cfg0",
                  "router_cfg0_perturbed"]


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test, the library's device status word must be clean
    (no kernel gave up a bounded wait)."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    from sb200 import _lib
    torch.cuda.synchronize()
    rc = _lib.load().sb_device_status(0)
    assert rc == 0, f"device status: {_lib.last_error()}"
