"""bench.py's roofline arithmetic (no GPU): the dominant kernel's achieved rate
is the step's algorithmic FLOPs divided by its launches per step, over the
average launch time, so a layer that launches the kernel once per token range
is not credited with the whole step's work per launch."""

from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


PEAK = {"bf16_tflops": 1000.0, "source": "measured"}


def test_one_launch_per_step():
    b = _bench()
    meta = {"dominant": "not_profiled_kernel", "dominant_flop": 2.0e11, "tokens_per_step": 4096}
    r = b.roofline_tensor(meta, {"not_profiled_kernel": (10, 2.0)}, PEAK, 0.0, 10)  # 0.2 ms a launch
    assert r["launches_per_step"] == 1.0
    assert r["algorithmic_flop_per_launch"] == pytest.approx(2.0e11)
    assert r["achieved"] == pytest.approx(1000.0, rel=1e-3)      # 2e11 FLOP / 0.2 ms
    assert r["frac"] == pytest.approx(1.0, rel=1e-3)
    assert "note" not in r and r["traffic"] is None


def test_chunked_launches_share_the_step():
    b = _bench()
    meta = {"dominant": "not_profiled_kernel", "dominant_flop": 2.0e11, "tokens_per_step": 4096}
    # two launches a step (two token ranges), each 0.1 ms: the same work per step
    r = b.roofline_tensor(meta, {"not_profiled_kernel": (20, 2.0)}, PEAK, 0.0, 10)
    assert r["launches_per_step"] == 2.0
    assert r["algorithmic_flop_per_launch"] == pytest.approx(1.0e11)
    assert r["achieved"] == pytest.approx(1000.0, rel=1e-3)
    assert "note" in r


def test_unprofiled_kernel_gives_no_roofline():
    b = _bench()
    meta = {"dominant": "k", "dominant_flop": 1.0, "tokens_per_step": 1}
    assert b.roofline_tensor(meta, {}, PEAK, 0.0, 1) is None
