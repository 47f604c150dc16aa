"""The allocation-free router entry point against the workspace entry point (needs a B200).

sb_router_forward_noalloc serves callers that cannot allocate device memory
when they route a batch (a serving process whose HBM is all reserved by its own
pool, or a runtime binding the C ABI without a device allocator): it takes its
scratch from a fixed 32 MiB array inside the library instead of a workspace.
This file is collected last so that a failure here leaves every other test run.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _outputs(B, k, L, NL, dev):
    return {"topk_ids": torch.empty(B, k, dtype=torch.int32, device=dev),
            "topk_weights": torch.empty(B, k, dtype=torch.float32, device=dev),
            "expert_id": torch.empty(B, dtype=torch.int64, device=dev),
            "expert_probs": torch.empty(B, NL, dtype=torch.float32, device=dev),
            "route_path": torch.empty(B, L, dtype=torch.int64, device=dev),
            "confidence": torch.empty(B, dtype=torch.float32, device=dev)}


def _call_noalloc(eng, x, precision, select, k, res):
    from sb200 import _lib
    o = _lib.RouterOutputs()
    for name, t in res.items():
        setattr(o, name, t.data_ptr())
    stream = torch.cuda.current_stream(x.device).cuda_stream
    dtype = _lib.SB_BF16 if x.dtype == torch.bfloat16 else _lib.SB_F32
    return eng.lib.sb_router_forward_noalloc(eng.handle, C.c_void_p(x.data_ptr()), dtype, x.shape[0],
                                             precision, select, k, C.byref(o), C.c_void_p(stream))


def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    from sb200 import _lib, synth
    from sb200.router import RouterEngine
    H, S, k = 2048, 256, 8
    eng = RouterEngine(H, S, (4, 4, 4), cuda_device)
    eng.upload(synth.router_weights(H, S, seed=7, perturb=True))
    # two calls in a row with different batches, inputs and modes: the second
    # call reuses the array the first one left behind
    for call, (B, select, prec, dtype) in enumerate([(3000, "hard", "fast", torch.bfloat16),
                                                      (1200, "soft", "exact", torch.float32)]):
        x = synth.hidden_states(B, H, seed=100 + call, dtype=dtype, device=cuda_device)
        ref = eng.forward(x, precision=prec, select=select, k=k,
                          want=("expert_id", "expert_probs", "route_path", "confidence"))
        got = _outputs(B, k, 3, 64, cuda_device)
        rc = _call_noalloc(eng, x, _lib.SB_PREC_FAST if prec == "fast" else _lib.SB_PREC_EXACT,
                           _lib.SB_SELECT_HARD if select == "hard" else _lib.SB_SELECT_SOFT, k, got)
        _lib.check(rc, "sb_router_forward_noalloc")
        torch.cuda.synchronize()
        # same kernels on the same inputs: ids and paths identical, weights within the
        # router tests' fp32 tolerance
        for key in ("topk_ids", "expert_id", "route_path"):
            assert torch.equal(got[key], ref[key]), f"call {call}: {key}"
        for key in ("topk_weights", "expert_probs", "confidence"):
            torch.testing.assert_close(got[key], ref[key], rtol=1e-5, atol=1e-8)


def test_noalloc_rejects_batches_beyond_its_array(cuda_device):
    from sb200 import _lib, synth
    from sb200.router import RouterEngine
    H, S = 2048, 256
    eng = RouterEngine(H, S, (4, 4, 4), cuda_device)
    eng.upload(synth.router_weights(H, S, seed=8))
    B = 20000   # 20000 x (4 KiB + 1 KiB) > 32 MiB
    x = torch.zeros(B, H, dtype=torch.bfloat16, device=cuda_device)
    got = _outputs(B, 8, 3, 64, cuda_device)
    rc = _call_noalloc(eng, x, _lib.SB_PREC_FAST, _lib.SB_SELECT_HARD, 8, got)
    assert rc == -1
    assert "fixed array" in _lib.last_error()
