"""Ternary packing: host packer against the reference extension, device layout round trip (no GPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden


def decode_device(words: np.ndarray, K: int) -> np.ndarray:
    """Inverse of the biased-code device layout (test-side restatement):
    element 2j+e of a word is code value+1 at bits 16e+2j .. 16e+2j+1."""
    w = np.asarray(words).view(np.uint32)
    N, KW = w.shape
    j = np.arange(8, dtype=np.uint32)
    out = np.zeros((N, KW, 8, 2), np.int8)
    for e in range(2):
        code = (w[:, :, None] >> (16 * e + 2 * j)) & 3
        assert (code <= 2).all(), "code 3 is not used"
        out[..., e] = code.astype(np.int8) - 1
    return out.reshape(N, KW * 16)[:, :K]


def test_pack_ternary_matches_reference_extension():
    import ternary_expert_ext as ext
    g = load_golden("ternary_small")
    if "pack/in" not in g:
        pytest.skip("golden made without the reference extension")
    got = ext.pack_ternary(torch.from_numpy(g["pack/in"]))
    assert got.dtype == torch.int32
    assert np.array_equal(got.numpy(), g["pack/out"])


def test_pack_ternary_rejects_non_cpu_int8():
    import ternary_expert_ext as ext
    with pytest.raises(RuntimeError):
        ext.pack_ternary(torch.zeros(4, 4, dtype=torch.float32))


@pytest.mark.parametrize("shape", [(7, 5), (128, 64), (40, 72), (256, 2048), (3, 1)])
def test_device_layout_round_trip(shape):
    from sb200.ternary import pack_device, row_words
    rng = np.random.default_rng(shape[0] * 1000 + shape[1])
    T = rng.integers(-1, 2, size=shape, dtype=np.int8)
    w = pack_device(T)
    assert w.shape == (shape[0], row_words(shape[1])) and w.dtype == np.uint32
    assert np.array_equal(decode_device(w, shape[1]), T)


def test_device_layout_pair_expansion_formula():
    """Two elements per word become 16-bit +-1/0 with shift, and-or and one packed
    subtraction of b+1 (b = 128 in bf16, 1024 in fp16): (b + code) - (b + 1)."""
    from sb200.ternary import pack_device
    rng = np.random.default_rng(5)
    T = rng.integers(-1, 2, size=(1, 16), dtype=np.int8)
    w = int(pack_device(T)[0, 0])
    for fmt, (bias, bias1) in {"bf16": (0x4300, 0x4301), "f16": (0x6400, 0x6401)}.items():
        def to_f(h):
            if fmt == "f16":
                return float(np.array([h], np.uint16).view(np.float16)[0])
            return float(np.array([h << 16], np.uint32).view(np.float32)[0])
        for j in range(8):
            t = ((w >> (2 * j)) & 0x00030003) | (bias | (bias << 16))
            for e in range(2):
                half = (t >> (16 * e)) & 0xFFFF
                # the subtraction is exact: both operands and the result are representable
                assert to_f(half) - to_f(bias1) == T[0, 2 * j + e]


def test_padding_decodes_to_zero():
    from sb200.ternary import pack_device
    T = np.ones((2, 5), np.int8)
    w = pack_device(T)
    d = decode_device(w, w.shape[1] * 16)
    assert (d[:, :5] == 1).all() and (d[:, 5:] == 0).all()


def test_torch_packer_matches_host_packer():
    from sb200.ternary import pack_device, pack_device_torch
    rng = np.random.default_rng(9)
    for shape in [(5, 70), (128, 2048), (3, 16)]:
        T = rng.integers(-1, 2, size=shape, dtype=np.int8)
        a = pack_device_torch(torch.from_numpy(T)).numpy().view(np.uint32)
        assert np.array_equal(a, pack_device(T))
