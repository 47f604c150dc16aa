"""Ternary packing: host packer against the reference extension, device layout round trip (no GPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden


POS = (0, 2, 4, 8, 10, 12, 6, 14)  # bit of pair j in each half (test-side restatement)


def decode_device(words: np.ndarray, K: int) -> np.ndarray:
    """Inverse of the biased-code device layout (test-side restatement):
    element 2j+e of a word is code value+1 at bits 16e+POS[j] .. 16e+POS[j]+1."""
    w = np.asarray(words).view(np.uint32)
    N, KW = w.shape
    p = np.array(POS, dtype=np.uint32)
    out = np.zeros((N, KW, 8, 2), np.int8)
    for e in range(2):
        code = (w[:, :, None] >> (16 * e + p)) & 3
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
    """Two elements per word become 16-bit +-1/0 with one and-or and one packed
    subtraction: with the exponent that makes bit p the mantissa's unit,
    (w & (3 << p)) | E is b + code, b = 2^(7-p) (bf16, p <= 4) or 2^(10-p)
    (fp16, p <= 8), and (b + code) - (b + 1) is the weight.  Pairs past the
    mantissa are first shifted by 8 (then sitting at p - 8) or down to bit 0,
    as the kernels' tern_pair_c does."""
    from sb200.ternary import pack_device, TERN_POS
    assert tuple(TERN_POS) == POS
    rng = np.random.default_rng(5)
    T = rng.integers(-1, 2, size=(4, 16), dtype=np.int8)
    for row in range(4):
        w = int(pack_device(T[row:row + 1])[0, 0])
        for fmt, lim in (("bf16", 4), ("f16", 8)):
            def to_f(h):
                if fmt == "f16":
                    return float(np.array([h], np.uint16).view(np.float16)[0])
                return float(np.array([h << 16], np.uint32).view(np.float32)[0])
            for j in range(8):
                p = POS[j]
                if p <= lim:
                    src, q = w, p
                elif p >= 8 and p - 8 <= lim:
                    src, q = w >> 8, p - 8
                else:
                    src, q = w >> p, 0
                base = ((134 - q) << 7) if fmt == "bf16" else ((25 - q) << 10)
                t = (src & (0x00030003 << q)) | (base | (base << 16))
                for e in range(2):
                    half = (t >> (16 * e)) & 0xFFFF
                    # the subtraction is exact: both operands and the result are representable
                    assert to_f(half) - to_f(base + (1 << q)) == T[row, 2 * j + e], (fmt, j, e)
                # the run-time form: shift to bit 0 by the nibble table
                sh = (0xE6CA8420 >> (4 * j)) & 15
                assert sh == p


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
