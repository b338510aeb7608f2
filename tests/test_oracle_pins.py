"""Pin the CPU oracle before trusting it (no GPU).

1. The reference's own known-answer packing tests (tests/test_pack.py in the
   reference), restated here with the same literal words.
2. Golden vectors produced by running the reference's kernels on the same
   seeded inputs (tests/golden/make_golden.py).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden.cases import CASES


# --- reference tests/test_pack.py:25-52, 101-111, restated ------------------
def test_pack_2bit_lsb_first_known_words():
    codes = np.zeros((1, 128), dtype=np.uint32)
    codes[0, 0], codes[0, 1], codes[0, 15], codes[0, 16] = 2, 1, 2, 3
    packed = oracle.pack_2bit(codes)
    assert packed.dtype == np.uint32 and packed.shape == (1, 8)
    assert packed[0, 0] == np.uint32((2 << 0) | (1 << 2) | (2 << 30))
    assert packed[0, 1] == np.uint32(3)
    np.testing.assert_array_equal(oracle.unpack_2bit(packed), codes)


def test_pack_2bit_sixteen_codes_one_word():
    codes = (np.arange(16, dtype=np.uint32) % 3).reshape(1, 16)
    expected = 0
    for i, c in enumerate(codes[0]):
        expected |= int(c) << (2 * i)
    assert oracle.pack_2bit(codes)[0, 0] == np.uint32(expected)


def test_pack_4bit_lsb_first_known_word():
    codes = np.zeros((1, 64), dtype=np.uint32)
    codes[0, 0], codes[0, 1], codes[0, 7] = 0xA, 0x3, 0xF
    packed = oracle.pack_4bit(codes)
    assert packed.shape == (1, 8)
    assert packed[0, 0] == np.uint32((0xA << 0) | (0x3 << 4) | (0xF << 28))
    np.testing.assert_array_equal(oracle.unpack_4bit(packed), codes)


def test_ternarize_sign_mask_alpha_zero_row():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((32, 128)).astype(np.float32)
    packed, alpha = oracle.ternarize(w)
    t = oracle.unpack_2bit(packed).astype(np.float32) - 1
    aw = np.abs(w)
    mask = aw > 0.7 * aw.mean(-1, keepdims=True)
    np.testing.assert_array_equal(t, np.sign(w) * mask)
    np.testing.assert_allclose(alpha, (aw * mask).sum(-1) / mask.sum(-1), rtol=1e-6)
    p0, a0 = oracle.ternarize(np.zeros((2, 128), np.float32))
    np.testing.assert_array_equal(oracle.unpack_2bit(p0), np.ones((2, 128), np.uint32))
    np.testing.assert_array_equal(a0, 0)
    with pytest.raises(ValueError, match="multiple"):
        oracle.ternarize(np.ones((4, 64), np.float32))


def test_quantize_rtn_roundtrip_within_half_scale():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((16, 64)).astype(np.float32)
    packed, s, b = oracle.quantize_rtn(w)
    rec = oracle.dequantize_rtn(packed, s, b)
    assert np.all(np.abs(rec - w) <= 0.5 * s[:, :1] + 1e-5)


def test_bf16_rne():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.0e38, np.nan, np.inf], np.float32)
    bits = oracle.bf16_bits(x)
    assert bits[0] == 0x3F80 and bits[1] == 0x3F80 and bits[2] == 0x3F81
    assert bits[4] == 0x7FC0 and bits[5] == 0x7F80


def test_oracle_exp_accuracy():
    x = np.linspace(-100, 80, 20001, dtype=np.float32)
    got = oracle.mexp(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    ok = ref > 1e-37
    rel = np.abs(got[ok] - ref[ok]) / ref[ok]
    assert rel.max() < 3e-7, rel.max()
    assert oracle.mexp(np.zeros(1))[0] == 1.0


# --- oracle vs the reference's own kernels on identical inputs ---------------
@pytest.mark.parametrize("name", [n for n, c in CASES.items() if c.kind == "ternary_gemv"])
def test_oracle_ternary_gemv_matches_reference(golden, name):
    case = CASES[name]
    d = case.inputs()
    y_ref = golden[f"{name}/y"]
    y = oracle.ternary_gemv(d["x"], d["packed"], d["alpha"], d["rms_weight"], 1e-6, out_bf16=False)
    # Both accumulate in >= fp32; the reference's tl.rsqrt is approximate.
    np.testing.assert_allclose(y, y_ref, rtol=2e-5, atol=2e-6 * np.abs(y_ref).max())
