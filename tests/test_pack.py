"""Host packers (deepseek-v4-in-c_b200/pack.py): format rules on the CPU."""
from __future__ import annotations

import numpy as np

import pack


def test_fp8_roundtrip_error_bound():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((300, 520)) * 0.02).astype(np.float32)
    W, S = pack.quantize_fp8(w)
    assert W.shape == w.shape and S.shape == (3, 5)
    back = pack.dequant_fp8(W, S)
    scale = np.repeat(np.repeat(pack.e8m0(S), 128, 0), 128, 1)[:300, :520]
    # e4m3 has 3 mantissa bits: error <= 2^-4 relative to the value, or half the
    # subnormal step 2^-10 * scale near zero
    err = np.abs(back - w)
    bound = np.maximum(np.abs(w) * 2.0 ** -4, scale * 2.0 ** -10) * 1.0001
    assert np.all(err <= bound)
    # block amax maps into (224, 448]
    amax = np.abs(w[:128, :128]).max() / pack.e8m0(S[0, 0])
    assert 224 < amax <= 448


def test_fp4_roundtrip_and_nibble_order():
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    W, S = pack.quantize_fp4(w)
    assert W.shape == (64, 128) and S.shape == (64, 8)
    back = pack.dequant_fp4(W, S, 256)
    sc = np.repeat(pack.e8m0(S), 32, 1)
    assert np.all(np.abs(back - w) <= sc * 1.0 + 1e-12)  # half the widest e2m1 step (2) * scale
    # even element is the low nibble
    W2, S2 = pack.quantize_fp4(np.array([[0.5, 1.0] + [0.0] * 30], np.float32) * 4)
    assert (W2[0, 0] & 15) != (W2[0, 0] >> 4)


def test_rne_ties_to_even():
    # e2m1 grid {0,.5,1,1.5,2,3,4,6}: 1.25 -> 1.0 (even code 2), 2.5 -> 2, 5 -> 4, 0.25 -> 0
    v = np.array([1.25, 2.5, 5.0, 0.25, 1.75, 3.5, 7.0], np.float32)
    codes = pack._rne_grid(v, pack._E2M1_POS)
    assert pack.E2M1[codes].tolist() == [1.0, 2.0, 4.0, 0.0, 2.0, 4.0, 6.0]
    # e4m3: 432 is the midpoint of 416 (0x7D) and 448 (0x7E) -> 448
    assert pack.E4M3[pack._rne_grid(np.array([432.0, 1000.0], np.float32), pack._E4M3_POS)].tolist() == [448, 448]


def test_bf16_round():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.14159], np.float32)
    r = pack.bf16_round(x)
    assert r[0] == 1.0 and r[1] == 1.0  # tie to even
    assert (r.view(np.uint32) & 0xFFFF).max() == 0
