"""Device weight quantizers match the host packer bit for bit."""
from __future__ import annotations

import numpy as np
import pytest

import pack

pytestmark = pytest.mark.gpu


def test_quantize_fp8_fp4_match_host(dev):
    t = __import__("torch")
    rng = np.random.default_rng(0)
    for rows, cols in ((300, 520), (128, 128), (7, 64)):
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        w.flat[::97] = 0.0
        if rows == 128:
            # block amax 448 * 2^-10 gives scale 2^-10; then exact rounding ties:
            # 432 (416|448 -> 448), 1.0625 (1|1.125 -> 1), 1.5 * 2^-9 (sub 1|2 -> 2)
            w[0, :5] = np.array([448.0, 432.0, -432.0, 1.0625, 1.5 * 2.0 ** -9], np.float32) * 2.0 ** -10
        src = t.from_numpy(w).cuda()
        W = t.empty((rows, cols), dtype=t.uint8, device="cuda")
        S = t.empty(((rows + 127) // 128) * ((cols + 127) // 128), dtype=t.uint8, device="cuda")
        dev.quantize_fp8(W, S, src, rows, cols)
        hW, hS = pack.quantize_fp8(w)
        t.cuda.synchronize()
        assert np.array_equal(S.cpu().numpy(), hS.reshape(-1))
        assert np.array_equal(W.cpu().numpy(), hW)
    for rows, cols in ((64, 256), (5, 32)):
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        w[0, :8] = np.array([1.25, 2.5, 5.0, 0.25, -1.75, 3.5, 6.0, 0.0], np.float32)
        src = t.from_numpy(w).cuda()
        W = t.empty((rows, cols // 2), dtype=t.uint8, device="cuda")
        S = t.empty((rows, cols // 32), dtype=t.uint8, device="cuda")
        dev.quantize_fp4(W, S, src, rows, cols)
        hW, hS = pack.quantize_fp4(w)
        t.cuda.synchronize()
        assert np.array_equal(S.cpu().numpy(), hS)
        assert np.array_equal(W.cpu().numpy(), hW)


def test_fill_normal_moments_and_determinism(dev):
    t = __import__("torch")
    a = t.empty(1 << 20, dtype=t.float32, device="cuda")
    b = t.empty(1 << 20, dtype=t.float32, device="cuda")
    dev.fill_normal(a, 123, 0.0, 0.02)
    dev.fill_normal(b, 123, 0.0, 0.02)
    t.cuda.synchronize()
    assert t.equal(a, b)
    assert abs(a.mean().item()) < 1e-4 and abs(a.std().item() - 0.02) < 2e-4
