"""Host-side packers for the reference weight layouts (numpy).

The same rule as the device quantizers (dsv4cu_quantize_fp8 / _fp4):
scale = 2^ceil(log2(amax / qmax)) stored as an E8M0 byte (127 + exponent),
values rounded to nearest-even on the e4m3 / e2m1 grid and saturated to
448 / 6. FP8 blocks are 128x128, FP4 blocks 1x32 with the low nibble holding
the even column (src/10_compute/dsv4_quant.h:31-56). The reference ships no
quantizer; its checkpoint arrives packed (tools/pack_trunk.py copies bytes).
"""
from __future__ import annotations

import numpy as np


def e4m3_table() -> np.ndarray:
    """f32 value of every e4m3fn code (0x7F/0xFF NaN)."""
    b = np.arange(256, dtype=np.uint32)
    s = (b >> 7) & 1
    e = (b >> 3) & 15
    m = (b & 7).astype(np.float64)
    v = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * 2.0 ** (e.astype(np.float64) - 7))
    v = np.where(s == 1, -v, v)
    v[(e == 15) & ((b & 7) == 7)] = np.nan
    return v.astype(np.float32)


E4M3 = e4m3_table()
E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0.0, -.5, -1, -1.5, -2, -3, -4, -6], np.float32)


def e8m0(b) -> np.ndarray:
    b = np.asarray(b, np.uint32)
    u = np.where(b == 255, 0x7FC00000, np.where(b == 0, 0x00400000, b << 23)).astype(np.uint32)
    return u.view(np.float32)


def _exponent(amax: np.ndarray, qf: float, qe: int) -> np.ndarray:
    """Exponent e of the smallest 2^e with amax / 2^e <= qmax = qf 2^qe."""
    f, E = np.frexp(amax.astype(np.float32))
    e = E - qe + (f > qf).astype(np.int64)
    e = np.where((amax > 0) & np.isfinite(amax), e, 0)
    return np.clip(e, -127, 127).astype(np.int64)


def _rne_grid(v: np.ndarray, grid: np.ndarray) -> np.ndarray:
    """Index into the ascending non-negative grid of the nearest value to |v|,
    ties to the even index (= even mantissa), saturating at the top."""
    a = np.abs(v).astype(np.float64)
    hi = np.clip(np.searchsorted(grid, a, side="left"), 1, len(grid) - 1)
    lo = hi - 1
    dlo = a - grid[lo]
    dhi = grid[hi] - a
    pick = np.where(dlo < dhi, lo, np.where(dhi < dlo, hi, np.where(lo % 2 == 0, lo, hi)))
    pick = np.where(a >= grid[-1], len(grid) - 1, pick)
    pick = np.where(a <= grid[0], 0, pick)
    return pick


_E4M3_POS = E4M3[:0x7F].astype(np.float64)          # codes 0x00..0x7E ascending
_E2M1_POS = E2M1[:8].astype(np.float64)


def quantize_fp8(w: np.ndarray):
    """fp32 [rows][cols] -> (e4m3 bytes [rows][cols], E8M0 [ceil(r/128)][ceil(c/128)])."""
    w = np.ascontiguousarray(w, np.float32)
    rows, cols = w.shape
    br, bc = -(-rows // 128), -(-cols // 128)
    pad = np.zeros((br * 128, bc * 128), np.float32)
    pad[:rows, :cols] = np.where(np.isfinite(w), np.abs(w), 0)
    amax = pad.reshape(br, 128, bc, 128).max(axis=(1, 3))
    e = _exponent(amax, 0.875, 9)
    S = (127 + e).astype(np.uint8)
    ef = np.repeat(np.repeat(e, 128, 0), 128, 1)[:rows, :cols]
    v = np.ldexp(w, -ef).astype(np.float32)
    code = _rne_grid(v, _E4M3_POS).astype(np.uint8)
    code = np.where(np.signbit(v), code | 0x80, code).astype(np.uint8)
    code = np.where(np.isnan(v), np.uint8(0x7F), code).astype(np.uint8)
    return code, S


def quantize_fp4(w: np.ndarray):
    """fp32 [rows][cols] (cols % 32 == 0) -> (packed [rows][cols/2], E8M0 [rows][cols/32])."""
    w = np.ascontiguousarray(w, np.float32)
    rows, cols = w.shape
    assert cols % 32 == 0
    blk = w.reshape(rows, cols // 32, 32)
    amax = np.where(np.isfinite(blk), np.abs(blk), 0).max(axis=2)
    e = _exponent(amax, 0.75, 3)
    S = (127 + e).astype(np.uint8)
    v = np.ldexp(blk, -e[:, :, None]).astype(np.float32).reshape(rows, cols)
    # Round to nearest on {0,.5,1,1.5,2,3,4,6}: count the midpoints below |v|.
    # A midpoint whose lower neighbour has an odd code (0.75, 1.75, 3.5) rounds
    # up on a tie (to the even code), the others round down: ties to even.
    a = np.abs(v)
    code = ((a > 0.25).astype(np.uint8) + (a >= 0.75) + (a > 1.25) + (a >= 1.75)
            + (a > 2.5) + (a >= 3.5) + (a > 5.0)).astype(np.uint8)
    code = np.where(np.signbit(v), code | 8, code).astype(np.uint8)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8)
    return packed, S


def dequant_fp8(W: np.ndarray, S: np.ndarray, blk_r=128, blk_c=128) -> np.ndarray:
    rows, cols = W.shape
    sc = e8m0(S)
    sf = np.repeat(np.repeat(sc, blk_r, 0), blk_c, 1)[:rows, :cols]
    return (E4M3[W].astype(np.float64) * sf).astype(np.float32)


def dequant_fp4(W: np.ndarray, S: np.ndarray, cols: int, blk_r=1, blk_c=32) -> np.ndarray:
    rows = W.shape[0]
    codes = np.empty((rows, cols), np.uint8)
    codes[:, 0::2] = W & 15
    codes[:, 1::2] = W >> 4
    sc = e8m0(S)
    sf = np.repeat(np.repeat(sc, blk_r, 0), blk_c, 1)[:rows, :cols]
    return (E2M1[codes].astype(np.float64) * sf).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 value (ties to even), kept as fp32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)
