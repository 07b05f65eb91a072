"""Known-answer cases transcribed from the reference's own unit tests.

Each case names the reference gate it restates (tests/unit/*.c of
Entkenntnis/deepseek-v4-in-c). The same cases pin the CPU oracle
(test_oracle_pins.py) and check the CUDA library (test_gpu_*.py).
"""
from __future__ import annotations

import math

import numpy as np

FP8, FP4, BF16 = 2, 3, 1


def matmul_cases():
    """(name, wdt, W, S, rows, cols, blk_r, blk_c, x[nt][cols], expected y[nt][rows] or None, check)
    check: 'exact' (bit equality), 'absmag' (compare |y|) or 'nan_row0'."""
    cases = []
    # test_matmul.c:205-228 GATE 1: one 128-wide block, both rows share S[0] = 2
    W = np.zeros((2, 128), np.uint8)
    W[0] = 0x38
    W[1] = 0x40
    S = np.array([128, 0], np.uint8)
    x = np.ones((1, 128), np.float32)
    cases.append(("fp8_gate1", FP8, W, S, 2, 128, 128, 128, x, np.array([[256, 512]], np.float32), "exact"))
    # :230-251 GATE 1b: the row dimension of the scale grid
    W = np.full((256, 128), 0x38, np.uint8)
    S = np.array([127, 129], np.uint8)
    y = np.concatenate([np.full(128, 128.0), np.full(128, 512.0)]).astype(np.float32)[None]
    cases.append(("fp8_gate1b", FP8, W, S, 256, 128, 128, 128, np.ones((1, 128), np.float32), y, "exact"))
    # :253-271 GATE 2: scales advance across blocks -> 384
    W = np.full((1, 256), 0x38, np.uint8)
    S = np.array([127, 128], np.uint8)
    cases.append(("fp8_gate2", FP8, W, S, 1, 256, 128, 128, np.ones((1, 256), np.float32),
                  np.array([[384]], np.float32), "exact"))
    # :274-293 GATE 3: FP4 per-row and per-block scales -> 96, 64
    W = np.full((2, 32), 0x22, np.uint8)
    S = np.array([127, 128, 127, 127], np.uint8)
    cases.append(("fp4_gate3", FP4, W, S, 2, 64, 1, 32, np.ones((1, 64), np.float32),
                  np.array([[96, 64]], np.float32), "exact"))
    # :295-315 GATE 4: FP4 row stride is in/2 bytes -> 32, 64
    W = np.zeros((2, 16), np.uint8)
    W[0] = 0x22
    W[1] = 0x44
    S = np.array([127, 127], np.uint8)
    cases.append(("fp4_gate4", FP4, W, S, 2, 32, 1, 32, np.ones((1, 32), np.float32),
                  np.array([[32, 64]], np.float32), "exact"))
    # :317-336 GATE 5: signed values, |y| = 32
    W = np.full((1, 16), 0xA2, np.uint8)
    S = np.array([128], np.uint8)
    x = np.arange(1, 33, dtype=np.float32)[None]
    cases.append(("fp4_gate5", FP4, W, S, 1, 32, 1, 32, x, np.array([[32]], np.float32), "absmag"))
    # :338-361 GATE 5b: four-block batch plus a tail block, scales 2^((b+o)%5)
    W = np.full((3, 80), 0x22, np.uint8)
    S = np.array([127 + ((b + o) % 5) for o in range(3) for b in range(5)], np.uint8)
    y = np.array([[sum(32.0 * 2 ** ((b + o) % 5) for b in range(5)) for o in range(3)]], np.float32)
    cases.append(("fp4_gate5b", FP4, W, S, 3, 160, 1, 32, np.ones((1, 160), np.float32), y, "exact"))
    # :363-380 GATE 5c: 513 blocks (over the batched path's bound) sum to IN
    W = np.full((1, 16416 // 2), 0x22, np.uint8)
    S = np.full(16416 // 32, 127, np.uint8)
    cases.append(("fp4_gate5c", FP4, W, S, 1, 16416, 1, 32, np.ones((1, 16416), np.float32),
                  np.array([[16416]], np.float32), "exact"))
    # :382-402 GATE 6: bf16 rows of 1.0 / 2.0 against 0.5 -> 16, 32
    W = np.zeros((2, 32), np.uint16)
    W[0] = 0x3F80
    W[1] = 0x4000
    cases.append(("bf16_gate6", BF16, W, None, 2, 32, 0, 0, np.full((1, 32), 0.5, np.float32),
                  np.array([[16, 32]], np.float32), "exact"))
    # :587-633 every E4M3 code: W[r][r] = r, x = 1 -> y[r] = decode(r)
    W = np.zeros((256, 256), np.uint8)
    W[np.arange(256), np.arange(256)] = np.arange(256, dtype=np.uint8)
    S = np.full(4, 127, np.uint8)
    cases.append(("fp8_all_codes", FP8, W, S, 256, 256, 128, 128, np.ones((1, 256), np.float32),
                  None, "all_codes"))
    # :636-688 normal-only blocks, then a subnormal, two NaNs and a zero in block 0
    r = 987654321
    x = np.zeros(512, np.float32)
    for i in range(512):
        r = (r * 1103515245 + 12345) & 0xFFFFFFFF
        x[i] = np.float32(((r >> 16) & 0xFF) - 128) * np.float32(0.01)
    Wn = np.zeros(256 * 512, np.uint8)
    for i in range(Wn.size):
        r = (r * 1103515245 + 12345) & 0xFFFFFFFF
        e = 1 + ((r >> 16) % 14)
        m = (r >> 20) & 7
        s = (r >> 24) & 1
        Wn[i] = (s << 7) | (e << 3) | m
    Wn = Wn.reshape(256, 512)
    S = np.full(2 * 4, 127, np.uint8)
    cases.append(("fp8_normal_blocks", FP8, Wn.copy(), S, 256, 512, 128, 128, x[None], None, "l2"))
    Ws = Wn.copy()
    Ws[0, 0], Ws[0, 1], Ws[0, 2], Ws[0, 3] = 0x01, 0x7F, 0xFF, 0x00
    cases.append(("fp8_special_block", FP8, Ws, S, 256, 512, 128, 128, x[None], None, "nan_row0"))
    return cases


def e4m3_value(b: int) -> float:
    s = (b >> 7) & 1
    e = (b >> 3) & 15
    m = b & 7
    if e == 15 and m == 7:
        return math.nan
    v = m * 2.0 ** -9 if e == 0 else (1 + m / 8) * 2.0 ** (e - 7)
    return -v if s else v


# test_quant.c:39-70 (E8M0) and :72-120 (E4M3 edges)
E8M0_KAT = [(127, 1.0), (128, 2.0), (126, 0.5), (137, 1024.0), (117, 1.0 / 1024.0),
            (1, 2.0 ** -126), (0, 2.0 ** -127)]
E4M3_KAT = [(0x00, 0.0), (0x38, 1.0), (0xB8, -1.0), (0x3C, 1.5), (0x3A, 1.25), (0x40, 2.0),
            (0x30, 0.5), (0x01, 2.0 ** -9), (0x02, 2.0 ** -8), (0x07, 7 * 2.0 ** -9),
            (0x7E, 448.0), (0x7B, 352.0)]
E2M1_KAT = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


def route_kat():
    """test_ops.c:120-218: (name, logits, bias, tid2eid, token_id, topk, scale, check fn)."""
    out = []
    logits = np.array([3.0, 0.1, 0.2, 0.3, 0.4, 2.0], np.float32)
    bias = np.array([0, 0, 0, 0, 0, 5.0], np.float32)

    def bias_check(idx, wts, scores, orig):
        s0 = np.float32(math.sqrt(math.log1p(math.exp(3.0))))
        s5 = np.float32(math.sqrt(math.log1p(math.exp(2.0))))
        return (idx[0] == 5 and idx[1] == 0 and abs(wts[0] - s5 / (s0 + s5)) < 1e-6
                and abs(wts[1] - s0 / (s0 + s5)) < 1e-6)
    out.append(("bias_selects_only", logits, bias, None, 0, 2, 1.0, bias_check))

    logits_h = np.array([9.0, 0.1, 0.2, 0.3, 0.4, 0.5], np.float32)
    tid = np.array([3, 4, 1, 2, 5, 0, 2, 3], np.int64)

    def hash_check(idx, wts, scores, orig):
        s5 = math.sqrt(math.log1p(math.exp(0.5)))
        s0 = math.sqrt(math.log1p(math.exp(9.0)))
        return idx[0] == 5 and idx[1] == 0 and abs(wts[0] - s5 / (s5 + s0)) < 1e-6
    out.append(("hash_route", logits_h, None, tid, 2, 2, 1.0, hash_check))

    logits_t = np.array([200.0, 100.0, 1.0, 0.5], np.float32)

    def thresh_check(idx, wts, scores, orig):
        return bool(np.all(np.isfinite(wts))) and abs(orig[0] - math.sqrt(200.0)) < 1e-4
    out.append(("softplus_threshold", logits_t, None, None, 0, 2, 1.0, thresh_check))

    logits_s = np.array([2.0, 1.0, 0.5, 0.2], np.float32)

    def scale_check(idx, wts, scores, orig):
        return abs(float(np.sum(wts.astype(np.float64))) - 2.5) < 1e-5
    out.append(("route_scale", logits_s, None, None, 0, 2, 2.5, scale_check))
    return out


def attn_kat():
    """test_attn.c:21-128: (name, q, kv, sink, idxs, scale, check fn(o))."""
    out = []
    kv = np.repeat(np.arange(1, 5, dtype=np.float32)[:, None], 4, 1)
    out.append(("uniform_mean", np.zeros((2, 4), np.float32), kv, np.array([-1000, -1000], np.float32),
                np.arange(4, dtype=np.int32), 1.0, lambda o: np.all(np.abs(o - 2.5) < 1e-5)))
    kv8 = np.array([[8.0, 8.0]], np.float32)
    out.append(("sink_denominator_only", np.zeros((1, 2), np.float32), kv8, np.array([0.0], np.float32),
                np.array([0], np.int32), 1.0, lambda o: abs(o[0, 0] - 4.0) < 1e-5))
    out.append(("sink_small", np.zeros((1, 2), np.float32), kv8, np.array([-20.0], np.float32),
                np.array([0], np.int32), 1.0, lambda o: abs(o[0, 0] - 8.0) < 1e-3))
    out.append(("sink_large", np.zeros((1, 2), np.float32), kv8, np.array([20.0], np.float32),
                np.array([0], np.int32), 1.0, lambda o: o[0, 0] < 1e-3))
    out.append(("sink_per_head", np.zeros((2, 2), np.float32), kv8, np.array([-20.0, 20.0], np.float32),
                np.array([0], np.int32), 1.0, lambda o: abs(o[0, 0] - 8) < 1e-3 and o[1, 0] < 1e-3))
    kv2 = np.repeat(np.arange(1, 5, dtype=np.float32)[:, None], 2, 1)
    out.append(("masked_slots", np.zeros((1, 2), np.float32), kv2, np.array([-1000.0], np.float32),
                np.array([0, -1, 2, -1], np.int32), 1.0, lambda o: abs(o[0, 0] - 2.0) < 1e-5))
    kv3 = np.array([[1, 0], [0, 1], [-1, 0]], np.float32)
    out.append(("scores_select", np.array([[0.0, 10.0]], np.float32), kv3, np.array([-1000.0], np.float32),
                np.array([0, 1, 2], np.int32), 1.0, lambda o: o[0, 1] > 0.99 and abs(o[0, 0]) < 0.01))
    out.append(("all_masked_is_zero", np.ones((1, 2), np.float32), kv3, np.array([0.5], np.float32),
                np.array([-1, -1], np.int32), 1.0, lambda o: np.all(o == 0)))
    return out


def window_kat():
    """test_attn.c:130-166: (pos, win, expected slots, expected count)."""
    return [(0, 4, [0, -1, -1, -1], 1), (2, 4, [2, 1, 0, -1], 3), (5, 4, [1, 0, 3, 2], 4)]


def topk_ref_scan(scores, k):
    """The definition the reference heap must match (test_indexer.c:20-34)."""
    n = len(scores)
    k = min(k, n)
    idx = []
    for _ in range(k):
        best = -1
        for c in range(n):
            if c in idx:
                continue
            if best < 0 or scores[c] > scores[best]:
                best = c
        idx.append(best)
    return np.array(idx, np.int32)
