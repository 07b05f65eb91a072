"""Packed matmul on the B200 against the reference (golden vectors, known
answers) and the CPU oracle, through both C-ABI layers.

Tolerance (the BASELINE contract for matmul outputs): max|y - y_ref| /
max|y_ref| <= 1e-3. The kernels are far tighter in practice (exact products,
fp32 accumulation), so the L2 relative error is also held to 1e-5.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

import canary
import kat
import oracle
import pack
from conftest import golden

pytestmark = pytest.mark.gpu

MAX_REL = 1e-3
L2_REL = 1e-5


def rel_err(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    den = max(float(np.abs(want).max()), 1e-30)
    return float(np.abs(got - want).max()) / den


def l2_rel(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return math.sqrt(float(((got - want) ** 2).sum()) / max(float((want ** 2).sum()), 1e-300))


def assert_close(got, want, what=""):
    assert rel_err(got, want) <= MAX_REL, (what, rel_err(got, want))
    assert l2_rel(got, want) <= L2_REL, (what, l2_rel(got, want))


@pytest.fixture(autouse=True)
def _fresh_registry(host):
    host.forget_all()
    yield
    host.forget_all()


@pytest.mark.parametrize("case", kat.matmul_cases(), ids=lambda c: c[0])
def test_matmul_known_answers(host, orc, case):
    import dsv4cu
    name, wdt, W, S, rows, cols, br, bc, x, y, chk = case
    m = dsv4cu.QMat(W.ctypes.data, None if S is None else S.ctypes.data, wdt, rows, cols, br, bc)
    got = host.mmq(x, m)
    if chk == "exact":
        assert np.array_equal(got, y), (got, y)
    elif chk == "absmag":
        assert np.array_equal(np.abs(got), y)
    elif chk == "all_codes":
        want = pack.E4M3
        nan = np.isnan(want)
        assert np.all(np.isnan(got[0][nan]))
        assert np.array_equal(got[0][~nan], want[~nan] + 0.0)
    else:
        want = orc.mmq(x, oracle.qmat(W, S, wdt, rows, cols, br, bc))
        if chk == "nan_row0":
            assert np.isnan(got[0][0])
            assert not np.any(np.isnan(got[0][1:]))
            assert_close(got[0][1:], want[0][1:], name)
        else:
            assert_close(got, want, name)


def test_matmul_reference_golden(host):
    import dsv4cu
    g = dict(golden("matmul.npz"))
    for tag, wdt, br, bc in (("fp8", 2, 128, 128), ("fp8g", 2, 128, 100), ("fp4", 3, 1, 32),
                             ("fp4t", 3, 1, 32), ("bf16", 1, 0, 0)):
        W, x = g[f"{tag}_W"], g[f"{tag}_x"]
        S = g.get(f"{tag}_S")
        m = dsv4cu.QMat(W.ctypes.data, None if S is None else S.ctypes.data, wdt, W.shape[0],
                        x.shape[1], br, bc)
        assert_close(host.mmq(x, m), g[f"{tag}_y"], tag)


SHAPES = [
    # (wdt, rows, cols, blk_r, blk_c, nt)
    (2, 7168, 7168, 128, 128, 1),
    (2, 1024, 4096, 128, 128, 1),     # wq_a
    (2, 512, 4096, 128, 128, 3),      # wkv, small batch
    (2, 4096, 8192, 128, 128, 2),     # wo_b
    (2, 129, 320, 128, 128, 5),       # ragged rows, K not a multiple of 128
    (2, 200, 256, 64, 32, 1),         # other block grid, fast path
    (2, 33, 100, 16, 20, 2),          # generic path (blk_c % 16 != 0)
    (3, 2048, 4096, 1, 32, 1),        # routed w1/w3
    (3, 4096, 2048, 1, 32, 4),        # routed w2, batch
    (3, 77, 160, 1, 32, 7),           # tail blocks, odd rows, nt not a tile multiple
    (3, 40, 96, 2, 64, 2),            # two-row scale blocks, 64-wide
    (3, 9, 72, 1, 24, 1),             # generic path (blk_c % 32 != 0)
    (1, 256, 4096, 0, 0, 1),          # router gate
    (1, 64, 4096, 0, 0, 2),           # indexer weights_proj
    (1, 19, 36, 0, 0, 3),             # bf16 generic (cols % 8 != 0)
]


def make_weights(rng, wdt, rows, cols, br, bc):
    if wdt == 2:
        W = rng.integers(0, 256, (rows, cols), dtype=np.uint8)
        W = np.where((W & 0x7F) == 0x7F, W & 0xFE, W).astype(np.uint8)
        S = rng.integers(112, 132, (-(-rows // br)) * (-(-cols // bc)), dtype=np.uint8)
    elif wdt == 3:
        W = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
        S = rng.integers(112, 132, (-(-rows // br)) * (-(-cols // bc)), dtype=np.uint8)
    else:
        W = pack.bf16_bits((rng.standard_normal((rows, cols)) * 0.05).astype(np.float32))
        S = None
    return W, S


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "w%d_%dx%d_b%dx%d_nt%d" % s)
def test_matmul_vs_oracle(host, dev, orc, shape):
    import torch
    import dsv4cu
    wdt, rows, cols, br, bc, nt = shape
    rng = np.random.default_rng(rows * 31 + cols + nt)
    W, S = make_weights(rng, wdt, rows, cols, br, bc)
    x = pack.bf16_round(rng.standard_normal((nt, cols)).astype(np.float32))
    want = orc.mmq(x, oracle.qmat(W, S, wdt, rows, cols, br, bc))
    # host-pointer reference ABI
    m = dsv4cu.QMat(W.ctypes.data, None if S is None else S.ctypes.data, wdt, rows, cols, br, bc)
    got = host.mmq(x, m)
    assert_close(got, want, shape)
    if wdt == 1:        # BF16 runs the reference's double fma tree: same bits
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), shape
    # native device ABI gives the same bits
    dW = torch.from_numpy(W).cuda()
    dS = None if S is None else torch.from_numpy(S).cuda()
    dx = torch.from_numpy(x).cuda()
    dy = canary.guarded_empty((nt, rows))
    dev.mmq(dy, dx, dev.qmat(dW, dS, wdt, rows, cols, br, bc), nt)
    canary.check(dy, "mmq")
    assert np.array_equal(dy.cpu().numpy().view(np.uint32), got.view(np.uint32))


def test_matmul_fp32_activations(host, orc):
    """Arbitrary fp32 (not bf16-valued) activations stay within the contract."""
    import dsv4cu
    rng = np.random.default_rng(5)
    W, S = make_weights(rng, 2, 512, 2048, 128, 128)
    x = (rng.standard_normal((2, 2048)) * np.exp(rng.uniform(-6, 6, (2, 2048)))).astype(np.float32)
    m = dsv4cu.QMat(W.ctypes.data, S.ctypes.data, 2, 512, 2048, 128, 128)
    assert_close(host.mmq(x, m), orc.mmq(x, oracle.qmat(W, S, 2, 512, 2048, 128, 128)))


def test_batched_equals_single_token_calls_bitwise(host):
    """test_matmul.c:690-793: a batch row is the same arithmetic as a 1-token
    call; NT > 128 also crosses the reference's tile size."""
    import dsv4cu
    rng = np.random.default_rng(9)
    for wdt, br, bc in ((2, 128, 128), (3, 1, 32), (1, 0, 0)):
        W, S = make_weights(rng, wdt, 130, 256, br, bc)
        x = rng.standard_normal((130, 256)).astype(np.float32)
        m = dsv4cu.QMat(W.ctypes.data, None if S is None else S.ctypes.data, wdt, 130, 256, br, bc)
        batched = host.mmq(x, m)
        singles = np.stack([host.mmq(x[t:t + 1], m)[0] for t in range(0, 130, 13)])
        assert np.array_equal(batched[::13].view(np.uint32), singles.view(np.uint32)), wdt


def test_deterministic_and_cache_refresh(host):
    import dsv4cu
    rng = np.random.default_rng(3)
    W, S = make_weights(rng, 3, 1024, 2048, 1, 32)
    x = rng.standard_normal((1, 2048)).astype(np.float32)
    m = dsv4cu.QMat(W.ctypes.data, S.ctypes.data, 3, 1024, 2048, 1, 32)
    a = host.mmq(x, m)
    b = host.mmq(x, m)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # refill the same host buffer with another expert: the mirror must notice
    W[:] = rng.integers(0, 256, W.shape, dtype=np.uint8)
    c = host.mmq(x, m)
    assert not np.array_equal(a, c)
    d = oracle.Oracle().mmq(x, oracle.qmat(W, S, 3, 1024, 2048, 1, 32))
    assert_close(c, d)


@pytest.mark.parametrize("rows,cols,nt", [(4096, 7168, 1), (1000, 7168, 5), (300, 4104, 2), (77, 1030, 1),
                                         (1024, 4096, 1), (16384, 4096, 1), (3, 17, 1)])
def test_bf16_bitwise_with_specials(dev, orc, rows, cols, nt):
    """BF16 weights with zeros, subnormals and infinities among them and
    arbitrary fp32 activations: the reference's bits (bf16_n,
    src/10_compute/dsv4_matmul.c:88-113), including a misaligned row start
    (cols % 8 != 0 takes the halfword-load variant)."""
    import torch
    rng = np.random.default_rng(rows + cols + nt)
    W = pack.bf16_bits((rng.standard_normal((rows, cols)) * 0.05).astype(np.float32))
    flat = W.reshape(-1)
    pick = rng.integers(0, flat.size, flat.size // 50)
    flat[pick[0::3]] = 0x0000
    flat[pick[1::3]] = 0x8000 | rng.integers(1, 0x80, pick[1::3].size).astype(np.uint16)   # -subnormal
    flat[pick[2::3][:3]] = 0x7F80                                                      # +inf, a few rows
    x = (rng.standard_normal((nt, cols)) * np.exp(rng.uniform(-8, 8, (nt, cols)))).astype(np.float32)
    want = orc.mmq(x, oracle.qmat(W, None, 1, rows, cols))
    dW = torch.from_numpy(W).cuda()
    dx = torch.from_numpy(x).cuda()
    dy = canary.guarded_empty((nt, rows))
    dev.mmq(dy, dx, dev.qmat(dW, None, 1, rows, cols), nt)
    canary.check(dy, "mmq bf16")
    got = dy.cpu().numpy()
    fin = ~np.isnan(want)
    assert np.array_equal(np.isnan(got), ~fin)
    assert np.array_equal(got[fin].view(np.uint32), want[fin].view(np.uint32))


@pytest.mark.parametrize("path", ["mx", "fast", "generic", "batch"])
def test_every_e4m3_code_keeps_reference_bits(dev, path):
    """test_matmul.c:588-632: W[r][r] = r, x = 1, scales 2^0, so y[r] is the
    decode of code r - NaN codes 0x7F / 0xFF included, whose bits must be the
    reference's quiet NaNs 0x7FC00000 / 0xFFC00000. -0.0 codes give +0.0."""
    import torch
    N = 256
    bc = {"fast": 48, "generic": 120}.get(path, 128)  # 48: TMA GEMV tile, 120: generic double path
    W = np.zeros((N, N), np.uint8)
    W[np.arange(N), np.arange(N)] = np.arange(N, dtype=np.uint8)
    S = np.full((-(-N // 128)) * (-(-N // bc)), 127, np.uint8)
    nt = 1 if path != "batch" else 40
    x = np.ones((nt, N), np.float32)
    dW, dS = torch.from_numpy(W).cuda(), torch.from_numpy(S).cuda()
    dy = torch.empty((nt, N), dtype=torch.float32, device="cuda")
    dev.mmq(dy, torch.from_numpy(x).cuda(), dev.qmat(dW, dS, 2, N, N, 128, bc), nt)
    got = dy.cpu().numpy().view(np.uint32)
    want = np.array([np.float32(kat.e4m3_value(c)) for c in range(N)], np.float32).view(np.uint32).copy()
    want[want == 0x80000000] = 0
    want[0x7F], want[0xFF] = 0x7FC00000, 0xFFC00000
    for t in range(nt):
        assert np.array_equal(got[t], want), [hex(v) for v in got[t][want != got[t]][:4]]


def test_nan_scale_gives_positive_quiet_nan(dev):
    """E8M0 0xFF decodes to 0x7FC00000 (dsv4_quant.h:82): rows whose scale
    block is NaN come back with exactly those bits, on FP4 and FP8."""
    import torch
    rng = np.random.default_rng(17)
    for wdt, rows, cols, br, bc in ((3, 256, 512, 1, 32), (2, 256, 512, 128, 128)):
        W, S = make_weights(rng, wdt, rows, cols, br, bc)
        S = S.copy()
        S[1] = 0xFF                       # row block 0 (FP4: row 0), column block 1
        dW, dS = torch.from_numpy(W).cuda(), torch.from_numpy(S).cuda()
        x = np.ones((1, cols), np.float32)
        dy = torch.empty((1, rows), dtype=torch.float32, device="cuda")
        dev.mmq(dy, torch.from_numpy(x).cuda(), dev.qmat(dW, dS, wdt, rows, cols, br, bc), 1)
        got = dy.cpu().numpy()[0]
        nan_rows = 1 if wdt == 3 else 128
        assert np.all(got[:nan_rows].view(np.uint32) == 0x7FC00000), wdt
        assert not np.any(np.isnan(got[nan_rows:])), wdt


def ref_argmax(lg):
    """src/90_cli/dsv4_decode.c:128-133, literally."""
    best = 0
    for v in range(1, len(lg)):
        if lg[v] > lg[best]:
            best = v
    return best


def test_argmax_rule(dev):
    import torch
    rng = np.random.default_rng(21)
    rows = []
    a = rng.standard_normal(129280).astype(np.float32)
    rows.append(a)
    b = a.copy(); b[5] = b[77777] = b.max() + 1; rows.append(b)               # tie: lower index
    c = a.copy(); c[0] = np.nan; rows.append(c)                               # NaN first: 0
    d = a.copy(); d[1000] = np.nan; d[2000] = np.float32(50); rows.append(d)  # NaN skipped
    e = np.full(129280, -np.inf, np.float32); rows.append(e)                  # all -inf: 0
    f = np.zeros(129280, np.float32); f[:10] = -0.0; f[3] = 0.0; rows.append(f)  # -0 == +0: 0
    g = np.full(129280, np.nan, np.float32); g[9] = 1.0; g[0] = 2.0; rows.append(g)
    lg = np.stack(rows)
    best = torch.empty(len(rows), dtype=torch.int32, device="cuda")
    dev.argmax(best, torch.from_numpy(lg).cuda(), lg.shape[1], len(rows))
    got = best.cpu().numpy()
    want = [ref_argmax(r.tolist()) for r in lg]
    assert got.tolist() == want


def test_head_bf16_logits_and_pick(dev, orc):
    """The output head: BF16 logits with the reference's bits, then the pick."""
    import torch
    rng = np.random.default_rng(22)
    rows, cols, nt = 12800, 4096, 2
    W = pack.bf16_bits((rng.standard_normal((rows, cols)) * 0.05).astype(np.float32))
    x = rng.standard_normal((nt, cols)).astype(np.float32)
    want = orc.mmq(x, oracle.qmat(W, None, 1, rows, cols))
    logits = torch.empty((nt, rows), dtype=torch.float32, device="cuda")
    best = torch.empty(nt, dtype=torch.int32, device="cuda")
    dW = torch.from_numpy(W).cuda()
    dev.head(logits, best, torch.from_numpy(x).cuda(), dev.qmat(dW, None, 1, rows, cols), nt)
    got = logits.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert best.cpu().numpy().tolist() == [int(np.argmax(want[t])) for t in range(nt)]


def test_fp8_n_fp4_n_bf16_n_entry_points(host, orc):
    rng = np.random.default_rng(4)
    W8, S8 = make_weights(rng, 2, 256, 512, 128, 128)
    W4, S4 = make_weights(rng, 3, 256, 512, 1, 32)
    Wb, _ = make_weights(rng, 1, 64, 512, 0, 0)
    x = rng.standard_normal((2, 512)).astype(np.float32)
    assert_close(host.fp8_n(x, W8, S8, 256, 512, 128, 128), orc.mmq(x, oracle.qmat(W8, S8, 2, 256, 512, 128, 128)))
    assert_close(host.fp4_n(x, W4, S4, 256, 512, 1, 32), orc.mmq(x, oracle.qmat(W4, S4, 3, 256, 512, 1, 32)))
    assert_close(host.bf16_n(x, Wb, 64, 512), orc.mmq(x, oracle.qmat(Wb, None, 1, 64, 512)))


def test_prefill_seam(host, orc):
    """dsv4_prefill_vk_* keep their 0 / -1 contract and the GEMM / expert math."""
    import ctypes as C
    import dsv4cu
    L = dsv4cu.lib()
    v = C.c_void_p()
    assert L.dsv4_prefill_vk_init(C.byref(v), None, None, None) == 0
    rng = np.random.default_rng(12)
    W, S = make_weights(rng, 2, 256, 512, 128, 128)
    x = rng.standard_normal((17, 512)).astype(np.float32)
    y = np.zeros((17, 256), np.float32)
    m = dsv4cu.QMat(W.ctypes.data, S.ctypes.data, 2, 256, 512, 128, 128)
    assert L.dsv4_prefill_vk_gemm(v, y.ctypes.data, x.ctypes.data, C.byref(m), 17) == 0
    assert_close(y, orc.mmq(x, oracle.qmat(W, S, 2, 256, 512, 128, 128)))
    g = dict(golden("expert.npz"))
    mats = [dsv4cu.QMat(g[f"fp4_{n}_W"].ctypes.data, g[f"fp4_{n}_S"].ctypes.data, 3, r, c, 1, 32)
            for n, r, c in (("w1", 256, 512), ("w3", 256, 512), ("w2", 512, 256))]
    xe = np.repeat(g["fp4_x"][None], 3, 0)
    ye = np.zeros((3, 512), np.float32)
    calls = []
    FILL = C.CFUNCTYPE(C.c_int, C.c_void_p)
    fill = FILL(lambda ctx: (calls.append(1), 0)[1])
    assert L.dsv4_prefill_vk_expert_fused(v, ye.ctypes.data, xe.ctypes.data, C.byref(mats[0]),
                                          C.byref(mats[1]), C.byref(mats[2]), 3, 256,
                                          C.c_float(10.0), fill, None) == 0
    for t in range(3):
        assert_close(ye[t], g["fp4_out"], "expert_fused")
    L.dsv4_prefill_vk_free(v)


GEMV_SHAPES = [
    # (wdt, rows, cols, blk_r, blk_c, nt): dsv4cu_gemv (streamed GEMV; other
    # shapes take dsv4cu_mmq)
    (2, 7168, 7168, 128, 128, 1),
    (2, 4096, 8192, 128, 128, 2),     # wo_b, two tokens
    (2, 1024, 4096, 128, 128, 1),     # wq_a: fewer row groups than SMs
    (3, 2048, 4096, 1, 32, 1),        # routed w1/w3
    (3, 4096, 2048, 1, 32, 2),        # routed w2
    (3, 512, 8192, 1, 32, 1),         # FP4 rows wider than one 1 KB stage
    (3, 77, 160, 1, 32, 2),           # not streamable: falls back to dsv4cu_mmq
    (2, 129, 320, 128, 128, 1),       # not streamable: falls back to dsv4cu_mmq
]


@pytest.mark.parametrize("shape", GEMV_SHAPES, ids=lambda s: "w%d_%dx%d_b%dx%d_nt%d" % s)
def test_gemv_stream_vs_oracle(dev, orc, shape):
    """dsv4cu_gemv against the oracle (the reference's matvec within the
    matmul tolerance), bit-identical run to run; an FP8 NaN code makes its
    row NaN as in the reference."""
    import torch
    wdt, rows, cols, br, bc, nt = shape
    rng = np.random.default_rng(rows * 7 + cols + nt)
    W, S = make_weights(rng, wdt, rows, cols, br, bc)
    if wdt == 2:
        W[rows // 2, cols - 3] = 0x7F
    x = pack.bf16_round(rng.standard_normal((nt, cols)).astype(np.float32))
    want = orc.mmq(x, oracle.qmat(W, S, wdt, rows, cols, br, bc))
    dW, dS, dx = (torch.from_numpy(a).cuda() for a in (W, S, x))
    m = dev.qmat(dW, dS, wdt, rows, cols, br, bc)
    y = torch.empty((nt, rows), dtype=torch.float32, device="cuda")
    y2 = torch.empty_like(y)
    dev.gemv(y, dx, m, nt)
    dev.gemv(y2, dx, m, nt)
    torch.cuda.synchronize()
    dev.check_status()
    got = y.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), y2.cpu().numpy().view(np.uint32))
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan), shape
    assert_close(np.where(nan, 0, got), np.where(nan, 0, want), shape)


def test_registry_refill_in_unsampled_bytes(host):
    """The host-pointer registry's content check. A refill confined to bytes
    the sampled fingerprint skips keeps the old HBM mirror (the documented
    limit); dsv4cu_host_forget or exact checking (dsv4cu_host_verify(1)) make
    the new bytes count. A refill that touches a sampled word is re-uploaded."""
    import dsv4cu
    rng = np.random.default_rng(11)
    rows, cols = 64, 1024                    # 64 KiB of e4m3: 16 pages
    W, S = make_weights(rng, 2, rows, cols, 128, 128)
    x = pack.bf16_round(rng.standard_normal((1, cols)).astype(np.float32))
    m = dsv4cu.QMat(W.ctypes.data, S.ctypes.data, 2, rows, cols, 128, 128)
    y0 = host.mmq(x, m)

    def bump(off):
        r, c = divmod(off, cols)
        W[r, c] = W[r, c] ^ 0x01 if (W[r, c] ^ 0x01) & 0x7F != 0x7F else W[r, c] ^ 0x02
        return r

    r1 = bump(2 * 4096 + 100)                # inside page 2, not a sampled word
    assert np.array_equal(host.mmq(x, m), y0)             # stale mirror: the documented limit
    host.forget(W.ctypes.data)
    y1 = host.mmq(x, m)
    assert y1[0, r1] != y0[0, r1]
    assert_close(y1, orc_mmq(W, S, x))
    host.verify(True)
    try:
        r2 = bump(5 * 4096 + 300)
        y2 = host.mmq(x, m)
        assert y2[0, r2] != y1[0, r2]
        assert_close(y2, orc_mmq(W, S, x))
    finally:
        host.verify(False)
    r3 = bump(7 * 4096)                      # a sampled word: seen without help
    y3 = host.mmq(x, m)
    assert y3[0, r3] != y2[0, r3]
    assert_close(y3, orc_mmq(W, S, x))


def orc_mmq(W, S, x):
    return oracle.Oracle().mmq(x, oracle.qmat(W, S, 2, W.shape[0], W.shape[1], 128, 128))
