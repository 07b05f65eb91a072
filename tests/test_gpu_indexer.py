"""Sparse-attention indexer on the B200: FP8 / fp32 scores bit-identical to the
reference, top-k indices identical (ties to the lower index), sparse attention
within tolerance; config 4 at full size (32768 keys, 64 heads x 128, top-2048).
"""
from __future__ import annotations

import numpy as np
import pytest

import canary
import kat
import pack
from conftest import golden

pytestmark = pytest.mark.gpu


def quant_rows(a):
    """e4m3 codes with one power-of-two fp32 scale per row."""
    amax = np.abs(a).max(axis=1)
    f, E = np.frexp(amax)
    e = E - 9 + (f > 0.875)
    sc = np.ldexp(np.ones_like(amax), e).astype(np.float32)
    v = np.ldexp(a, -e[:, None]).astype(np.float32)
    codes = pack._rne_grid(v, pack._E4M3_POS).astype(np.uint8)
    codes = np.where(np.signbit(v), codes | 0x80, codes).astype(np.uint8)
    return codes, sc


def dev_score(dev, q, kv, w):
    t = __import__("torch")
    h, d = q.shape
    n = kv.shape[0]
    out = canary.guarded_empty(n)
    dev.indexer_score(out, t.from_numpy(q).cuda(), t.from_numpy(kv).cuda(), t.from_numpy(w).cuda(), h, d, n)
    canary.check(out, "indexer_score")
    return out.cpu().numpy()


def dev_score8(dev, q8, qs, k8, ks, w, stride=None):
    t = __import__("torch")
    h, d = q8.shape
    n = k8.shape[0]
    stride = stride or k8.shape[1]
    out = canary.guarded_empty(n)
    dev.indexer_score_fp8(out, t.from_numpy(q8).cuda(), t.from_numpy(qs).cuda(), t.from_numpy(k8).cuda(),
                          t.from_numpy(ks).cuda(), t.from_numpy(w).cuda(), h, d, n, stride)
    canary.check(out, "indexer_score_fp8")
    return out.cpu().numpy()


def dev_topk(dev, s, k):
    t = __import__("torch")
    kk = max(0, min(k, s.size))
    out = canary.guarded_empty(max(kk, 1), t.int32)
    out.fill_(-7)
    dev.topk(out, t.from_numpy(np.ascontiguousarray(s, np.float32)).cuda(), s.size, k)
    canary.check(out, "topk")
    return out.cpu().numpy()[:kk]


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_indexer_golden_bitexact(dev, host):
    g = dict(golden("indexer.npz"))
    assert np.array_equal(bits(dev_score(dev, g["q"], g["kv"], g["w"])), bits(g["score"]))
    assert np.array_equal(bits(dev_score8(dev, g["q8"], g["qsc"], g["k8"], g["ksc"], g["w"])), bits(g["score8"]))
    assert np.array_equal(bits(dev_score(dev, g["q3"], g["k3"], g["w3"])), bits(g["score3"]))
    assert np.array_equal(bits(host.indexer_score(g["q"], g["kv"], g["w"])), bits(g["score"]))


def test_indexer_kat(host):
    out = host.indexer_score(np.array([[1, 0], [0, 0]], np.float32), np.array([[1, 0], [-1, 0]], np.float32),
                             np.array([1, 1], np.float32))
    assert out[0] > 0 and out[1] == 0.0
    out = host.indexer_score(np.eye(2, dtype=np.float32), np.eye(2, dtype=np.float32), np.array([1, 4], np.float32))
    assert abs(out[1] / out[0] - 4) < 1e-4


@pytest.mark.parametrize("h,d,n", [(64, 128, 4097), (3, 7, 50), (8, 48, 31), (1, 16, 1), (64, 256, 33),
                                   (16, 64, 5), (48, 64, 130), (32, 128, 3), (64, 128, 1)])
def test_indexer_random_bitexact(dev, orc, h, d, n):
    rng = np.random.default_rng(h * d + n)
    q = rng.standard_normal((h, d)).astype(np.float32)
    kv = rng.standard_normal((n, d)).astype(np.float32)
    w = rng.standard_normal(h).astype(np.float32)
    assert np.array_equal(bits(dev_score(dev, q, kv, w)), bits(orc.indexer_score(q, kv, w)))


def test_config4_full_fp8_score_topk(dev, orc):
    """32768 FP8 keys (per-token pow2 scale), 64 heads x 128, top-2048."""
    rng = np.random.default_rng(7)
    k8, ks = quant_rows(rng.standard_normal((32768, 128)).astype(np.float32))
    q8, qs = quant_rows(rng.standard_normal((64, 128)).astype(np.float32))
    w = rng.standard_normal(64).astype(np.float32)
    got = dev_score8(dev, q8, qs, k8, ks, w)
    kf = (pack.E4M3[k8] * ks[:, None]).astype(np.float32)
    qf = (pack.E4M3[q8] * qs[:, None]).astype(np.float32)
    want = orc.indexer_score(qf, kf, w)
    assert np.array_equal(bits(got), bits(want))
    idx = dev_topk(dev, got, 2048)
    assert np.array_equal(idx, orc.topk(want, 2048))


@pytest.mark.parametrize("path", ["auto", "fp64"])
@pytest.mark.parametrize("case", ["keys-mixed", "q-nonpow2", "zero-scale", "nan-key", "nan-q", "stride-144",
                                  "stride-136"])
def test_config4_fp8_scale_forms(dev, orc, case, path):
    """The FP8 path computes exact dots on tensor cores (int8 digit GEMMs, or
    FP64) only where every scale is a power of two and no byte is NaN, and
    replays the reference's fma chains elsewhere; key rows that are not 16-byte
    aligned take the FP64 kernel. All must give the reference's bits, in the
    same launch."""
    rng = np.random.default_rng(31 + ["keys-mixed", "q-nonpow2", "zero-scale", "nan-key", "nan-q", "stride-144",
                                      "stride-136"].index(case))
    n = 1000
    k8, ks = quant_rows(rng.standard_normal((n, 128)).astype(np.float32))
    q8, qs = quant_rows(rng.standard_normal((64, 128)).astype(np.float32))
    stride = None
    if case == "keys-mixed":
        bad = rng.random(n) < 0.05                     # a few 16-position tasks fall back
        ks = np.where(bad, ks * np.float32(1.2345), ks).astype(np.float32)
    elif case == "q-nonpow2":
        qs = (qs * np.float32(0.7771)).astype(np.float32)
    elif case == "zero-scale":
        ks[::7] = 0.0
    elif case == "nan-key":
        k8[rng.integers(0, n, 6), rng.integers(0, 128, 6)] = np.uint8(0x7F)
        k8[rng.integers(0, n, 3), rng.integers(0, 128, 3)] = np.uint8(0xFF)
    elif case == "nan-q":
        q8[5, 77] = np.uint8(0xFF)
    w = rng.standard_normal(64).astype(np.float32)
    kf = (pack.E4M3[k8] * ks[:, None]).astype(np.float32)
    qf = (pack.E4M3[q8] * qs[:, None]).astype(np.float32)
    if case.startswith("stride-"):
        stride = int(case[7:])
        padded = rng.integers(0, 256, (n, stride)).astype(np.uint8)   # garbage beyond head_dim
        padded[:, :128] = k8
        k8 = padded
    dev.indexer_set_path(path)
    try:
        got = dev_score8(dev, q8, qs, k8, ks, w, stride)
    finally:
        dev.indexer_set_path("auto")
    want = orc.indexer_score(qf, kf, w)
    assert np.array_equal(bits(got), bits(want))


def test_config4_int8_and_fp64_kernels_agree(dev):
    """Full config-4 size: the int8-digit kernel and the FP64 tensor-core
    kernel compute the same exact dots, hence the same score bits."""
    rng = np.random.default_rng(77)
    k8, ks = quant_rows(rng.standard_normal((32768, 128)).astype(np.float32) * 3.0)
    q8, qs = quant_rows(rng.standard_normal((64, 128)).astype(np.float32))
    w = rng.standard_normal(64).astype(np.float32)
    a = dev_score8(dev, q8, qs, k8, ks, w)
    dev.indexer_set_path("fp64")
    try:
        b = dev_score8(dev, q8, qs, k8, ks, w)
    finally:
        dev.indexer_set_path("auto")
    assert np.array_equal(bits(a), bits(b))
    assert np.count_nonzero(a) > 1000


def test_topk_golden_and_kat(dev, host):
    g = dict(golden("topk.npz"))
    for key in g:
        if key.endswith("_scores"):
            base = key[:-len("_scores")]
            k = int(base.split("_k")[1])
            assert np.array_equal(dev_topk(dev, g[key], k), g[base + "_idx"]), base
    s = np.array([1, 5, 5, 2, 0, 5], np.float32)
    idx, r = host.topk(s, 4)
    assert idx.tolist() == [1, 2, 5, 3] and r == 4
    idx, r = host.topk(s, 10)
    assert r == 6 and idx.tolist() == [1, 2, 5, 3, 0, 4]
    assert host.topk(s, 0)[1] == 0 and host.topk(s, -3)[1] == -3


@pytest.mark.parametrize("n,k", [(32768, 2048), (32768, 512), (1, 1), (5, 5), (100000, 1024),
                                 (3000, 8192), (65536, 8192)])
def test_topk_random_with_ties(dev, orc, n, k):
    rng = np.random.default_rng(n + k)
    s = (rng.integers(-300, 300, n) * 0.125).astype(np.float32)   # many exact ties
    s[rng.integers(0, n, max(1, n // 50))] = -0.0
    s[rng.integers(0, n, max(1, n // 50))] = 0.0
    assert np.array_equal(dev_topk(dev, s, k), orc.topk(s, k))


def test_topk_all_equal_and_extremes(dev, orc):
    s = np.zeros(5000, np.float32)
    assert np.array_equal(dev_topk(dev, s, 2048), np.arange(2048))
    s = np.array([np.inf, -np.inf, 3e38, -3e38, 1e-45, -1e-45, 0.0, -0.0], np.float32)
    assert np.array_equal(dev_topk(dev, s, 8), orc.topk(s, 8))


def test_offset_and_window(host):
    assert host.indexer_offset([0, 3, -1, 7, -1], 128).tolist() == [128, 131, -1, 135, -1]
    for pos, win, want, n in kat.window_kat():
        got, cnt = host.window_idxs(pos, win)
        assert got.tolist() == want and cnt == n


# ----------------------------------------------------------------- attention
ATT_TOL = 1e-5


def att_err(got, want):
    return float(np.abs(got.astype(np.float64) - want).max()) / max(float(np.abs(want).max()), 1e-30)


@pytest.mark.parametrize("case", kat.attn_kat(), ids=lambda c: c[0])
def test_attn_kat(host, case):
    name, q, kv, sink, idxs, scale, check = case
    o = host.sparse_attn(q, kv, sink, idxs, scale)     # head dims 2 and 4, as the reference tests them
    assert check(o), (name, o)


@pytest.mark.parametrize("d", [1, 2, 7, 130, 513])
@pytest.mark.parametrize("bf16", [0, 1])
def test_attn_any_head_dim(dev, orc, d, bf16):
    """Head dims that are not multiples of 4 (dsv4_sparse_attn takes any d):
    rows gathered element by element, tail columns stored one by one."""
    t = __import__("torch")
    rng = np.random.default_rng(d + 7 * bf16)
    H, N, T = 5, 300, 70
    kv = pack.bf16_round(rng.standard_normal((N, d)).astype(np.float32))
    q = rng.standard_normal((H, d)).astype(np.float32)
    sink = rng.standard_normal(H).astype(np.float32)
    idx = rng.choice(N, T, replace=False).astype(np.int32)
    idx[::9] = -1
    scale = np.float32(1 / np.sqrt(d))
    o = canary.guarded_empty((H, d))
    kvd = t.from_numpy(kv).cuda()
    if bf16:
        kvd = kvd.to(t.bfloat16)
    dev.sparse_attn(o, t.from_numpy(q).cuda(), kvd, bf16, t.from_numpy(sink).cuda(), t.from_numpy(idx).cuda(),
                    H, d, T, float(scale))
    canary.check(o, "sparse_attn")
    want = orc.sparse_attn(q, kv, sink, idx, scale)
    assert att_err(o.cpu().numpy(), want) <= ATT_TOL


def test_attn_golden(host):
    g = dict(golden("attn.npz"))
    o = host.sparse_attn(g["q"], g["kv"], g["sink"], g["idx"], np.float32(1 / np.sqrt(64)))
    assert att_err(o, g["o"]) <= ATT_TOL


@pytest.mark.parametrize("bf16", [0, 1])
def test_attn_config4_full(dev, orc, bf16):
    """64 heads, d = 512, 2048 indexer rows + a 128-slot window with masked slots."""
    t = __import__("torch")
    rng = np.random.default_rng(5 + bf16)
    H, D, N, T = 64, 512, 32768, 2176
    kv = pack.bf16_round(rng.standard_normal((N, D)).astype(np.float32))
    q = pack.bf16_round(rng.standard_normal((H, D)).astype(np.float32))
    sink = rng.standard_normal(H).astype(np.float32)
    idx = rng.choice(N, T, replace=False).astype(np.int32)
    idx[2048 + 100:] = -1
    scale = np.float32(1 / np.sqrt(D))
    o = canary.guarded_empty((H, D))
    kvd = t.from_numpy(kv).cuda()
    if bf16:
        kvd = kvd.to(t.bfloat16)
    dev.sparse_attn(o, t.from_numpy(q).cuda(), kvd, bf16, t.from_numpy(sink).cuda(), t.from_numpy(idx).cuda(),
                    H, D, T, float(scale))
    canary.check(o, "sparse_attn")
    want = orc.sparse_attn(q, kv, sink, idx, scale)
    assert att_err(o.cpu().numpy(), want) <= ATT_TOL


@pytest.mark.parametrize("D,H,T,qscale", [(576, 64, 2048, 1.0), (576, 16, 1000, 3.0), (512, 32, 2176, 1.0),
                                          (576, 64, 64, 0.3), (576, 64, 5000, 1.0)])
@pytest.mark.parametrize("path", ["auto", "cluster8", "fp32"])
def test_attn_tensor_core_chunks(dev, orc, D, H, T, qscale, path):
    """The bf16 tensor-core cluster kernel (fp32 q and weights as three bf16
    terms each, online softmax over each CTA's 64-row sub-chunks, combine in
    distributed shared memory) against the reference: fp32 q off the bf16
    grid, peaky softmax (qscale 3), a ragged last sub-chunk, a fully masked
    64-slot sub-chunk, scattered masked slots and fewer sub-chunks than CTAs
    (T = 64); 16- and 8-CTA clusters and the fp32 kernel on the same inputs."""
    t = __import__("torch")
    rng = np.random.default_rng(D + H + T)
    N = 8192
    kv = pack.bf16_round(rng.standard_normal((N, D)).astype(np.float32))
    q = (rng.standard_normal((H, D)) * qscale).astype(np.float32)
    sink = rng.standard_normal(H).astype(np.float32)
    idx = rng.choice(N, T, replace=False).astype(np.int32)
    idx[::13] = -1
    if T >= 256:
        idx[128:192] = -1
    scale = np.float32(1 / np.sqrt(D))
    o = canary.guarded_empty((H, D))
    kvd = t.from_numpy(kv).cuda().to(t.bfloat16)
    dev.sparse_attn_set_path(path)
    try:
        dev.sparse_attn(o, t.from_numpy(q).cuda(), kvd, 1, t.from_numpy(sink).cuda(), t.from_numpy(idx).cuda(),
                        H, D, T, float(scale))
        t.cuda.synchronize()
    finally:
        dev.sparse_attn_set_path("auto")
    canary.check(o, "sparse_attn (tensor-core cluster)")
    want = orc.sparse_attn(q, kv, sink, idx, scale)
    got = o.cpu().numpy()
    assert np.isfinite(got).all()
    assert att_err(got, want) <= ATT_TOL


@pytest.mark.parametrize("path", ["auto", "cluster8"])
def test_attn_tensor_core_all_masked(dev, path):
    """Every slot masked: the reference output is zero (denominator = sink
    only), with no NaN from the empty sub-chunks."""
    t = __import__("torch")
    H, D, T = 32, 576, 300
    q = t.randn((H, D), dtype=t.float32, device="cuda")
    kv = t.randn((1000, D), dtype=t.float32, device="cuda").to(t.bfloat16)
    sink = t.randn(H, dtype=t.float32, device="cuda")
    idx = t.full((T,), -1, dtype=t.int32, device="cuda")
    o = t.full((H, D), 7.0, dtype=t.float32, device="cuda")
    dev.sparse_attn_set_path(path)
    try:
        dev.sparse_attn(o, q, kv, 1, sink, idx, H, D, T, 0.05)
        t.cuda.synchronize()
    finally:
        dev.sparse_attn_set_path("auto")
    assert t.count_nonzero(o).item() == 0
