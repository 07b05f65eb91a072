"""dsv4cu_hc_pre / dsv4cu_hc_post against the oracle's dsv4_hc_pre / dsv4_hc_post
(src/10_compute/dsv4_hc.c), and
dsv4cu_rmsnorm against the oracle's dsv4_rmsnorm (src/10_compute/dsv4_ops.c:26-33),
bit for bit: ordinary rows of the engine's widths, many rows at once (the
parallel sum with its rounding certificate), and rows that take the
sequential replay (a zero row, NaN, inf), subnormal inputs, and y aliasing x."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(dev, x, w, eps):
    import torch
    nt, n = x.shape
    dx = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    dy = torch.empty_like(dx)
    dev.rmsnorm(dy, dx, torch.from_numpy(w).cuda(), n, nt, eps)
    return dy.cpu().numpy(), dx


def _want(orc, x, w, eps):
    return np.stack([orc.rmsnorm(r, w, eps) for r in x])


@pytest.mark.parametrize("n", [1, 7, 512, 4096, 7168])
def test_rmsnorm_bitwise(dev, orc, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((6, n)) * np.array([1e-3, 0.1, 1, 3, 40, 1e4])[:, None]).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    got, _ = _run(dev, x, w, 1e-6)
    assert np.array_equal(got.view(np.uint32), _want(orc, x, w, 1e-6).view(np.uint32))


def test_rmsnorm_many_rows(dev, orc):
    rng = np.random.default_rng(3)
    n, nt = 4096, 1500
    x = (rng.standard_normal((nt, n)) * rng.uniform(0.01, 10, (nt, 1))).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    got, _ = _run(dev, x, w, 1e-6)
    assert np.array_equal(got.view(np.uint32), _want(orc, x, w, 1e-6).view(np.uint32))


def test_rmsnorm_replay_rows_and_alias(dev, orc):
    import torch
    rng = np.random.default_rng(4)
    n = 1024
    x = rng.standard_normal((5, n)).astype(np.float32)
    x[0] = 0.0
    x[1, 17] = np.nan
    x[2, 5] = np.inf
    x[3] *= np.float32(1e-40)          # float subnormal inputs
    w = rng.standard_normal(n).astype(np.float32)
    got, _ = _run(dev, x, w, 1e-6)
    want = _want(orc, x, w, 1e-6)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    fin = ~np.isnan(want)
    assert np.array_equal(got[fin].view(np.uint32), want[fin].view(np.uint32))
    # in place: y aliases x
    dx = torch.from_numpy(x[4:].copy()).cuda()
    dev.rmsnorm(dx, dx, torch.from_numpy(w).cuda(), n, 1, 1e-6)
    assert np.array_equal(dx.cpu().numpy().view(np.uint32), want[4:].view(np.uint32))


def test_rmsnorm_reference_symbol(host, orc):
    """dsv4_rmsnorm, the reference's host-pointer symbol (src/10_compute/dsv4_kernels.h:20)."""
    rng = np.random.default_rng(8)
    for n in (7, 4096):
        x = rng.standard_normal(n).astype(np.float32)
        w = rng.standard_normal(n).astype(np.float32)
        assert np.array_equal(host.rmsnorm(x, w, 1e-6).view(np.uint32), orc.rmsnorm(x, w, 1e-6).view(np.uint32))


@pytest.mark.parametrize("hc,hidden", [(4, 4096), (4, 7), (2, 130)])
def test_hc_post_bitwise(dev, orc, hc, hidden):
    import torch
    rng = np.random.default_rng(hc * 1000 + hidden)
    nt = 3
    x = rng.standard_normal((nt, hidden)).astype(np.float32)
    res = rng.standard_normal((nt, hc, hidden)).astype(np.float32)
    post = rng.uniform(0, 2, (nt, hc)).astype(np.float32)
    comb = rng.uniform(0, 1, (nt, hc, hc)).astype(np.float32)
    y = torch.empty((nt, hc, hidden), dtype=torch.float32, device="cuda")
    dev.hc_post(y, *(torch.from_numpy(a).cuda() for a in (x, res, post, comb)), nt, hc, hidden)
    got = y.cpu().numpy()
    for t in range(nt):
        want = orc.hc_post(x[t], res[t], post[t], comb[t])
        assert np.array_equal(got[t].view(np.uint32), want.view(np.uint32)), t


@pytest.mark.parametrize("hc,hidden", [(4, 4096), (4, 35), (2, 64)])
def test_hc_pre_vs_oracle(dev, orc, hc, hidden):
    """The dots, sums and float arithmetic are the reference's; only expf is not
    glibc's (exp in double rounded to float), so the bar is 1e-6 relative, and
    the test reports how many outputs match bit for bit."""
    import torch
    rng = np.random.default_rng(hc * 100 + hidden)
    nt, mix = 4, (2 + hc) * hc
    x = rng.standard_normal((nt, hc, hidden)).astype(np.float32)
    fn = (rng.standard_normal((mix, hc * hidden)) * 0.02).astype(np.float32)
    base = rng.standard_normal(mix).astype(np.float32)
    scale = rng.uniform(0.5, 2, 3).astype(np.float32)
    t = torch
    y = t.empty((nt, hidden), dtype=t.float32, device="cuda")
    post = t.empty((nt, hc), dtype=t.float32, device="cuda")
    comb = t.empty((nt, hc, hc), dtype=t.float32, device="cuda")
    mixes = t.empty((nt, mix), dtype=t.float32, device="cuda")
    dev.hc_pre(y, post, comb, mixes, *(t.from_numpy(a).cuda() for a in (x, fn, base, scale)), nt, hc, hidden)
    got = [a.cpu().numpy() for a in (y, post, comb, mixes)]
    same = total = 0
    for k in range(nt):
        want = orc.hc_pre(x[k], fn, base, scale, 20, 1e-6, 1e-6)
        # the dots and rsqrt do not involve expf: mixes are bit-exact
        assert np.array_equal(got[3][k].view(np.uint32), want[3].view(np.uint32))
        for g, w in zip(got[:3], want[:3]):
            gk = g[k]
            assert float(np.abs(gk - w).max()) <= 1e-6 * max(float(np.abs(w).max()), 1e-30)
            same += int(np.sum(gk.view(np.uint32) == w.view(np.uint32)))
            total += gk.size
    print(f"hc_pre: {same} of {total} outputs bit-identical")


def test_head_path_hc_norm_gemv_pick(dev, orc):
    """dsv4_head_from_h (src/90_cli/dsv4_decode.c:138-148) on the device: hc_head,
    the final RMS norm, the BF16 head and the greedy pick, against the oracle's
    restatements step by step (hc_head's expf aside, the same bits)."""
    import torch
    import oracle
    import pack
    rng = np.random.default_rng(31)
    hc, hidden, vocab, nt = 4, 1024, 3000, 2
    x = rng.standard_normal((nt, hc, hidden)).astype(np.float32)
    fn = (rng.standard_normal((hc, hc * hidden)) * 0.02).astype(np.float32)
    base = rng.standard_normal(hc).astype(np.float32)
    scale = np.array([1.3], np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    W = pack.bf16_bits((rng.standard_normal((vocab, hidden)) * 0.05).astype(np.float32))
    t = torch
    h = t.empty((nt, hidden), dtype=t.float32, device="cuda")
    dev.hc_head(h, t.from_numpy(x).cuda(), t.from_numpy(fn).cuda(), t.from_numpy(base).cuda(),
                t.from_numpy(scale).cuda(), nt, hc, hidden)
    dev.rmsnorm(h, h, t.from_numpy(norm_w).cuda(), hidden, nt, 1e-6)
    logits = t.empty((nt, vocab), dtype=t.float32, device="cuda")
    best = t.empty(nt, dtype=t.int32, device="cuda")
    dev.head(logits, best, h, dev.qmat(t.from_numpy(W).cuda(), None, 1, vocab, hidden), nt)
    got_h, got_l, got_b = h.cpu().numpy(), logits.cpu().numpy(), best.cpu().numpy()
    for k in range(nt):
        hh = orc.hc_head(x[k], fn, base, scale, 1e-6, 1e-6)
        hn = orc.rmsnorm(hh, norm_w, 1e-6)
        assert float(np.abs(got_h[k] - hn).max()) <= 1e-6 * float(np.abs(hn).max())
        want = orc.mmq(got_h[k][None], oracle.qmat(W, None, 1, vocab, hidden))[0]   # the head itself is exact
        assert np.array_equal(got_l[k].view(np.uint32), want.view(np.uint32))
        assert int(got_b[k]) == int(np.argmax(want))
        print(f"head path token {k}: normalised state bit-identical: {np.array_equal(got_h[k].view(np.uint32), hn.view(np.uint32))}")


@pytest.mark.parametrize("ratio", [4, 8, 128])
def test_compress_steps_vs_oracle(dev, orc, ratio):
    """dsv4cu_compress_step over several windows against the oracle's
    dsv4_compress_step (pinned live to the reference): the emit contract and the
    ring states bit for bit, the pooled rows within 1e-6 (expf) and counted
    bit-identical. The score ring starts at -inf as the reference requires, so
    the first windows pool over unfilled slots; in the second window every
    score is -inf, so with no overlap (ratio 8, 128) its emitted row is 0."""
    import torch
    rng = np.random.default_rng(ratio + 1)
    d = 128
    coff = 2 if ratio == 4 else 1
    width = coff * d
    ape = rng.standard_normal((ratio, width)).astype(np.float32)
    ks = np.zeros((coff * ratio, width), np.float32)
    ss = np.full((coff * ratio, width), -np.inf, np.float32)
    dks = torch.zeros((coff * ratio, width), dtype=torch.float32, device="cuda")
    dss = torch.full((coff * ratio, width), float("-inf"), dtype=torch.float32, device="cuda")
    zero_rows = 0
    dape = torch.from_numpy(ape).cuda()
    out = torch.empty(d, dtype=torch.float32, device="cuda")
    same = total = 0
    for pos in range(3 * ratio):
        kv = rng.standard_normal(width).astype(np.float32)
        sc = rng.standard_normal(width).astype(np.float32)
        sc[rng.integers(0, width, 2)] = -np.inf
        if ratio <= pos < 2 * ratio:
            sc[:] = -np.inf
        r_want, o_want = orc.compress_step(kv, sc, ape, ks, ss, pos, ratio, d)
        r_got = dev.compress_step(out, torch.from_numpy(kv).cuda(), torch.from_numpy(sc).cuda(), dape, dks, dss, pos,
                                  ratio, d)
        assert r_got == r_want
        if r_got:
            got = out.cpu().numpy()
            assert float(np.abs(got - o_want).max()) <= 1e-6 * max(float(np.abs(o_want).max()), 1e-30)
            same += int(np.sum(got.view(np.uint32) == o_want.view(np.uint32)))
            total += d
            if coff == 1 and pos == 2 * ratio - 1:
                assert not np.any(got) and not np.any(o_want)
                zero_rows += 1
        assert np.array_equal(dks.cpu().numpy().view(np.uint32), ks.view(np.uint32))
        assert np.array_equal(dss.cpu().numpy().view(np.uint32), ss.view(np.uint32))
    assert zero_rows == (1 if coff == 1 else 0)
    print(f"compress ratio {ratio}: {same} of {total} pooled values bit-identical")
