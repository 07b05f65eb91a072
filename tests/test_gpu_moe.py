"""Fused MoE decode step (router + routed FP4 experts + FP8 shared expert +
k-order combine) against the CPU oracle; router indices and weights bit-exact.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import canary
import oracle
import pack

pytestmark = pytest.mark.gpu


def rel_err(got, want):
    return float(np.abs(got.astype(np.float64) - want).max()) / max(float(np.abs(want).max()), 1e-30)


class MoeFixture:
    """Device-resident synthetic MoE layer (routed FP4, shared FP8 or FP4)."""

    def __init__(self, dev, n_experts, hidden, inter, shared_fmt=2, seed=0, routed_fmt=3):
        import torch
        import dsv4cu
        self.dev, self.torch = dev, torch
        self.E, self.H, self.I = n_experts, hidden, inter
        self.bufs = []
        descs = []
        for e in range(n_experts):
            descs.append(self._expert(routed_fmt, seed * 1000 + e))
        self.experts_host = descs
        self.shared = self._expert(shared_fmt, seed * 1000 + 999) if shared_fmt else None
        self.layer = dev.moe_create([d[0] for d in descs], None if self.shared is None else self.shared[0],
                                    hidden, inter)

    def close(self):
        self.dev.moe_destroy(self.layer)

    def _mat(self, fmt, rows, cols, seed):
        import dsv4cu
        t = self.torch
        src = t.empty(rows * cols, dtype=t.float32, device="cuda")
        self.dev.fill_normal(src, seed, 0.0, 0.02)
        if fmt == 3:
            W = t.empty(rows * cols // 2, dtype=t.uint8, device="cuda")
            S = t.empty(rows * cols // 32, dtype=t.uint8, device="cuda")
            self.dev.quantize_fp4(W, S, src, rows, cols)
            q = dsv4cu.QMat(W.data_ptr(), S.data_ptr(), 3, rows, cols, 1, 32)
        else:
            W = t.empty(rows * cols, dtype=t.uint8, device="cuda")
            S = t.empty(((rows + 127) // 128) * ((cols + 127) // 128), dtype=t.uint8, device="cuda")
            self.dev.quantize_fp8(W, S, src, rows, cols)
            q = dsv4cu.QMat(W.data_ptr(), S.data_ptr(), 2, rows, cols, 128, 128)
        self.bufs += [W, S]
        return q, W, S

    def _expert(self, fmt, seed):
        import dsv4cu
        m1 = self._mat(fmt, self.I, self.H, seed * 3 + 1)
        m3 = self._mat(fmt, self.I, self.H, seed * 3 + 2)
        m2 = self._mat(fmt, self.H, self.I, seed * 3 + 3)
        return dsv4cu.Expert(m1[0], m3[0], m2[0]), (m1, m3, m2)

    def host_expert(self, d):
        """Copy one expert to host numpy and describe it for the oracle."""
        mats, keep = [], []
        for (q, W, S) in d[1]:
            Wh, Sh = W.cpu().numpy(), S.cpu().numpy()
            keep += [Wh, Sh]
            mats.append(oracle.qmat(Wh, Sh, q.wdt, q.rows, q.cols, q.blk_r, q.blk_c))
        return mats, keep

    def oracle_out(self, orc, x, logits, topk, scale, limit, bias=None, tid2eid=None, token_id=0):
        idx, wts, _, _ = orc.route(logits, topk, scale, bias, tid2eid, token_id)
        keep = []
        dummy = np.zeros(16, np.uint8)
        experts = [[oracle.qmat(dummy, dummy, 3, 1, 32, 1, 32)] * 3 for _ in range(self.E)]
        for e in set(idx.tolist()):
            mats, k = self.host_expert(self.experts_host[e])
            keep += k
            experts[e] = mats
        shared = None
        if self.shared is not None:
            shared, k = self.host_expert(self.shared)
            keep += k
        else:
            shared = None
        if shared is None:
            out = np.zeros(self.H, np.float32)
            for k_, e in enumerate(idx):
                out += np.float32(wts[k_]) * orc.expert_forward(x, experts[e], self.I, limit)
            return out, idx, wts
        out, i2, w2 = orc.moe_decode(x, logits, experts, shared, topk, scale, self.H, self.I, limit,
                                     bias, tid2eid, token_id)
        return out, i2, w2


def run(dev, fx, x, logits, topk, scale, limit, bias=None, tid2eid=None, token_ids=None):
    t = fx.torch
    nt = x.shape[0]
    dx = t.from_numpy(x).cuda()
    dl = t.from_numpy(logits).cuda()
    out = canary.guarded_empty((nt, fx.H))
    idx = canary.guarded_empty((nt, topk), t.int32)
    wts = canary.guarded_empty((nt, topk))
    db = None if bias is None else t.from_numpy(bias).cuda()
    dt = None if tid2eid is None else t.from_numpy(tid2eid).cuda()
    dtok = None if token_ids is None else t.from_numpy(token_ids).cuda()
    dev.moe_decode(fx.layer, out, dx, dl, topk, scale, limit, nt, idx, wts, db, dt, dtok)
    for buf, what in ((out, "moe_decode out"), (idx, "moe_decode idx"), (wts, "moe_decode wts")):
        canary.check(buf, what)
    return out.cpu().numpy(), idx.cpu().numpy(), wts.cpu().numpy()


@pytest.mark.parametrize("nt", [1, 2, 5])
def test_moe_small_vs_oracle(dev, orc, nt):
    fx = MoeFixture(dev, 16, 512, 256, shared_fmt=2, seed=nt)
    rng = np.random.default_rng(nt)
    x = pack.bf16_round(rng.standard_normal((nt, 512)).astype(np.float32))
    logits = pack.bf16_round(rng.standard_normal((nt, 16)).astype(np.float32))
    out, idx, wts = run(dev, fx, x, logits, 4, 1.5, 10.0)
    for t in range(nt):
        want, widx, wwts = fx.oracle_out(orc, x[t], logits[t], 4, 1.5, 10.0)
        assert np.array_equal(idx[t], widx)
        assert np.array_equal(wts[t].view(np.uint32), wwts.view(np.uint32))
        assert rel_err(out[t], want) <= 1e-3, rel_err(out[t], want)
        assert rel_err(out[t], want) <= 1e-5


def test_moe_bias_hash_noshared(dev, orc):
    fx = MoeFixture(dev, 16, 512, 256, shared_fmt=0, seed=7)
    rng = np.random.default_rng(17)
    x = pack.bf16_round(rng.standard_normal((3, 512)).astype(np.float32))
    logits = rng.standard_normal((3, 16)).astype(np.float32)
    bias = (rng.standard_normal(16) * 0.5).astype(np.float32)
    logits = pack.bf16_round(logits)
    out, idx, wts = run(dev, fx, x, logits, 4, 2.5, 10.0, bias=bias)
    for t in range(3):
        want, widx, wwts = fx.oracle_out(orc, x[t], logits[t], 4, 2.5, 10.0, bias=bias)
        assert np.array_equal(idx[t], widx)
        assert rel_err(out[t], want) <= 1e-5
    tid = rng.integers(0, 16, (11, 4)).astype(np.int64)
    toks = np.array([3, 10, 3], np.int32)
    out, idx, wts = run(dev, fx, x, logits, 4, 1.5, 10.0, tid2eid=tid, token_ids=toks)
    for t in range(3):
        want, widx, _ = fx.oracle_out(orc, x[t], logits[t], 4, 1.5, 10.0, tid2eid=tid, token_id=int(toks[t]))
        assert np.array_equal(idx[t], tid[toks[t]])
        assert rel_err(out[t], want) <= 1e-5


@pytest.mark.parametrize("path", ["tensor", "stream"])
def test_moe_full_config2(dev, orc, path):
    """BASELINE config 2 geometry: 256 FP4 experts 2048x4096 / 4096x2048, top-8,
    FP8 shared expert, hidden 4096, route_scale 1.5, SwiGLU limit 10; both
    decode paths."""
    fx = MoeFixture(dev, 256, 4096, 2048, shared_fmt=2, seed=42)
    dev.moe_set_path(fx.layer, path)
    rng = np.random.default_rng(2)
    for trial in range(2):
        x = pack.bf16_round(rng.standard_normal((1, 4096)).astype(np.float32))
        logits = pack.bf16_round(rng.standard_normal((1, 256)).astype(np.float32))
        out, idx, wts = run(dev, fx, x, logits, 8, 1.5, 10.0)
        want, widx, wwts = fx.oracle_out(orc, x[0], logits[0], 8, 1.5, 10.0)
        assert np.array_equal(idx[0], widx)
        assert np.array_equal(wts[0].view(np.uint32), wwts.view(np.uint32))
        assert rel_err(out[0], want) <= 1e-5, rel_err(out[0], want)


@pytest.mark.parametrize("shared_fmt,nt", [(2, 1), (3, 2), (0, 1), (0, 2)])
def test_moe_stream_path_vs_oracle(dev, orc, shared_fmt, nt):
    """The streamed decode path (forced) against the oracle, with an FP8, an
    FP4 or no shared expert, one or two tokens; two runs agree bit for bit."""
    fx = MoeFixture(dev, 16, 1024, 512, shared_fmt=shared_fmt, seed=20 + nt)
    dev.moe_set_path(fx.layer, "stream")
    rng = np.random.default_rng(30 + shared_fmt)
    x = pack.bf16_round(rng.standard_normal((nt, 1024)).astype(np.float32))
    logits = pack.bf16_round(rng.standard_normal((nt, 16)).astype(np.float32))
    out, idx, wts = run(dev, fx, x, logits, 6, 1.5, 10.0)
    again, _, _ = run(dev, fx, x, logits, 6, 1.5, 10.0)
    assert np.array_equal(out.view(np.uint32), again.view(np.uint32))
    for t in range(nt):
        want, widx, wwts = fx.oracle_out(orc, x[t], logits[t], 6, 1.5, 10.0)
        assert np.array_equal(idx[t], widx)
        assert np.array_equal(wts[t].view(np.uint32), wwts.view(np.uint32))
        assert rel_err(out[t], want) <= 1e-5, rel_err(out[t], want)
    fx.close()


def test_moe_set_path_rejects(dev):
    fx = MoeFixture(dev, 4, 512, 256, shared_fmt=0, seed=3)
    assert dev.L.dsv4cu_moe_set_path(fx.layer, 7) != 0
    dev.moe_set_path(fx.layer, "auto")
    fx.close()


def test_router_bitexact_vs_reference_golden(dev):
    from conftest import golden
    t = __import__("torch")
    g = dict(golden("route.npz"))
    T = g["logits"].shape[0]
    for tag, b, tid in (("plain", None, None), ("bias", g["bias"], None), ("hash", None, g["tid2eid"])):
        idx = t.empty((T, 8), dtype=t.int32, device="cuda")
        wts = t.empty((T, 8), dtype=t.float32, device="cuda")
        sc = t.empty((T, 256), dtype=t.float32, device="cuda")
        orig = t.empty((T, 256), dtype=t.float32, device="cuda")
        toks = t.tensor([(i * 7) % 97 for i in range(T)], dtype=t.int32, device="cuda")
        dev.route(idx, wts, sc, orig, t.from_numpy(g["logits"]).cuda(), 8, 1.5, T,
                  None if b is None else t.from_numpy(b).cuda(),
                  None if tid is None else t.from_numpy(tid).cuda(), toks)
        t.cuda.synchronize()
        assert np.array_equal(idx.cpu().numpy(), g[f"{tag}_idx"])
        assert np.array_equal(wts.cpu().numpy().view(np.uint32), g[f"{tag}_wts"].view(np.uint32))
        assert np.array_equal(orig.cpu().numpy().view(np.uint32), g[f"{tag}_orig"].view(np.uint32))
        assert np.array_equal(sc.cpu().numpy().view(np.uint32), g[f"{tag}_scores"].view(np.uint32))


def test_router_random_bitexact_and_host_abi(dev, host, orc):
    """bf16-valued logits (the configs' router input): indices and weights
    bit-exact. Arbitrary fp32 logits: indices exact, weights within 2 ulp
    (glibc's log1pf is not correctly rounded; the device rounds correctly)."""
    t = __import__("torch")
    rng = np.random.default_rng(99)
    T = 512
    raw = (rng.standard_normal((T, 256)) * rng.uniform(0.2, 6, (T, 1))).astype(np.float32)
    for exact, logits in ((True, pack.bf16_round(raw)), (False, raw)):
        logits = logits.copy()
        logits[0, 5] = logits[0, 9] = 3.0     # exact ties go to the lower index
        idx = t.empty((T, 8), dtype=t.int32, device="cuda")
        wts = t.empty((T, 8), dtype=t.float32, device="cuda")
        dev.route(idx, wts, None, None, t.from_numpy(logits).cuda(), 8, 1.5, T)
        t.cuda.synchronize()
        idx, wts = idx.cpu().numpy(), wts.cpu().numpy()
        for i in range(T):
            ri, rw, _, _ = orc.route(logits[i], 8, 1.5)
            assert np.array_equal(idx[i], ri), i
            if exact:
                assert np.array_equal(wts[i].view(np.uint32), rw.view(np.uint32)), i
            else:
                ulp = np.abs(wts[i].view(np.int32).astype(np.int64) - rw.view(np.int32).astype(np.int64))
                assert ulp.max() <= 2, (i, ulp)
    lb = pack.bf16_round(raw)
    for i in range(8):
        hi, hw, hs, ho = host.route(lb[i], 8, 1.5)
        oi, ow, os_, oo = orc.route(lb[i], 8, 1.5)
        assert np.array_equal(hi, oi) and np.array_equal(hw.view(np.uint32), ow.view(np.uint32))
        assert np.array_equal(ho.view(np.uint32), oo.view(np.uint32))


def test_swiglu_and_expert_forward_host_abi(host, orc):
    from conftest import golden
    g = dict(golden("expert.npz"))
    import dsv4cu
    for tag, fmt, br, bc in (("fp4", 3, 1, 32), ("fp8", 2, 128, 128)):
        mats = [dsv4cu.QMat(g[f"{tag}_{n}_W"].ctypes.data, g[f"{tag}_{n}_S"].ctypes.data, fmt, r, c, br, bc)
                for n, r, c in (("w1", 256, 512), ("w3", 256, 512), ("w2", 512, 256))]
        out, gate, up, mid = host.expert_forward(g[f"{tag}_x"], mats, 256, 10.0)
        assert rel_err(out, g[f"{tag}_out"]) <= 1e-5
        assert rel_err(mid, orc.swiglu(gate, up, 10.0)) <= 1e-6
    gate = np.array([1.0, -50.0, 50.0, 10.0, 3.0], np.float32)
    up = np.array([-50.0, 1.0, 1.0, 1.0, 50.0], np.float32)
    for lim in (10.0, 0.0):
        got = host.swiglu(gate, up, lim)
        want = orc.swiglu(gate, up, lim)
        assert np.allclose(got, want, rtol=1e-6, atol=1e-30)
    assert got.dtype == np.float32


def test_moe_batch40_nan_and_ties(dev, orc):
    """40 tokens over 32 experts (one warp per token routes, 160 pairs bucket by
    per-expert counts), then the small-batch path with a NaN score and a row of
    equal scores (ties go to the lower index; a NaN is never preferred unless it
    is the first candidate)."""
    fx = MoeFixture(dev, 32, 512, 256, shared_fmt=2, seed=40)
    rng = np.random.default_rng(40)
    x = pack.bf16_round(rng.standard_normal((40, 512)).astype(np.float32))
    logits = pack.bf16_round(rng.standard_normal((40, 32)).astype(np.float32))
    out, idx, wts = run(dev, fx, x, logits, 4, 1.5, 10.0)
    for t in range(40):
        want, widx, wwts = fx.oracle_out(orc, x[t], logits[t], 4, 1.5, 10.0)
        assert np.array_equal(idx[t], widx), t
        assert np.array_equal(wts[t].view(np.uint32), wwts.view(np.uint32)), t
        assert rel_err(out[t], want) <= 1e-5, (t, rel_err(out[t], want))
    x2 = x[:2].copy()
    lg2 = logits[:2].copy()
    lg2[0, 5] = np.nan
    lg2[1, :] = np.float32(0.5)
    out, idx, wts = run(dev, fx, x2, lg2, 4, 1.5, 10.0)
    for t in range(2):
        want, widx, wwts = fx.oracle_out(orc, x2[t], lg2[t], 4, 1.5, 10.0)
        assert np.array_equal(idx[t], widx), (t, idx[t], widx)
        assert np.array_equal(wts[t].view(np.uint32), wwts.view(np.uint32)), t
        assert rel_err(out[t], want) <= 1e-5


def _oracle_batch(fx, orc, x, logits, topk, scale, limit):
    """Oracle MoE output of every token; all experts copied to the host once."""
    cache = [fx.host_expert(d) for d in fx.experts_host]
    experts = [c[0] for c in cache]
    shared, keep = fx.host_expert(fx.shared)
    outs, idxs, wtss = [], [], []
    for t in range(x.shape[0]):
        o, i, w = orc.moe_decode(x[t], logits[t], experts, shared, topk, scale, fx.H, fx.I, limit, None, None, 0)
        outs.append(o)
        idxs.append(i)
        wtss.append(w)
    del cache, keep
    return np.stack(outs), np.stack(idxs), np.stack(wtss)


def _prefill(dev, fx, x, logits, topk, scale, limit, terms):
    t = fx.torch
    nt = x.shape[0]
    out = canary.guarded_empty((nt, fx.H))
    idx = canary.guarded_empty((nt, topk), t.int32)
    wts = canary.guarded_empty((nt, topk))
    dev.moe_prefill(fx.layer, out, t.from_numpy(x).cuda(), t.from_numpy(logits).cuda(), topk, scale, limit, nt,
                    terms, idx, wts)
    for buf, what in ((out, "moe_prefill out"), (idx, "moe_prefill idx"), (wts, "moe_prefill wts")):
        canary.check(buf, what)
    return out.cpu().numpy(), idx.cpu().numpy(), wts.cpu().numpy()


@pytest.mark.parametrize("terms,bound", [(2, 1.5e-3), (3, 1e-4), (4, 1e-5)])
def test_moe_prefill_small_vs_oracle(dev, orc, terms, bound):
    """300 tokens over 16 experts (top-4): buckets of about 75 tokens, several
    192/256-column tiles per expert plus the shared expert over all tokens.
    Two terms (128 tokens per tile) lands at the 1e-3 matmul bar (1.0e-3 on
    this case: the activation error enters twice, before gate/up and after
    SwiGLU), so three terms stay the default."""
    fx = MoeFixture(dev, 16, 512, 256, shared_fmt=2, seed=300 + terms)
    rng = np.random.default_rng(300 + terms)
    x = pack.bf16_round(rng.standard_normal((300, 512)).astype(np.float32))
    logits = pack.bf16_round(rng.standard_normal((300, 16)).astype(np.float32))
    out, idx, wts = _prefill(dev, fx, x, logits, 4, 1.5, 10.0, terms)
    want, widx, wwts = _oracle_batch(fx, orc, x, logits, 4, 1.5, 10.0)
    assert np.array_equal(idx, widx)
    assert np.array_equal(wts.view(np.uint32), wwts.view(np.uint32))
    errs = [rel_err(out[t], want[t]) for t in range(300)]
    print(f"prefill terms={terms}: max-rel over tokens {max(errs):.3e}")
    assert max(errs) <= bound, max(errs)
    fx.close()


def test_moe_prefill_matches_decode(dev):
    """The prefill path and the decode step agree on the same tokens."""
    t = __import__("torch")
    fx = MoeFixture(dev, 16, 512, 256, shared_fmt=2, seed=77)
    rng = np.random.default_rng(77)
    x = pack.bf16_round(rng.standard_normal((48, 512)).astype(np.float32))
    logits = pack.bf16_round(rng.standard_normal((48, 16)).astype(np.float32))
    outp, idxp, wtsp = _prefill(dev, fx, x, logits, 4, 1.5, 10.0, 4)
    outd, idxd, wtsd = run(dev, fx, x, logits, 4, 1.5, 10.0)
    assert np.array_equal(idxp, idxd)
    assert np.array_equal(wtsp.view(np.uint32), wtsd.view(np.uint32))
    assert max(rel_err(outp[i], outd[i].astype(np.float64)) for i in range(48)) <= 1e-5
    fx.close()


def test_moe_prefill_config3_sampled(dev, orc):
    """BASELINE config 3 shape: 4096 tokens, 256 FP4 experts (top-8), FP8 shared
    expert; every routing result checked, outputs of 12 sampled tokens against
    the oracle (the oracle is scalar double: the full batch would take minutes)."""
    fx = MoeFixture(dev, 256, 4096, 2048, shared_fmt=2, seed=4096)
    rng = np.random.default_rng(4096)
    nt = 4096
    x = pack.bf16_round(rng.standard_normal((nt, 4096)).astype(np.float32))
    logits = pack.bf16_round(rng.random((nt, 256)).astype(np.float32))   # uniform(0,1), bf16-valued
    out, idx, wts = _prefill(dev, fx, x, logits, 8, 1.5, 10.0, 3)
    for t_ in range(nt):
        i_, w_, _, _ = orc.route(logits[t_], 8, 1.5, None, None, 0)
        assert np.array_equal(idx[t_], i_), t_
        assert np.array_equal(wts[t_].view(np.uint32), w_.view(np.uint32)), t_
    sample = rng.choice(nt, 12, replace=False)
    for t_ in sample:
        want, _, _ = fx.oracle_out(orc, x[t_], logits[t_], 8, 1.5, 10.0)
        assert rel_err(out[t_], want) <= 1e-4, (t_, rel_err(out[t_], want))
    fx.close()


def test_moe_decode_host_matches_device_call(dev):
    """dsv4cu_moe_decode_host (host buffers, copies on the stream) gives the
    same bits as dsv4cu_moe_decode on device buffers."""
    t = __import__("torch")
    fx = MoeFixture(dev, 16, 512, 256, shared_fmt=2, seed=91)
    rng = np.random.default_rng(91)
    nt = 3
    x = pack.bf16_round(rng.standard_normal((nt, 512)).astype(np.float32))
    lg = pack.bf16_round(rng.standard_normal((nt, 16)).astype(np.float32))
    want, _, _ = run(dev, fx, x, lg, 4, 1.5, 10.0)
    hx, hl = t.from_numpy(x).pin_memory(), t.from_numpy(lg).pin_memory()
    hout = t.full((nt, 512), float("nan"), dtype=t.float32).pin_memory()
    dev.moe_decode_host(fx.layer, hout, hx, hl, 4, 1.5, 10.0, nt)
    t.cuda.synchronize()
    assert np.array_equal(hout.numpy().view(np.uint32), want.view(np.uint32))
    fx.close()
