"""One decoder layer's attention on the device (dsv4cu_attn_step /
dsv4cu_attn_block) against the REFERENCE's own attention block running on its
CPU kernels (oracle/_ref/libdsv4layer.so: src/70_decode/dsv4_layer_attn.c
dsv4_layer_attention and the attention half of dsv4_layer_forward, behind the
harness oracle/layer_ref.c), token after token from position 0, with the same
seeded random weights uploaded to the GPU.

Covered: ratio 0 (window only), ratio 4 (overlapped compressor + the CSA
indexer with its main-cache stride, top-k truncation once more rows than
index_topk exist) and another ratio (compressor, all rows taken), at small
shapes and at the Flash shapes of BASELINE config 5 (hidden 4096, 64 heads of
512, q_lora 1024, 8 wo_a groups of 1024, window 128, 64 x 128 indexer heads,
top-512). The bar is the matmul contract, max |d| / max |ref| <= 1e-3 per token;
the compressed-row counts must match exactly."""
from __future__ import annotations

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

SMALL = [512, 8, 128, 256, 128, 4, 64, 16, 4, 64, 6, 4]
FLASH = [4096, 64, 512, 1024, 1024, 8, 64, 128, 64, 128, 512, 4]
TOL = 1e-3


def _rel(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / max(float(np.max(np.abs(b))), 1e-30))


@pytest.fixture(scope="module")
def need_layer_ref():
    if not oracle.RefLayer.available():
        pytest.skip("oracle/_ref/libdsv4layer.so not built (reference tree absent at build time)")


def _device_layer(dev, ref, dims, ratio, max_pos):
    import torch
    import dsv4cu
    keep = []
    w = dsv4cu.AttnWeights()
    for name in oracle.RefLayer.MATS:
        got = ref.qmat(name)
        if got is None:
            continue
        m, wb, sb = got
        tw = torch.from_numpy(wb.copy()).cuda()
        ts = None if sb is None else torch.from_numpy(sb.copy()).cuda()
        keep += [tw, ts]
        setattr(w, name, dsv4cu.QMat(tw.data_ptr(), None if ts is None else ts.data_ptr(), m.wdt, m.rows, m.cols,
                                     m.blk_r, m.blk_c))
    for name in oracle.RefLayer.VECS:
        v = ref.vec(name)
        if v is None:
            continue
        t = torch.from_numpy(v.copy()).cuda()
        keep.append(t)
        setattr(w, name, t.data_ptr())
    c = dsv4cu.AttnCfg(*dims[:11], dims[11], 20, 1e-6, 1e-6, ratio, max_pos)
    return dev.attn_create(c, w), keep


@pytest.mark.parametrize("dims,ratio,steps", [
    (SMALL, 0, 24), (SMALL, 4, 48), (SMALL, 8, 40), (FLASH, 0, 4), (FLASH, 4, 12), (FLASH, 128, 6)],
    ids=["small-r0", "small-r4", "small-r8", "flash-r0", "flash-r4", "flash-r128"])
def test_attn_step_matches_reference(dev, need_layer_ref, dims, ratio, steps):
    import torch
    max_pos = max(64, steps + 8)
    ref = oracle.RefLayer(dims, ratio, max_pos, seed=ratio * 7 + dims[0])
    a, keep = _device_layer(dev, ref, dims, ratio, max_pos)
    rng = np.random.default_rng(dims[0] + ratio)
    out = torch.empty(dims[0], dtype=torch.float32, device="cuda")
    worst = 0.0
    for pos in range(steps):
        x = rng.standard_normal(dims[0]).astype(np.float32)
        want = ref.attention(x, pos)
        dev.attn_step(a, out, torch.from_numpy(x).cuda(), pos)
        got = out.cpu().numpy()
        dev.check_status()
        assert np.isfinite(got).all(), pos
        e = _rel(got, want)
        worst = max(worst, e)
        assert e <= TOL, (pos, e)
        assert dev.L.dsv4cu_attn_n_compressed(a) == ref.n_compressed(), pos
    print(f"attention {dims[0]}/{dims[1]}x{dims[2]} ratio {ratio}: {steps} tokens, worst rel {worst:.2e}, "
          f"{ref.n_compressed()} compressed rows")
    dev.attn_destroy(a)
    ref.close()


@pytest.mark.parametrize("dims,ratio,steps", [(SMALL, 4, 20), (FLASH, 4, 6)], ids=["small-r4", "flash-r4"])
def test_attn_block_matches_reference(dev, need_layer_ref, dims, ratio, steps):
    """mHC pre-mix, attn_norm, attention and the mHC update on h [hc][hidden]."""
    import torch
    max_pos = 64
    ref = oracle.RefLayer(dims, ratio, max_pos, seed=11 + ratio)
    a, keep = _device_layer(dev, ref, dims, ratio, max_pos)
    rng = np.random.default_rng(5)
    hc, d = dims[11], dims[0]
    for pos in range(steps):
        h = rng.standard_normal((hc, d)).astype(np.float32)
        want = ref.attn_block(h, pos)
        dh = torch.from_numpy(h).cuda()
        dev.attn_block(a, dh, pos)
        got = dh.cpu().numpy()
        dev.check_status()
        assert _rel(got, want) <= TOL, (pos, _rel(got, want))
    dev.attn_destroy(a)
    ref.close()


def test_attn_rejects_out_of_order_position(dev, need_layer_ref):
    import torch
    import dsv4cu
    ref = oracle.RefLayer(SMALL, 0, 64, seed=3)
    a, keep = _device_layer(dev, ref, SMALL, 0, 64)
    out = torch.empty(SMALL[0], dtype=torch.float32, device="cuda")
    x = torch.zeros(SMALL[0], dtype=torch.float32, device="cuda")
    with pytest.raises(dsv4cu.DSV4CUError):
        dev.attn_step(a, out, x, 3)
    dev.attn_destroy(a)
    ref.close()


def _device_ffn(dev, ref, dims, keep):
    """Upload the harness's FFN weights and build the device FFN half."""
    import torch
    import dsv4cu

    def up(e, m):
        q, wb, sb = ref.expert_qmat(e, m)
        tw = torch.from_numpy(wb.copy()).cuda()
        ts = None if sb is None else torch.from_numpy(sb.copy()).cuda()
        keep.extend([tw, ts])
        return dsv4cu.QMat(tw.data_ptr(), None if ts is None else ts.data_ptr(), q.wdt, q.rows, q.cols,
                           q.blk_r, q.blk_c)

    experts = [dsv4cu.Expert(up(e, 0), up(e, 1), up(e, 2)) for e in range(ref.n_experts)]
    shared = dsv4cu.Expert(up(ref.n_experts, 0), up(ref.n_experts, 1), up(ref.n_experts, 2))
    moe = dev.moe_create(experts, shared, dims[0], ref.inter)
    vec = {}
    for name in ("bias", "ffn_norm", "hc_fn", "hc_base", "hc_scale"):
        v = ref.ffn_vec(name)
        vec[name] = None if v is None else torch.from_numpy(v.copy()).cuda()
        keep.append(vec[name])
    d = dsv4cu.FfnDesc()
    d.moe = moe
    d.gate = up(-1, 0)
    d.bias = None if vec["bias"] is None else vec["bias"].data_ptr()
    d.tid2eid = None
    d.ffn_norm, d.hc_fn = vec["ffn_norm"].data_ptr(), vec["hc_fn"].data_ptr()
    d.hc_base, d.hc_scale = vec["hc_base"].data_ptr(), vec["hc_scale"].data_ptr()
    d.hidden, d.hc_mult, d.hc_sinkhorn_iters, d.n_experts, d.topk = dims[0], dims[11], 20, ref.n_experts, ref.topk
    d.nt_max = 8
    d.rms_eps, d.hc_eps, d.route_scale, d.swiglu_limit = 1e-6, 1e-6, 1.5, 10.0
    return dev.ffn_create(d), moe


@pytest.mark.parametrize("dims,ratio,experts,inter,topk,steps", [
    (SMALL, 4, 16, 256, 4, 12), (FLASH, 4, 32, 2048, 6, 6), (FLASH, 128, 32, 2048, 6, 4)],
    ids=["small-r4", "flash-r4", "flash-r128"])
def test_layer_step_matches_reference(dev, need_layer_ref, dims, ratio, experts, inter, topk, steps):
    """The whole decoder layer (dsv4_layer_forward: attention half, then the
    FFN half with the reference's dsv4_layer_moe) token after token: the
    residual streams h [hc][hidden] after every layer step."""
    import torch
    ref = oracle.RefLayer(dims, ratio, 64, seed=21 + ratio)
    ref.ffn_create(experts, topk, inter, 1.5, 10.0, True, 22)
    a, keep = _device_layer(dev, ref, dims, ratio, 64)
    f, moe = _device_ffn(dev, ref, dims, keep)
    rng = np.random.default_rng(9)
    hc, d = dims[11], dims[0]
    worst = 0.0
    for pos in range(steps):
        h = rng.standard_normal((hc, d)).astype(np.float32)
        want = ref.layer(h, pos)
        dh = torch.from_numpy(h).cuda()
        dev.layer_step(a, f, dh, pos)
        got = dh.cpu().numpy()
        dev.check_status()
        e = _rel(got, want)
        worst = max(worst, e)
        assert e <= TOL, (pos, e)
    print(f"layer {dims[0]} ratio {ratio}, {experts} experts top-{topk}: {steps} tokens, worst rel {worst:.2e}")
    dev.ffn_destroy(f)
    dev.moe_destroy(moe)
    dev.attn_destroy(a)
    ref.close()
