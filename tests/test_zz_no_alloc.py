"""dsv4cu_sparse_attn_noalloc: the allocation-free sparse attention entry point.

Called through the C-ABI with ctypes and compared with dsv4cu_sparse_attn on
the same inputs, twice in a row with different shapes, so a stale scratch
array from the first call would show in the second. The file name sorts last
so that it also runs after every other GPU test.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import pack

ATT_TOL = 1e-5


def _lib():
    import dsv4cu
    L = dsv4cu.lib()
    f = L.dsv4cu_sparse_attn_noalloc
    vp = C.c_void_p
    f.argtypes = [vp, vp, vp, C.c_int, vp, vp, C.c_int, C.c_int, C.c_int, C.c_float, vp]
    f.restype = C.c_int
    return L


def _case(rng, H, D, N, T, n_valid):
    kv = pack.bf16_round(rng.standard_normal((N, D)).astype(np.float32))
    q = pack.bf16_round(rng.standard_normal((H, D)).astype(np.float32))
    sink = rng.standard_normal(H).astype(np.float32)
    idx = rng.choice(N, T, replace=False).astype(np.int32)
    idx[n_valid:] = -1
    return q, kv, sink, idx


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice(dev, orc):
    t = __import__("torch")
    L = _lib()
    rng = np.random.default_rng(77)
    # config 4 shape (64 heads, d = 576 = 512 latent + 64 rope, 2048 + 128 slots), then a smaller one
    for (H, D, N, T, n_valid, bf16) in [(64, 576, 32768, 2176, 2148, 1), (16, 512, 4096, 300, 257, 0)]:
        q, kv, sink, idx = _case(rng, H, D, N, T, n_valid)
        scale = float(np.float32(1 / np.sqrt(D)))
        qd = t.from_numpy(q).cuda()
        kvd = t.from_numpy(kv).cuda()
        if bf16:
            kvd = kvd.to(t.bfloat16)
        sd, idd = t.from_numpy(sink).cuda(), t.from_numpy(idx).cuda()
        o_ws = t.empty((H, D), dtype=t.float32, device="cuda")
        o_na = t.full((H, D), float("nan"), dtype=t.float32, device="cuda")
        dev.sparse_attn(o_ws, qd, kvd, bf16, sd, idd, H, D, T, scale)
        r = L.dsv4cu_sparse_attn_noalloc(o_na.data_ptr(), qd.data_ptr(), kvd.data_ptr(), bf16, sd.data_ptr(),
                                         idd.data_ptr(), H, D, T, scale, dev.stream())
        assert r == 0, L.dsv4cu_last_error()
        t.cuda.synchronize()
        a, b = o_na.cpu().numpy(), o_ws.cpu().numpy()
        assert np.isfinite(a).all()
        # the same kernels on the same inputs: the same bits
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert _rel(a, orc.sparse_attn(q, kv, sink, idx, np.float32(scale))) <= ATT_TOL
        # the entry point's purpose: inside a stream capture (nothing allocated), replayed
        o_g = t.full((H, D), float("nan"), dtype=t.float32, device="cuda")
        g = t.cuda.CUDAGraph()
        with t.cuda.graph(g):
            r = L.dsv4cu_sparse_attn_noalloc(o_g.data_ptr(), qd.data_ptr(), kvd.data_ptr(), bf16, sd.data_ptr(),
                                             idd.data_ptr(), H, D, T, scale, dev.stream())
        assert r == 0, L.dsv4cu_last_error()
        for _ in range(2):
            o_g.fill_(float("nan"))
            g.replay()
            t.cuda.synchronize()
            assert np.array_equal(o_g.cpu().numpy().view(np.uint32), b.view(np.uint32))
        del g


@pytest.mark.gpu
def test_noalloc_rejects_oversize_shapes(dev):
    t = __import__("torch")
    L = _lib()
    H, D, T = 128, 1024, 4096           # partials need 128 * 1026 * 128 * 4 B > 12 MiB
    o = t.zeros((H, D), dtype=t.float32, device="cuda")
    q = t.zeros((H, D), dtype=t.float32, device="cuda")
    kv = t.zeros((8, D), dtype=t.float32, device="cuda")
    sink = t.zeros(H, dtype=t.float32, device="cuda")
    idx = t.zeros(T, dtype=t.int32, device="cuda")
    r = L.dsv4cu_sparse_attn_noalloc(o.data_ptr(), q.data_ptr(), kv.data_ptr(), 0, sink.data_ptr(),
                                     idx.data_ptr(), H, D, T, 0.03, dev.stream())
    assert r == -2                      # DSV4CU_ERR_UNSUPPORTED, nothing launched
    assert b"limit" in L.dsv4cu_last_error()
