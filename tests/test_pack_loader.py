"""Routed experts from the reference's pack into HBM (dsv4cu_experts_load).

CPU: the index reader against a synthetic pack (tests/packfix.py) - records,
shard numbering in name order, malformed and mismatched packs. GPU: experts
loaded from the pack run through dsv4cu_moe_rows and match the oracle's
dsv4_expert_forward (src/10_compute/dsv4_ops.c:85-93) on the same bytes.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import dsv4cu
import oracle
import pack
import packfix

H, I = 256, 256


def test_index_records_and_shard_order(tmp_path):
    tensors, paths = packfix.write_pack(str(tmp_path), 2, 5, H, I, seed=1)
    nl, ne, recs = dsv4cu.experts_index(str(tmp_path), 1, 3)
    assert (nl, ne) == (2, 5)
    blobs = [open(p, "rb").read() for p in paths]
    for t, (shard, off, nbytes) in enumerate(recs):
        assert blobs[shard][off:off + nbytes] == tensors[(1, 3)][t].tobytes()


def test_index_rejects_bad_files(tmp_path):
    packfix.write_pack(str(tmp_path), 1, 2, H, I)
    idx = os.path.join(str(tmp_path), "experts.idx")
    good = open(idx, "rb").read()
    open(idx, "wb").write(b"DSV4EXP2" + good[8:])
    with pytest.raises(dsv4cu.DSV4CUError, match="DSV4EXP1"):
        dsv4cu.experts_index(str(tmp_path))
    open(idx, "wb").write(good[:-10])
    with pytest.raises(dsv4cu.DSV4CUError, match="truncated"):
        dsv4cu.experts_index(str(tmp_path))
    with pytest.raises(dsv4cu.DSV4CUError, match="cannot open"):
        dsv4cu.experts_index(str(tmp_path / "missing"))
    open(idx, "wb").write(good)
    with pytest.raises(dsv4cu.DSV4CUError, match="out of range"):
        dsv4cu.experts_index(str(tmp_path), 1, 0)


def test_load_rejects_mismatched_sizes_before_touching_the_device(tmp_path):
    """inter 512 against a pack of inter 256: every record is checked first."""
    import ctypes as C
    packfix.write_pack(str(tmp_path), 1, 2, H, I)
    L = dsv4cu.lib()
    h = C.c_void_p()
    arr = (dsv4cu.Expert * 2)()
    rc = L.dsv4cu_experts_load(C.byref(h), arr, str(tmp_path).encode(), str(tmp_path).encode(), 0, 0, 2, H, 512,
                               None)
    assert rc == -7 and "want" in dsv4cu.last_error()
    rc = L.dsv4cu_experts_load(C.byref(h), arr, str(tmp_path).encode(), str(tmp_path).encode(), 0, 1, 2, H, I, None)
    assert rc == -1 and "outside the index" in dsv4cu.last_error()


@pytest.mark.gpu
def test_loaded_experts_run_through_moe_rows(tmp_path, dev, orc):
    import torch
    tensors, _ = packfix.write_pack(str(tmp_path), 2, 6, H, I, seed=3)
    store, experts = dev.experts_load(str(tmp_path), str(tmp_path), 1, 2, 3, H, I)   # experts 2, 3, 4 of layer 1
    layer = dev.moe_create(experts, None, H, I)
    rng = np.random.default_rng(5)
    n = 24
    x = pack.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    ids = rng.integers(0, 3, n).astype(np.int32)
    y = torch.empty((n, H), dtype=torch.float32, device="cuda")
    dev.moe_rows(layer, y, torch.from_numpy(x).cuda(), H, torch.from_numpy(ids).cuda(), n, 10.0)
    dev.check_status()
    got = y.cpu().numpy()
    for r in range(n):
        w1, s1, w2, s2, w3, s3 = tensors[(1, 2 + int(ids[r]))]
        mats = [oracle.qmat(w1, s1, 3, I, H, 1, 32), oracle.qmat(w3, s3, 3, I, H, 1, 32),
                oracle.qmat(w2, s2, 3, H, I, 1, 32)]
        want = orc.expert_forward(x[r], mats, I, 10.0).astype(np.float64)
        err = float(np.abs(got[r] - want).max()) / max(float(np.abs(want).max()), 1e-30)
        assert err <= 1e-5, (r, err)
    dev.moe_destroy(layer)
    dev.experts_free(store)
