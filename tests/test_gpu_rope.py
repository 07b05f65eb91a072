"""dsv4cu_rope_apply against the oracle's dsv4_rope_apply (src/10_compute/dsv4_rope.c),
bit for bit: several tokens and heads with per-token positions, both directions,
and a position outside the table (status set, heads left unchanged)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _tables(rng, npos, half):
    cs = rng.uniform(-1, 1, (npos, half)).astype(np.float32)
    sn = rng.uniform(-1, 1, (npos, half)).astype(np.float32)
    return cs, sn


@pytest.mark.parametrize("head_dim,rd", [(576, 64), (128, 64), (64, 64)])
@pytest.mark.parametrize("inverse", [0, 1])
def test_rope_bitwise(dev, orc, head_dim, rd, inverse):
    import torch
    rng = np.random.default_rng(head_dim + rd + inverse)
    nt, nh, npos = 5, 8, 300
    cs, sn = _tables(rng, npos, 32)
    v = rng.standard_normal((nt, nh, head_dim)).astype(np.float32)
    pos = rng.integers(0, npos, nt).astype(np.int32)
    dv = torch.from_numpy(v.copy()).cuda()
    dev.rope_apply(dv, nt, nh, head_dim, rd, torch.from_numpy(cs).cuda(), torch.from_numpy(sn).cuda(),
                   torch.from_numpy(pos).cuda(), inverse)
    dev.check_status()
    got = dv.cpu().numpy()
    for t in range(nt):
        for h in range(nh):
            want = orc.rope_apply(v[t, h], rd, cs, sn, int(pos[t]), inverse)
            assert np.array_equal(got[t, h].view(np.uint32), want.view(np.uint32)), (t, h)


def test_rope_bad_position_sets_status(dev):
    import torch
    import dsv4cu
    rng = np.random.default_rng(1)
    cs, sn = _tables(rng, 10, 32)
    v = rng.standard_normal((2, 2, 64)).astype(np.float32)
    dv = torch.from_numpy(v.copy()).cuda()
    pos = torch.tensor([3, 10], dtype=torch.int32, device="cuda")
    dev.rope_apply(dv, 2, 2, 64, 64, torch.from_numpy(cs).cuda(), torch.from_numpy(sn).cuda(), pos)
    with pytest.raises(dsv4cu.DSV4CUError):
        dev.check_status()
    assert np.array_equal(dv.cpu().numpy()[1], v[1])
    dev.check_status()
