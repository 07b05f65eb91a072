"""Expert-parallel MoE on the GPU: the per-row expert entry (dsv4cu_moe_rows)
against the oracle, the EP layer at world 1 against the single-device decode
layer, the peer-memory step (dsv4cu_ep_forward) against the NCCL-exchange
layer bitwise, and (with 2 or more GPUs) both exchanges at world N against
world 1, bitwise."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

import pack
from test_gpu_moe import MoeFixture, rel_err

pytestmark = pytest.mark.gpu

H, I, E = 512, 256, 16


def _device_ops(dev, layer, n_experts, epr, n_ranks, topk):
    from ep import DeviceOps
    return DeviceOps(dev, layer, n_experts, epr, n_ranks, H, topk, 1.5, 10.0)


def test_moe_rows_vs_oracle(dev, orc):
    """Rows with mixed expert ids, the shared expert (id E) among them."""
    t = __import__("torch")
    fx = MoeFixture(dev, E, H, I, shared_fmt=2, seed=41)
    rng = np.random.default_rng(41)
    n = 300
    x = pack.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    ids = rng.integers(0, E + 1, n).astype(np.int32)
    y = t.empty((n, H), dtype=t.float32, device="cuda")
    dev.moe_rows(fx.layer, y, t.from_numpy(x).cuda(), H, t.from_numpy(ids).cuda(), n, 10.0)
    dev.check_status()
    got = y.cpu().numpy()
    cache = {}
    worst = 0.0
    for r in rng.choice(n, 40, replace=False):
        e = int(ids[r])
        if e not in cache:
            cache[e] = fx.host_expert(fx.shared if e == E else fx.experts_host[e])
        want = orc.expert_forward(x[r], cache[e][0], I, 10.0)
        worst = max(worst, rel_err(got[r], want.astype(np.float64)))
    print(f"moe_rows max-rel={worst:.3e}")
    assert worst <= 1e-5
    fx.close()


def test_moe_rows_bad_id_sets_status(dev):
    import dsv4cu
    t = __import__("torch")
    fx = MoeFixture(dev, E, H, I, shared_fmt=2, seed=42)
    ids = t.tensor([0, E + 5, 3], dtype=t.int32, device="cuda")
    y = t.full((3, H), 7.0, dtype=t.float32, device="cuda")
    x = t.ones((3, H), dtype=t.float32, device="cuda")
    dev.moe_rows(fx.layer, y, x, H, ids, 3, 10.0)
    with pytest.raises(dsv4cu.DSV4CUError):
        dev.check_status()
    assert float(y[1].abs().max()) == 0.0
    dev.check_status()          # the status was cleared by the read
    fx.close()


def test_ep_world1_matches_decode(dev):
    """All experts local: route, pack, rows, combine against the decode layer."""
    t = __import__("torch")
    from ep import ExpertParallelMoE
    from test_gpu_moe import run
    fx = MoeFixture(dev, E, H, I, shared_fmt=2, seed=43)
    rng = np.random.default_rng(43)
    nt, topk = 40, 4
    x = pack.bf16_round(rng.standard_normal((nt, H)).astype(np.float32))
    lg = pack.bf16_round(rng.standard_normal((nt, E)).astype(np.float32))
    out, idx, wts = ExpertParallelMoE(_device_ops(dev, fx.layer, E, E, 1, topk), 0, 1).forward(
        t.from_numpy(x).cuda(), t.from_numpy(lg).cuda())
    dev.check_status()
    outd, idxd, wtsd = run(dev, fx, x, lg, topk, 1.5, 10.0)
    assert np.array_equal(idx.cpu().numpy(), idxd)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), wtsd.view(np.uint32))
    got = out.cpu().numpy()
    bitwise = np.array_equal(got.view(np.uint32), outd.view(np.uint32))
    worst = max(rel_err(got[i], outd[i].astype(np.float64)) for i in range(nt))
    print(f"ep world1 vs decode: bitwise={bitwise} max-rel={worst:.3e}")
    assert worst <= 1e-5
    fx.close()


def test_ep_peer_world1_matches_exchange_layer(dev):
    """dsv4cu_ep_forward at world 1: the same bits as the all-to-all layer over
    dsv4cu_moe_rows, over several steps (epochs), with skipped capacity rows,
    any nt up to nt_max, and routing outputs equal to the decode layer's."""
    t = __import__("torch")
    from ep import ExpertParallelMoE, PeerExpertParallel
    from test_gpu_moe import run
    fx = MoeFixture(dev, E, H, I, shared_fmt=2, seed=45)
    topk, nt_max = 4, 48
    pe = PeerExpertParallel(dev, fx.layer, 0, 1, nt_max, H, topk, E, 1.5, 10.0, lambda b: [b])
    rng = np.random.default_rng(45)
    for step, nt in enumerate((48, 5, 1, 48, 17)):
        x = pack.bf16_round(rng.standard_normal((nt, H)).astype(np.float32))
        lg = pack.bf16_round(rng.standard_normal((nt, E)).astype(np.float32))
        dx, dl = t.from_numpy(x).cuda(), t.from_numpy(lg).cuda()
        idx = t.empty((nt, topk), dtype=t.int32, device="cuda")
        wts = t.empty((nt, topk), dtype=t.float32, device="cuda")
        got = pe.forward(dx, dl, idx=idx, wts=wts).cpu().numpy()
        ref, ridx, rwts = ExpertParallelMoE(_device_ops(dev, fx.layer, E, E, 1, topk), 0, 1).forward(dx, dl)
        dev.check_status()
        assert np.array_equal(idx.cpu().numpy(), ridx.cpu().numpy()), step
        assert np.array_equal(wts.cpu().numpy().view(np.uint32), rwts.cpu().numpy().view(np.uint32)), step
        assert np.array_equal(got.view(np.uint32), ref.cpu().numpy().view(np.uint32)), step
        outd, _, _ = run(dev, fx, x, lg, topk, 1.5, 10.0)
        assert max(rel_err(got[i], outd[i].astype(np.float64)) for i in range(nt)) <= 1e-5
    with pytest.raises(Exception):
        pe.forward(t.zeros((nt_max + 1, H), device="cuda"), t.zeros((nt_max + 1, E), device="cuda"))
    pe.close()
    fx.close()


def test_ep_peer_rejects_mismatched_handles(dev):
    import dsv4cu
    a = dev.ep_create(0, 1, 8, H, 4, E)
    b = dev.ep_create(0, 1, 16, H, 4, E)
    with pytest.raises(dsv4cu.DSV4CUError):
        dev.ep_connect(a, [dev.ep_handle(b)])
    dev.ep_destroy(a)
    dev.ep_destroy(b)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_rank(rank, world, port, q):
    try:
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [os.path.join(root, "deepseek-v4-in-c_b200"), os.path.join(root, "tests"),
                        os.path.join(root, "oracle")]
        import datetime
        import torch
        import torch.distributed as dist
        import dsv4cu
        from ep import ExpertParallelMoE
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        dev = dsv4cu.Device(rank)
        fx = MoeFixture(dev, E, H, I, shared_fmt=2, seed=44)
        epr = E // world
        local = dev.moe_create([d[0] for d in fx.experts_host[rank * epr:(rank + 1) * epr]], fx.shared[0], H, I)
        rng = np.random.default_rng(44)
        nt, topk = 24, 4
        x = pack.bf16_round(rng.standard_normal((world * nt, H)).astype(np.float32))[rank * nt:(rank + 1) * nt]
        lg = pack.bf16_round(rng.standard_normal((world * nt, E)).astype(np.float32))[rank * nt:(rank + 1) * nt]
        dx, dl = torch.from_numpy(x).cuda(), torch.from_numpy(lg).cuda()
        out, _, _ = ExpertParallelMoE(_device_ops(dev, local, E, epr, world, topk), rank, world).forward(dx, dl)
        ref, _, _ = ExpertParallelMoE(_device_ops(dev, fx.layer, E, E, 1, topk), 0, 1).forward(dx, dl)
        from ep import PeerExpertParallel, torch_allgather
        pe = PeerExpertParallel(dev, local, rank, world, nt, H, topk, epr, 1.5, 10.0, torch_allgather())
        peer = [pe.forward(dx, dl).cpu().numpy() for _ in range(3)]
        dev.check_status()
        ok = np.array_equal(out.cpu().numpy().view(np.uint32), ref.cpu().numpy().view(np.uint32))
        ok = ok and all(np.array_equal(p.view(np.uint32), ref.cpu().numpy().view(np.uint32)) for p in peer)
        dist.barrier()
        pe.close()
        dist.barrier()
        dist.destroy_process_group()
        dev.moe_destroy(local)
        fx.close()
        q.put((rank, ok, ""))
    except Exception as e:      # reported to the parent
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_nccl_and_peer_match_world1(world):
    t = __import__("torch")
    if t.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in sorted(res):
        assert ok, f"rank {rank}: {err or 'EP output differs from world 1'}"
