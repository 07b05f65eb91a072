"""Expert-parallel MoE host logic on CPU ranks (gloo), world 2 and 4.

ExpertParallelMoE (deepseek-v4-in-c_b200/ep.py) runs its real exchange -
counts all-to-all, rows all-to-all, reverse all-to-all - with a CPU ops
object whose per-row expert math is the oracle's dsv4_expert_forward
restatement. Each rank's output for its own tokens must be the same bits as
the single-process layer: routing, then the k-order combine of the routed
experts plus the shared expert (src/70_decode/dsv4_layer.c:48-117). A wrong
split, permutation or id mapping shows up as a mismatch.
"""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "deepseek-v4-in-c_b200")
ORACLE = os.path.join(ROOT, "oracle")

N_EXPERTS, HIDDEN, INTER, TOPK, NT = 8, 256, 128, 3, 6
ROUTE_SCALE, LIMIT = 1.5, 10.0


def _paths():
    for p in (PKG, ORACLE):
        if p not in sys.path:
            sys.path.insert(0, p)


def _layer(seed=11):
    """Routed FP4 experts + an FP8 shared expert, in the reference pack layout."""
    _paths()
    import oracle
    import pack
    rng = np.random.default_rng(seed)
    keep, experts = [], []
    for _ in range(N_EXPERTS):
        mats = []
        for rows, cols in ((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER)):
            W, S = pack.quantize_fp4((rng.standard_normal((rows, cols)) * 0.05).astype(np.float32))
            keep += [W, S]
            mats.append(oracle.qmat(W, S, 3, rows, cols, 1, 32))
        experts.append(mats)
    shared = []
    for rows, cols in ((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER)):
        W, S = pack.quantize_fp8((rng.standard_normal((rows, cols)) * 0.05).astype(np.float32))
        keep += [W, S]
        shared.append(oracle.qmat(W, S, 2, rows, cols, 128, 128))
    return experts, shared, keep


def _tokens(world, seed=12):
    _paths()
    import pack
    rng = np.random.default_rng(seed)
    x = pack.bf16_round(rng.standard_normal((world * NT, HIDDEN)).astype(np.float32))
    lg = pack.bf16_round(rng.standard_normal((world * NT, N_EXPERTS)).astype(np.float32))
    return x, lg


class CpuOps:
    """The DeviceOps interface on CPU torch tensors, computed by the oracle."""

    def __init__(self, orc, experts, shared, epr, rank, n_ranks):
        import torch
        self.torch, self.orc = torch, orc
        self.local = experts[rank * epr:(rank + 1) * epr]
        self.shared, self.epr, self.n_ranks = shared, epr, n_ranks

    def empty(self, shape, dtype="float32"):
        return self.torch.zeros(shape, dtype=getattr(self.torch, dtype))

    def route(self, logits):
        lg = logits.numpy()
        idx = np.zeros((lg.shape[0], TOPK), np.int32)
        wts = np.zeros((lg.shape[0], TOPK), np.float32)
        for t in range(lg.shape[0]):
            i, w, _, _ = self.orc.route(lg[t], TOPK, ROUTE_SCALE, None, None, 0)
            idx[t], wts[t] = i, w
        return self.torch.from_numpy(idx), self.torch.from_numpy(wts)

    def pack(self, x, idx):
        nt = x.shape[0]
        pairs = idx.numpy().reshape(-1)
        owner = pairs // self.epr
        order = np.argsort(owner, kind="stable")              # grouped by owner, pair order inside
        send = np.zeros((nt * TOPK, HIDDEN + 4), np.float32)
        pair_slot = np.zeros(nt * TOPK, np.int32)
        for r, p in enumerate(order):
            send[r, :HIDDEN] = x.numpy()[p // TOPK]
            send[r, HIDDEN] = pairs[p] % self.epr
            pair_slot[p] = r
        counts = np.bincount(owner, minlength=self.n_ranks).astype(np.int32)
        return self.torch.from_numpy(send), self.torch.from_numpy(counts), self.torch.from_numpy(pair_slot)

    def tail(self, recv, nrecv, x):
        nt = x.shape[0]
        recv[nrecv:, :HIDDEN] = x
        ids = np.empty(nrecv + nt, np.int32)
        ids[:nrecv] = recv[:nrecv, HIDDEN].numpy().astype(np.int32)
        ids[nrecv:] = self.epr
        return self.torch.from_numpy(ids)

    def rows(self, recv, ids, nrows):
        y = np.zeros((nrows, HIDDEN), np.float32)
        rv = recv.numpy()
        for r in range(nrows):
            e = int(ids[r])
            mats = self.shared if e == self.epr else self.local[e]
            y[r] = self.orc.expert_forward(np.ascontiguousarray(rv[r, :HIDDEN]), mats, INTER, LIMIT)
        return self.torch.from_numpy(y)

    def combine(self, back, pair_slot, wts, shared_y, nt):
        b, ps, w, sh = back.numpy(), pair_slot.numpy(), wts.numpy(), shared_y.numpy()
        out = np.zeros((nt, HIDDEN), np.float32)
        for t in range(nt):
            o = np.zeros(HIDDEN, np.float32)
            for k in range(TOPK):
                o = o + np.float32(w[t, k]) * b[ps[t * TOPK + k]]
            out[t] = o + sh[t]
        return self.torch.from_numpy(out)


def reference_layer(orc, experts, shared, x, lg):
    out = np.zeros((x.shape[0], HIDDEN), np.float32)
    for t in range(x.shape[0]):
        idx, w, _, _ = orc.route(lg[t], TOPK, ROUTE_SCALE, None, None, 0)
        o = np.zeros(HIDDEN, np.float32)
        for k in range(TOPK):
            o = o + np.float32(w[k]) * orc.expert_forward(x[t], experts[idx[k]], INTER, LIMIT)
        out[t] = o + orc.expert_forward(x[t], shared, INTER, LIMIT)
    return out


def _rank_main(rank, world, port, q):
    try:
        import datetime
        import torch
        import torch.distributed as dist
        _paths()
        import oracle
        from ep import ExpertParallelMoE
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        orc = oracle.Oracle()
        experts, shared, keep = _layer()
        x, lg = _tokens(world)
        mine = slice(rank * NT, (rank + 1) * NT)
        ops = CpuOps(orc, experts, shared, N_EXPERTS // world, rank, world)
        out, idx, wts = ExpertParallelMoE(ops, rank, world).forward(torch.from_numpy(x[mine]),
                                                                   torch.from_numpy(lg[mine]))
        want = reference_layer(orc, experts, shared, x[mine], lg[mine])
        ok = np.array_equal(out.numpy().view(np.uint32), want.view(np.uint32))
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:      # reported to the parent
        q.put((rank, False, repr(e)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_ep_exchange_matches_single_process(world):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in sorted(res):
        assert ok, f"rank {rank}: {err or 'output differs from the single-process layer'}"


def test_ep_world1_without_collectives():
    """world 1: the same steps with no process group at all."""
    import torch
    _paths()
    import oracle
    from ep import ExpertParallelMoE
    orc = oracle.Oracle()
    experts, shared, keep = _layer()
    x, lg = _tokens(1)
    out, _, _ = ExpertParallelMoE(CpuOps(orc, experts, shared, N_EXPERTS, 0, 1), 0, 1).forward(
        torch.from_numpy(x), torch.from_numpy(lg))
    want = reference_layer(orc, experts, shared, x, lg)
    assert np.array_equal(out.numpy().view(np.uint32), want.view(np.uint32))


# ---- failure paths (host side, gloo): a peer that fails or never arrives
# ends the other ranks' step with an error within the process-group timeout.

class _FailingOps(CpuOps):
    """Raises on one rank after routing, before the exchange."""

    def __init__(self, *a, fail_rank=1, **kw):
        super().__init__(*a, **kw)
        self.fail_rank, self.rank = fail_rank, a[4]

    def pack(self, x, idx):
        if self.rank == self.fail_rank:
            raise RuntimeError("injected failure before the exchange")
        return super().pack(x, idx)


class _BadCountsOps(CpuOps):
    """Claims one row more for rank 0 than it sends (a corrupt count exchange)."""

    def pack(self, x, idx):
        send, counts, pair_slot = super().pack(x, idx)
        counts = counts.clone()
        counts[0] += 1
        return send, counts, pair_slot


def _failure_rank(rank, world, port, q, mode):
    try:
        import datetime
        import torch
        import torch.distributed as dist
        _paths()
        import oracle
        from ep import ExpertParallelMoE
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=8))
        if mode == "absent" and rank == world - 1:
            q.put((rank, "left"))
            return                          # joins, then never takes part in the step
        orc = oracle.Oracle()
        experts, shared, keep = _layer()
        x, lg = _tokens(world)
        mine = slice(rank * NT, (rank + 1) * NT)
        cls = {"raise": _FailingOps, "absent": CpuOps, "counts": _BadCountsOps}[mode]
        ops = cls(orc, experts, shared, N_EXPERTS // world, rank, world)
        try:
            ExpertParallelMoE(ops, rank, world).forward(torch.from_numpy(x[mine]), torch.from_numpy(lg[mine]))
            q.put((rank, "completed"))
        except Exception as e:      # the outcome under test
            q.put((rank, "error:" + type(e).__name__))
    except Exception as e:
        q.put((rank, "setup:" + repr(e)))


@pytest.mark.parametrize("mode", ["raise", "absent", "counts"])
def test_ep_failures_end_with_an_error(mode):
    """No rank hangs: the failing / absent rank's peers get an exception from
    the exchange (gloo timeout 8 s, or a size mismatch), well inside the
    test's bound."""
    import multiprocessing as mp
    import time
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failure_rank, args=(r, world, port, q, mode)) for r in range(world)]
    t0 = time.time()
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert time.time() - t0 < 120
    if mode == "raise":
        assert res[1].startswith("error"), res
        assert res[0].startswith("error"), res          # the peer's exchange times out
    elif mode == "absent":
        assert res[1] == "left" and res[0].startswith("error"), res
    else:
        assert any(v.startswith("error") for v in res.values()), res
