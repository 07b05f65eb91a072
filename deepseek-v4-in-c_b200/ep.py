"""Expert-parallel MoE layer: one process per GPU.

PeerExpertParallel is the product path: one call of the library's
dsv4cu_ep_forward per step, the rows crossing NVLink as peer stores inside
the library's kernels (include/dsv4cu.h, csrc/ep_p2p.cu), nothing
synchronised with the host. Python only all-gathers the ranks' handles once.

ExpertParallelMoE below is the same layer with the exchange done by
torch.distributed all-to-all (NCCL, or gloo in the CPU tests); it keeps the
host-side logic testable without GPUs and serves as the NCCL comparison.

The reference keeps every expert of a layer reachable from one process and
streams them through a disk cache (src/60_cache); here the 256 experts of a
layer are HBM-resident and partitioned over the ranks: expert e lives on
rank e // experts_per_rank. Every rank is the home of its own tokens. One call:

  1. route      the home rank routes its tokens (dsv4cu_route = dsv4_route,
                src/10_compute/dsv4_ops.c:117-156): idx, wts [nt][topk];
  2. pack       every (token, slot) pair becomes a send row for the expert's
                owner, rows grouped by owner in pair order (dsv4cu_ep_pack);
  3. exchange   all-to-all of the per-rank row counts, then of the rows;
  4. compute    the owner runs every received row through its expert, and
                its own tokens through the replicated shared expert, in one
                grouped tensor-core launch sequence (dsv4cu_moe_rows);
  5. return     reverse all-to-all of the result rows;
  6. combine    out[t] = sum over k in order of wts[t][k] * y(t, k) + shared(t)
                (dsv4_layer_moe's order, src/70_decode/dsv4_layer.c:109-116;
                dsv4cu_ep_combine).

Every per-row result and the combine are the same float operations as on one
device, so the output does not depend on the number of ranks.

The exchange and bookkeeping live in ExpertParallelMoE; the device work goes
through an ops object (DeviceOps here), so the same host logic runs in the
CPU tests with a CPU implementation of the ops.
"""
from __future__ import annotations


class DeviceOps:
    """The layer's device work on one GPU through the CUDA library.

    layer: a dsv4cu_moe handle holding this rank's experts (local ids
    0 .. experts_per_rank - 1) and the shared expert (local id
    experts_per_rank)."""

    def __init__(self, dev, layer, n_experts: int, experts_per_rank: int, n_ranks: int, hidden: int, topk: int,
                 route_scale: float, limit: float, bias=None):
        import torch
        self.torch = torch
        self.dev, self.layer = dev, layer
        self.n_experts, self.epr, self.n_ranks = n_experts, experts_per_rank, n_ranks
        self.hidden, self.topk = hidden, topk
        self.route_scale, self.limit, self.bias = route_scale, limit, bias

    def empty(self, shape, dtype="float32"):
        return self.torch.empty(shape, dtype=getattr(self.torch, dtype), device="cuda")

    def route(self, logits):
        nt = logits.shape[0]
        idx = self.empty((nt, self.topk), "int32")
        wts = self.empty((nt, self.topk))
        self.dev.route(idx, wts, None, None, logits, self.topk, self.route_scale, nt, self.bias)
        return idx, wts

    def pack(self, x, idx):
        nt = x.shape[0]
        send = self.empty((nt * self.topk, self.hidden + 4))
        counts = self.empty((self.n_ranks,), "int32")
        pair_slot = self.empty((nt * self.topk,), "int32")
        self.dev.ep_pack(send, counts, pair_slot, x, idx, nt, self.topk, self.hidden, self.epr, self.n_ranks)
        return send, counts, pair_slot

    def tail(self, recv, nrecv, x):
        nt = x.shape[0]
        ids = self.empty((nrecv + nt,), "int32")
        self.dev.ep_tail(recv, nrecv, x, nt, self.hidden, self.epr, ids)
        return ids

    def rows(self, recv, ids, nrows):
        y = self.empty((nrows, self.hidden))
        self.dev.moe_rows(self.layer, y, recv, self.hidden + 4, ids, nrows, self.limit)
        return y

    def combine(self, back, pair_slot, wts, shared_y, nt):
        out = self.empty((nt, self.hidden))
        self.dev.ep_combine(out, back, pair_slot, wts, shared_y, nt, self.topk, self.hidden)
        return out


class ExpertParallelMoE:
    """The exchange around the ops; world == 1 runs the same steps without
    collectives. group: the torch.distributed group (None = default)."""

    def __init__(self, ops, rank: int, world: int, group=None):
        self.ops, self.rank, self.world, self.group = ops, rank, world, group

    def forward(self, x, logits):
        import torch
        ops = self.ops
        nt, hidden = x.shape[0], x.shape[1]
        idx, wts = ops.route(logits)
        send, counts, pair_slot = ops.pack(x, idx)
        if self.world > 1:
            import torch.distributed as dist
            rcounts = torch.empty_like(counts)
            dist.all_to_all_single(rcounts, counts, group=self.group)
            sc, rc = counts.tolist(), rcounts.tolist()
        else:
            sc = rc = counts.tolist()
        nsend, nrecv = sum(sc), sum(rc)
        recv = ops.empty((nrecv + nt, hidden + 4))
        if self.world > 1:
            dist.all_to_all_single(recv[:nrecv], send[:nsend], rc, sc, group=self.group)
        else:
            recv[:nrecv].copy_(send[:nsend])
        ids = ops.tail(recv, nrecv, x)
        y = ops.rows(recv, ids, nrecv + nt)
        if self.world > 1:
            back = ops.empty((nsend, hidden))
            dist.all_to_all_single(back, y[:nrecv], sc, rc, group=self.group)
        else:
            back = y[:nrecv]
        return ops.combine(back, pair_slot, wts, y[nrecv:], nt), idx, wts


def torch_allgather(group=None):
    """allgather(bytes) -> list of every rank's bytes in rank order, over torch.distributed."""
    def gather(blob: bytes):
        import torch.distributed as dist
        if not dist.is_initialized() or dist.get_world_size(group) == 1:
            return [blob]
        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, blob, group=group)
        return out
    return gather


class PeerExpertParallel:
    """The layer step through dsv4cu_ep_* (peer memory over NVLink).

    layer: this rank's dsv4cu_moe (experts_per_rank routed experts + the shared
    expert). allgather: callable(bytes) -> list[bytes] in rank order, used
    once to exchange the ranks' buffer handles. All ranks call forward in
    lockstep."""

    def __init__(self, dev, layer, rank: int, world: int, nt_max: int, hidden: int, topk: int,
                 experts_per_rank: int, route_scale: float, limit: float, allgather):
        import torch
        self.torch, self.dev, self.layer = torch, dev, layer
        self.hidden, self.topk = hidden, topk
        self.route_scale, self.limit = route_scale, limit
        self.ep = dev.ep_create(rank, world, nt_max, hidden, topk, experts_per_rank)
        try:
            dev.ep_connect(self.ep, allgather(dev.ep_handle(self.ep)))
        except Exception:
            dev.ep_destroy(self.ep)
            self.ep = None
            raise

    def forward(self, x, logits, out=None, idx=None, wts=None, events=None):
        nt = x.shape[0]
        if out is None:
            out = self.torch.empty((nt, self.hidden), dtype=self.torch.float32, device=x.device)
        self.dev.ep_forward(self.ep, self.layer, out, x, logits, nt, self.route_scale, self.limit, idx, wts, events)
        return out

    def close(self):
        if self.ep is not None:
            self.dev.ep_destroy(self.ep)
            self.ep = None
