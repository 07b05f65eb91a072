"""Synthetic packs in the reference's expert layout, for the loader tests.

Writes what the reference's tools/pack_trunk.py writes for routed experts
(read by src/40_io/dsv4_st.c:65-143): experts.idx = b"DSV4EXP1", int32
n_layers, int32 n_experts, then per (layer, expert) six records {int32 shard,
int32 pad, int64 offset, int64 bytes} for w1, w1 scales, w2, w2 scales, w3,
w3 scales; shards = *.safetensors files numbered in name order. Payloads are
placed at scattered offsets across the shards, behind filler bytes.
"""
from __future__ import annotations

import os
import struct

import numpy as np

SHARD_NAMES = ["model-00002-of-00002.safetensors", "model-00001-of-00002.safetensors"]


def expert_tensors(rng, hidden, inter):
    """w1, w1 scales, w2, w2 scales, w3, w3 scales as uint8 arrays (FP4 1x32 E8M0)."""
    def mat(rows, cols):
        W = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
        S = rng.integers(118, 127, (rows, cols // 32), dtype=np.uint8)
        return W, S
    w1, s1 = mat(inter, hidden)
    w2, s2 = mat(hidden, inter)
    w3, s3 = mat(inter, hidden)
    return [w1, s1, w2, s2, w3, s3]


def write_pack(root, n_layers, n_experts, hidden, inter, seed=0):
    """Returns {(layer, expert): [six arrays]} and the shard paths in index order."""
    rng = np.random.default_rng(seed)
    os.makedirs(root, exist_ok=True)
    paths = sorted(os.path.join(root, n) for n in SHARD_NAMES)      # shard i = i-th in name order
    blobs = [bytearray(rng.integers(0, 256, 123, dtype=np.uint8).tobytes()) for _ in paths]
    tensors, recs = {}, []
    for L in range(n_layers):
        for e in range(n_experts):
            ts = expert_tensors(rng, hidden, inter)
            tensors[(L, e)] = ts
            for t in ts:
                sh = int(rng.integers(0, len(paths)))
                blobs[sh] += rng.integers(0, 256, int(rng.integers(0, 40)), dtype=np.uint8).tobytes()
                recs.append((sh, 0, len(blobs[sh]), t.nbytes))
                blobs[sh] += t.tobytes()
    for p, b in zip(paths, blobs):
        with open(p, "wb") as f:
            f.write(bytes(b))
    with open(os.path.join(root, "experts.idx"), "wb") as f:
        f.write(b"DSV4EXP1" + struct.pack("<ii", n_layers, n_experts))
        for r in recs:
            f.write(struct.pack("<iiqq", *r))
    return tensors, paths
