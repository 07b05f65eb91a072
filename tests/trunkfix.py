"""Synthetic dense trunks in the reference's pack layout, for the trunk loader tests.

Writes what the reference's tools/pack_trunk.py writes for the dense trunk
(read by src/50_loader/dsv4_trunk_manifest.c:24-110 and dsv4_trunk.c:14-35):
trunk.idx, a text manifest ("DSV4TRUNK 2", "n_layers N", "layout 1", per
layer "layer L file_off nbytes n_tensors widen_bytes" and per tensor "slot id
off nbytes dtype rows cols wdt blk_r blk_c", off within the layer run), and
trunk.bin holding each layer's run at a 4 KiB aligned file offset. Slot ids
follow the pack's pairing of a packed matrix X with its scales X_S in the next
id (src/50_loader/dsv4_bind_layer.c:10-23).
"""
from __future__ import annotations

import os

import numpy as np

import pack

DT_U8, DT_BF16, DT_F32, DT_E4M3, DT_E8M0, DT_I64 = 1, 2, 4, 5, 6, 8
WF32, WBF16, WFP8, WFP4 = 0, 1, 2, 3
ALIGN = 4096


def _bf16_bits(a):
    return (pack.bf16_round(a.astype(np.float32)).view(np.uint32) >> 16).astype(np.uint16)


def layer_tensors(rng, hidden, rows_a):
    """(slot, dtype, rows, cols, wdt, blk_r, blk_c, payload array) of one layer."""
    out = []
    out.append((1, DT_BF16, 1, hidden, WF32, 0, 0, _bf16_bits(rng.standard_normal(hidden))))   # a norm
    out.append((3, DT_F32, 1, 64, WF32, 0, 0, rng.standard_normal(64).astype(np.float32)))     # a sink
    w = (rng.standard_normal((rows_a, hidden)) * 0.02).astype(np.float32)
    W, S = pack.quantize_fp8(w)                                                                 # FP8 128x128
    out.append((10, DT_E4M3, rows_a, hidden, WFP8, 128, 128, W))
    out.append((11, DT_E8M0, S.shape[0], S.shape[1], WF32, 0, 0, S))
    w4 = (rng.standard_normal((256, hidden)) * 0.02).astype(np.float32)
    W4, S4 = pack.quantize_fp4(w4)                                                              # FP4 1x32
    out.append((50, DT_U8, 256, hidden, WFP4, 1, 32, W4))
    out.append((51, DT_E8M0, S4.shape[0], S4.shape[1], WF32, 0, 0, S4))
    g = _bf16_bits(rng.standard_normal((16, hidden)))                                           # bf16 matrix
    out.append((40, DT_BF16, 16, hidden, WBF16, 0, 0, g))
    out.append((41, DT_I64, 1, 16, WF32, 0, 0, rng.integers(0, 16, 16).astype(np.int64)))
    return out


def write_trunk(root, n_layers, hidden=512, rows_a=384, empty_layers=(), seed=0):
    """Returns {layer: {slot: (record tuple, payload)}}; layers in empty_layers
    have no tensors and an empty run."""
    rng = np.random.default_rng(seed)
    os.makedirs(root, exist_ok=True)
    blob = bytearray(rng.integers(0, 256, 777, dtype=np.uint8).tobytes())   # leading filler
    lines = ["DSV4TRUNK 2", f"n_layers {n_layers}", "layout 1"]
    layers = {}
    for L in range(n_layers):
        blob += bytes((-len(blob)) % ALIGN)
        file_off = len(blob)
        ts = [] if L in empty_layers else layer_tensors(rng, hidden, rows_a)
        run = bytearray()
        recs, widen = [], 0
        for (slot, dt, r, c, wdt, br, bc, a) in ts:
            run += rng.integers(0, 256, int(rng.integers(0, 3)) * 16, dtype=np.uint8).tobytes()   # gaps
            run += bytes((-len(run)) % 16)
            recs.append((slot, len(run), a.nbytes, dt, r, c, wdt, br, bc))
            run += a.tobytes()
            if dt == DT_BF16 and r == 1:
                widen += c * 4
        blob += run
        lines.append(f"layer {L} {file_off} {len(run)} {len(recs)} {widen}")
        lines += ["slot " + " ".join(str(v) for v in rec) for rec in recs]
        if not recs:
            lines.append("")   # blank lines are skipped
        layers[L] = {rec[0]: (rec, t[7]) for rec, t in zip(recs, ts)}
    with open(os.path.join(root, "trunk.bin"), "wb") as f:
        f.write(bytes(blob))
    with open(os.path.join(root, "trunk.idx"), "w") as f:
        f.write("\n".join(lines) + "\n")
    return layers
