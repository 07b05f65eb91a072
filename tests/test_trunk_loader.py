"""Dense trunk loader (dsv4cu_trunk_*): trunk.idx / trunk.bin of the
reference's pack (src/50_loader/dsv4_trunk_manifest.c:24-110,
dsv4_trunk.c:37-131) straight into HBM. The manifest reader runs on the host
(CPU tests); the upload, slot lookup, matrix descriptors and vector widening
run on the device (GPU tests), with a loaded FP8 matrix driven through the
GEMV against the oracle."""
from __future__ import annotations

import os

import numpy as np
import pytest

import dsv4cu
import trunkfix


def _ix_lines(root):
    with open(os.path.join(root, "trunk.idx")) as f:
        return f.read().split("\n")


def _write_ix(root, lines):
    with open(os.path.join(root, "trunk.idx"), "w") as f:
        f.write("\n".join(lines))


class _DevBytes:
    """A device byte range as an array torch can view (CUDA array interface)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def test_manifest_records(tmp_path):
    root = str(tmp_path)
    layers = trunkfix.write_trunk(root, 3, empty_layers=(1,), seed=5)
    nl, run, recs = dsv4cu.trunk_manifest(root)
    assert nl == 3 and run is None and recs is None
    for L in range(3):
        _, run, recs = dsv4cu.trunk_manifest(root, L)
        want = layers[L]
        assert len(recs) == len(want)
        if not want:
            assert run[1] == 0
        for r in recs:
            rec, _ = want[r.slot]
            assert (r.slot, r.off, r.nbytes, r.dtype, r.rows, r.cols, r.wdt, r.blk_r, r.blk_c) == rec
        assert run[0] % trunkfix.ALIGN == 0
        assert run[2] == sum(rec[5] * 4 for rec, _ in want.values() if rec[3] == trunkfix.DT_BF16 and rec[4] == 1)


@pytest.mark.parametrize("edit", ["magic", "version", "n_layers", "layout", "layer_index", "tensor_fields",
                                  "dtype", "wdt", "outside_run", "missing"])
def test_manifest_rejects_malformed(tmp_path, edit):
    root = str(tmp_path)
    trunkfix.write_trunk(root, 2, seed=6)
    lines = _ix_lines(root)
    first_slot = next(i for i, s in enumerate(lines) if s.startswith("slot "))
    f = lines[first_slot].split()
    if edit == "magic":
        lines[0] = "DSV4TRUNX 2"
    elif edit == "version":
        lines[0] = "DSV4TRUNK 1"
    elif edit == "n_layers":
        lines[1] = "n_layers 0"
    elif edit == "layout":
        lines[2] = "layout 2"
    elif edit == "layer_index":
        lines[3] = lines[3].replace("layer 0", "layer 1", 1)
    elif edit == "tensor_fields":
        lines[first_slot] = " ".join(f[:-1])
    elif edit == "dtype":
        f[4] = "9"
        lines[first_slot] = " ".join(f)
    elif edit == "wdt":
        f[7] = "4"
        lines[first_slot] = " ".join(f)
    elif edit == "outside_run":
        f[2] = str(10 ** 9)
        lines[first_slot] = " ".join(f)
    elif edit == "missing":
        os.remove(os.path.join(root, "trunk.idx"))
    if edit != "missing":
        _write_ix(root, lines)
    with pytest.raises(dsv4cu.DSV4CUError):
        dsv4cu.trunk_manifest(root)


def _ours(root, L):
    nl, run, recs = dsv4cu.trunk_manifest(root, L)
    return nl, run, [(r.slot, r.off, r.nbytes, r.dtype, r.rows, r.cols, r.wdt, r.blk_r, r.blk_c) for r in recs]


_ref_trunk = pytest.mark.skipif(not __import__("oracle").ref_trunk_available(),
                                reason="oracle/_ref/libdsv4trunk.so not built (needs the reference tree)")


@_ref_trunk
def test_manifest_matches_reference_reader(tmp_path):
    """The library's trunk.idx reader against the reference's own
    (dsv4_trunk_load_manifest, compiled into oracle/_ref): the same layers,
    runs and records in order, blank lines and an empty layer included."""
    import oracle
    root = str(tmp_path)
    trunkfix.write_trunk(root, 4, empty_layers=(2,), seed=11)
    assert oracle.ref_trunk_manifest(root)[0] == dsv4cu.trunk_manifest(root)[0] == 4
    for L in range(4):
        assert oracle.ref_trunk_manifest(root, L) == _ours(root, L), L


@_ref_trunk
@pytest.mark.parametrize("edit", ["magic", "version", "n_layers", "layout", "layer_index", "tensor_fields",
                                  "dtype", "wdt", "missing"])
def test_manifest_rejections_match_reference(tmp_path, edit):
    """Every malformed index the reference's reader rejects, the library's
    rejects too. (The library also rejects a tensor lying outside its layer's
    run, which the reference accepts: its device copy of the run would not
    hold that tensor.)"""
    import oracle
    root = str(tmp_path)
    trunkfix.write_trunk(root, 2, seed=12)
    lines = _ix_lines(root)
    first_slot = next(i for i, s in enumerate(lines) if s.startswith("slot "))
    f = lines[first_slot].split()
    edits = {"magic": (0, "DSV4TRUNX 2"), "version": (0, "DSV4TRUNK 1"), "n_layers": (1, "n_layers 0"),
             "layout": (2, "layout 2"), "layer_index": (3, lines[3].replace("layer 0", "layer 1", 1)),
             "tensor_fields": (first_slot, " ".join(f[:-1])),
             "dtype": (first_slot, " ".join(f[:4] + ["9"] + f[5:])),
             "wdt": (first_slot, " ".join(f[:7] + ["4"] + f[8:]))}
    if edit == "missing":
        os.remove(os.path.join(root, "trunk.idx"))
    else:
        i, v = edits[edit]
        lines[i] = v
        _write_ix(root, lines)
    assert oracle.ref_trunk_manifest(root) is None
    with pytest.raises(dsv4cu.DSV4CUError):
        dsv4cu.trunk_manifest(root)


@pytest.mark.gpu
def test_trunk_upload_slots_and_widen(tmp_path, dev):
    import torch
    root = str(tmp_path)
    layers = trunkfix.write_trunk(root, 3, empty_layers=(1,), seed=7)
    h = dev.trunk_load(root)
    try:
        assert dev.trunk_resident_bytes(h) % trunkfix.ALIGN == 0
        for L, slots in layers.items():
            for slot, (rec, arr) in slots.items():
                d, p = dev.trunk_slot(h, L, slot)
                assert p % 16 == 0 and d.nbytes == arr.nbytes
                got = torch.as_tensor(_DevBytes(p, arr.nbytes), device="cuda").cpu().numpy()
                assert np.array_equal(got, np.frombuffer(arr.tobytes(), np.uint8)), (L, slot)
        # packed matrices: weights and the next slot's scales
        q = dev.trunk_qmat(h, 0, 10)
        d, p = dev.trunk_slot(h, 0, 10)
        _, ps = dev.trunk_slot(h, 0, 11)
        assert (q.w, q.s, q.wdt, q.rows, q.cols, q.blk_r, q.blk_c) == (p, ps, 2, d.rows, d.cols, 128, 128)
        q4 = dev.trunk_qmat(h, 2, 50)
        assert q4.wdt == 3 and q4.blk_c == 32 and q4.s == dev.trunk_slot(h, 2, 51)[1]
        # vectors widened as the reference binds them: bf16 exactly, f32 copied
        rec, bits = layers[0][1]
        out = torch.full((rec[5],), float("nan"), device="cuda")
        dev.trunk_widen(h, 0, 1, out)
        want = (bits.astype(np.uint32) << 16).view(np.float32)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
        rec3, v3 = layers[2][3]
        out3 = torch.empty(rec3[5], device="cuda")
        dev.trunk_widen(h, 2, 3, out3)
        assert np.array_equal(out3.cpu().numpy(), v3)
        with pytest.raises(dsv4cu.DSV4CUError):
            dev.trunk_widen(h, 0, 41, out3)      # i64 is not a vector the bind widens
        with pytest.raises(dsv4cu.DSV4CUError):
            dev.trunk_slot(h, 1, 10)             # the empty layer has no tensors
        with pytest.raises(dsv4cu.DSV4CUError):
            dev.trunk_slot(h, 0, 12)             # no such slot
    finally:
        dev.trunk_free(h)
    dev.check_status()


@pytest.mark.gpu
def test_trunk_partial_load_and_gemv(tmp_path, dev, orc):
    """Layers [2, 3) only; its FP8 matrix runs through the GEMV against the
    oracle on the file's bytes."""
    import torch
    import oracle
    import pack
    root = str(tmp_path)
    layers = trunkfix.write_trunk(root, 3, hidden=1024, rows_a=512, seed=8)
    h = dev.trunk_load(root, 2, 1)
    try:
        with pytest.raises(dsv4cu.DSV4CUError):
            dev.trunk_slot(h, 0, 10)             # not resident
        q = dev.trunk_qmat(h, 2, 10)
        (rec, W), (_, S) = layers[2][10], layers[2][11]
        x = pack.bf16_round(np.random.default_rng(9).standard_normal((1, 1024)).astype(np.float32))
        y = torch.empty((1, 512), dtype=torch.float32, device="cuda")
        dev.mmq(y, torch.from_numpy(x).cuda(), q, 1)
        qm = oracle.qmat(W, S, 2, 512, 1024, 128, 128)
        want = orc.mmq(x, qm)
        err = float(np.max(np.abs(y.cpu().numpy() - want)) / max(1e-30, np.max(np.abs(want))))
        assert err <= 1e-5, err
    finally:
        dev.trunk_free(h)
    dev.check_status()
