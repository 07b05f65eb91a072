"""The C-ABI library loads and exports every entry point include/*.h declares.

CPU only: nothing here launches a kernel.
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from conftest import PKG, ROOT

HEADERS = [os.path.join(ROOT, "include", h) for h in sorted(os.listdir(os.path.join(ROOT, "include")))
           if h.endswith(".h")]
LIB = os.path.join(PKG, "libdsv4cu.so")


def declared_functions():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(", src, flags=re.M):
            name = m.group(1)
            line = src[m.start():src.find("\n", m.start())]
            if line.lstrip().startswith(("typedef", "#", "return", "if", "enum", "struct")):
                continue
            names.add(name)
    return sorted(names)


@pytest.fixture(scope="module")
def built_lib():
    if not os.path.exists(LIB):
        subprocess.run(["make", "-s", "-C", PKG], check=True)
    return LIB


def test_headers_declare_the_reference_entry_points():
    names = set(declared_functions())
    # src/10_compute/dsv4_matmul.h:40-52, dsv4_kernels.h, 80_prefill/dsv4_prefill_vk.h:31-49
    for ref in ("dsv4_mmq_n", "dsv4_mmq", "bf16_n", "fp8_n", "fp4_n", "dsv4_route", "dsv4_swiglu", "dsv4_rmsnorm",
                "dsv4_expert_forward", "dsv4_indexer_score", "dsv4_topk", "dsv4_indexer_offset",
                "dsv4_sparse_attn", "dsv4_window_idxs", "dsv4_prefill_vk_init",
                "dsv4_prefill_vk_free", "dsv4_prefill_vk_gemm", "dsv4_prefill_vk_expert_fused"):
        assert ref in names, ref


def test_library_exports_every_declared_symbol(built_lib):
    lib = ctypes.CDLL(built_lib)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_no_cxx_types_in_headers():
    for h in HEADERS:
        src = open(h).read()
        for bad in ("torch", "std::", "at::Tensor", "c10::"):
            assert bad not in src, (h, bad)


def test_binding_raises_without_library(tmp_path, monkeypatch):
    import dsv4cu
    monkeypatch.setattr(dsv4cu, "LIB_PATH", str(tmp_path / "missing.so"))
    monkeypatch.setattr(dsv4cu, "_lib", None)
    with pytest.raises(dsv4cu.DSV4CUError):
        dsv4cu.lib()


def test_reference_engine_links_against_the_library(built_lib):
    """The reference's whole engine, linked with the CPU kernel files the library
    replaces left out (oracle/Makefile target `engine`): every compute symbol the
    engine uses resolves in libdsv4cu.so. Needs the reference tree (built where
    oracle/_ref/libdsv4ref.so was built)."""
    import json
    with open(os.path.join(ROOT, "BASELINE.json")) as f:
        tree = json.load(f).get("reference_path") or ""
    if not os.path.isdir(os.path.join(tree, "src", "10_compute")):
        pytest.skip("reference tree not available here")
    r = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "engine", f"REF={tree}"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    exe = os.path.join(ROOT, "oracle", "_ref", "dsv4-serve-cuda")
    und = subprocess.run(["nm", "-u", exe], capture_output=True, text=True).stdout.split()
    need = {s for s in und if s.startswith("dsv4_") or s in ("fp8_n", "fp4_n", "bf16_n")}
    lib = ctypes.CDLL(built_lib)
    assert need and all(hasattr(lib, s) for s in need), sorted(need)


def test_bf16w_workspace_follows_the_dequantization_path(built_lib):
    """Host logic only: the exact-weight GEMM's workspace holds the bf16
    activation rows, plus a bf16 copy of the matrix when the call takes the
    pre-dequantized path (automatic above 256 token rows, or forced); bad
    path codes are rejected and the automatic choice is restored."""
    import sys
    sys.path.insert(0, PKG)
    import dsv4cu
    L = dsv4cu.lib()
    q = dsv4cu.QMat(None, None, 2, 6144, 4096, 128, 128)
    ws = lambda nt, terms: L.dsv4cu_gemm_bf16w_workspace(ctypes.byref(q), nt, terms)
    x_bytes = lambda nt, terms: -(-nt * terms * 4096 * 2 // 256) * 256
    copy = 6144 * 4096 * 2
    try:
        assert L.dsv4cu_gemm_bf16w_set_path(0) == 0
        assert ws(128, 2) == x_bytes(128, 2)                 # one 256-row token tile: converters
        assert ws(129, 2) == x_bytes(129, 2) + copy          # more: one bf16 copy per call
        assert ws(4096, 1) == x_bytes(4096, 1) + copy
        assert L.dsv4cu_gemm_bf16w_set_path(1) == 0
        assert ws(4096, 1) == x_bytes(4096, 1)
        assert L.dsv4cu_gemm_bf16w_set_path(2) == 0
        assert ws(8, 1) == x_bytes(8, 1) + copy
        assert L.dsv4cu_gemm_bf16w_set_path(3) != 0
        assert ws(0, 1) == 0 and ws(8, 3) == 0
    finally:
        L.dsv4cu_gemm_bf16w_set_path(0)
