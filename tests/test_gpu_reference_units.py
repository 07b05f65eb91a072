"""The reference's own unit tests, run against this library.

oracle/Makefile (target `units`) compiles the reference's tests/unit/test_matmul.c,
test_indexer.c, test_attn.c and test_ops.c (with tests/unit/ref_kernels.c and the
reference files that define no replaced symbol), and test_layer.c with the rest of
the engine, and links them against libdsv4cu.so in place of the reference's
src/10_compute kernel objects: dsv4_mmq_n, fp8_n, fp4_n, bf16_n, dsv4_rmsnorm,
dsv4_route, dsv4_swiglu, dsv4_expert_forward, dsv4_indexer_score, dsv4_topk,
dsv4_indexer_offset, dsv4_window_idxs and dsv4_sparse_attn then resolve to the
CUDA library, and the reference's own gates (exact fixtures, batch == GEMV bit
equality, the 1e-6 L2 bound, tie order, masks and sinks, router and SwiGLU
edge cases, a whole transformer block through a fake expert cache) judge it. The binaries are built where the reference tree is
present and travel with the repository; the test is skipped without them.
"""
from __future__ import annotations

import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BIN = os.path.join(ROOT, "oracle", "_ref")


@pytest.mark.parametrize("unit", ["matmul", "indexer", "attn", "ops", "layer"])
def test_reference_unit_passes_on_the_library(unit):
    exe = os.path.join(REF_BIN, f"test_{unit}")
    if not os.path.exists(exe):
        pytest.skip(f"{exe} not built (needs the reference tree at build time)")
    env = dict(os.environ, OMP_NUM_THREADS=os.environ.get("OMP_NUM_THREADS", "8"))
    r = subprocess.run([exe], capture_output=True, text=True, timeout=900, env=env)
    tail = (r.stdout + r.stderr)[-3000:]
    print(tail)
    assert r.returncode == 0, tail
