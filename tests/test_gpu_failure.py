"""The failure path of the bounded device waits, driven on purpose without
faulting anything: a test-only option (dsv4cu_ctx_inject) makes the streamed
GEMV's first CTA skip one weight stage, so nothing ever arrives on that
stage's barrier. The consumers' 2 s wait must expire, every role of the
kernel must stop through its own bounded waits, the host must read the
timeout from dsv4cu_ctx_status, and the next call must give the same bits as
before - the context stays usable."""
from __future__ import annotations

import time

import numpy as np
import pytest

import oracle
import pack

pytestmark = pytest.mark.gpu

SMV_CODES = {51: "full", 52: "empty", 53: "epilogue", 54: "dependency", 55: "epilogue buffer", 56: "operand"}


def test_withheld_stage_times_out_and_context_recovers(dev, orc):
    import torch
    rows = cols = 7168                      # config 1: ~10 stages per CTA, so CTA 0 has a stage 2
    src = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    dev.fill_normal(src, 77, 0.0, 0.02)
    W = torch.empty(rows * cols, dtype=torch.uint8, device="cuda")
    S = torch.empty((rows // 128) * (cols // 128), dtype=torch.uint8, device="cuda")
    dev.quantize_fp8(W, S, src, rows, cols)
    del src
    m = dev.qmat(W, S, 2, rows, cols, 128, 128)
    rng = np.random.default_rng(3)
    x = pack.bf16_round(rng.standard_normal((1, cols)).astype(np.float32))
    dx = torch.from_numpy(x).cuda()
    y0, y1, y2 = (torch.empty((1, rows), dtype=torch.float32, device="cuda") for _ in range(3))

    dev.gemv(y0, dx, m, 1)
    assert dev.status_code() == 0
    hW, hS = W.cpu().numpy(), S.cpu().numpy()        # kept alive: the QMat holds raw pointers
    want = orc.mmq(x, oracle.qmat(hW, hS, 2, rows, cols, 128, 128))
    got = y0.cpu().numpy()
    assert float(np.abs(got - want).max() / np.abs(want).max()) <= 1e-3

    dev.inject(dev.INJECT_WITHHOLD_STAGE)
    t0 = time.perf_counter()
    dev.gemv(y1, dx, m, 1)
    code = dev.status_code()
    dt = time.perf_counter() - t0
    assert code in SMV_CODES, code
    assert 1.5 <= dt <= 60.0, dt              # the 2 s limit ran out, and the kernel then ended

    dev.gemv(y2, dx, m, 1)                    # the next call: normal, same bits
    assert dev.status_code() == 0
    assert np.array_equal(y2.cpu().numpy().view(np.uint32), got.view(np.uint32))


def test_inject_rejects_unknown_fault(dev):
    import dsv4cu
    with pytest.raises(dsv4cu.DSV4CUError):
        dev.inject(99)
