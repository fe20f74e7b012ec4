"""Failure detection on one GPU without a fault: a bounded device wait that runs out.

The tensor-parallel consumer kernels wait for every rank's flag before summing the ranks'
partial rows (the peer-memory all-reduce; the reference has no counterpart, its thread row
split has no reduction, src/inference/tensor_parallel.rs:33-105). Here one rank's flag is
never raised: the wait gives up after its iteration limit (well under a second), the kernel
returns, ssd_ctx_device_status reports SSD_ERR_TIMEOUT once and clears it, and the same
context then runs the call correctly once the flag is set. Nothing faults, traps or hangs."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from _util import rel_err  # noqa: E402

SSD_ERR_TIMEOUT = 5  # include/ssdllm_cuda.h


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


@pytest.mark.parametrize("impl", ["fma", "i8"])
def test_peer_wait_times_out_reports_and_recovers(ctx, monkeypatch, impl):
    monkeypatch.setenv("SSD_MV_IMPL", impl)
    assert ssdllm.lib().ssd_status_str(SSD_ERR_TIMEOUT) == b"device wait timed out"
    rng = np.random.default_rng(8)
    rows, cols, ranks = 512, 1024, 2
    raw = ora.quantize((rng.standard_normal((rows, cols)) * 0.02).astype(np.float32), ora.Q4_0)
    w = ssdllm.Weight.upload(ctx, raw, ora.Q4_0, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    part = rng.standard_normal((ranks, cols)).astype(np.float32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")
    xd, pd = dev(x), dev(part)
    flags = torch.zeros(ranks, dtype=torch.int64, device="cuda:0")
    epoch = torch.zeros(1, dtype=torch.int64, device="cuda:0")
    y = torch.zeros(rows, device="cuda:0")
    assert ctx.device_status() == 0

    # rank 1's flag is never raised: the bounded wait gives up
    flags[0] = 1
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ssdllm.matvec_peer_input(ctx, w, xd, pd, ranks, flags, epoch, 0, y)
    st = ctx.device_status()  # synchronises the device
    waited = time.perf_counter() - t0
    assert st == SSD_ERR_TIMEOUT, st
    assert waited < 10.0, waited
    assert ctx.device_status() == 0  # read once, then cleared

    # the same context, the flag now raised: the call completes with the right sum
    flags[1] = 1
    y.zero_()
    ssdllm.matvec_peer_input(ctx, w, xd, pd, ranks, flags, epoch, 0, y)
    assert ctx.device_status() == 0
    xe = (x + part[0]) + part[1]
    ref = ora.matvec_quantized(raw, xe, rows, cols, ora.Q4_0)
    assert rel_err(y.cpu().numpy(), ref) <= 1e-3
    # and a plain call afterwards
    y2 = torch.zeros(rows, device="cuda:0")
    ssdllm.matvec(ctx, w, xd, y2)
    assert ctx.device_status() == 0
    assert rel_err(y2.cpu().numpy(), ora.matvec_quantized(raw, x, rows, cols, ora.Q4_0)) <= 1e-3
    w.free()
