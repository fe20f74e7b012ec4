"""16-bit dense weights (F16, BF16) on the GPU against the oracle (matvec_f16_cpu /
matvec_bf16_cpu, src/metal/compute.rs:2250-2285): the reference's own known-answer tests
through the host-pointer entry point (2 x 2 matrices: any column count), bit-exact
dequantization, byte round trip, and random matrices within rel. error 1e-3 (fp64 arbiter)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from _util import parity, rel_err  # noqa: E402

DEV = "cuda:0"
F16, BF16 = 1, 30


@pytest.fixture(scope="module")
def comp():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.CudaCompute(0)


def test_kats_through_the_host_entry_point(comp):
    """compute.rs:2988-3040 (the four matvec KATs)."""
    cases = [
        ([0x80, 0x3F, 0x00, 0x00, 0x00, 0x00, 0x80, 0x3F], [3.0, 7.0], BF16, [3.0, 7.0]),
        ([0x80, 0x3F, 0x00, 0x40, 0x40, 0x40, 0x80, 0x40], [1.0, 1.0], BF16, [3.0, 7.0]),
        ([0x00, 0x3C, 0x00, 0x00, 0x00, 0x00, 0x00, 0x3C], [5.0, 9.0], F16, [5.0, 9.0]),
        ([0x00, 0x3C, 0x00, 0x40, 0x00, 0x42, 0x00, 0x44], [1.0, 1.0], F16, [3.0, 7.0]),
    ]
    for w, x, t, expect in cases:
        y = comp.matvec_quantized(np.array(w, np.uint8), np.array(x, np.float32), 2, 2, t)
        assert np.allclose(y, expect, atol=1e-2), (t, y)


def raw16(rng, rows, cols, t):
    if t == F16:
        return (rng.standard_normal((rows, cols)) * 0.05).astype(np.float16).view(np.uint8)
    f = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32)
    return (f.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)


@pytest.mark.parametrize("t", [F16, BF16])
@pytest.mark.parametrize("rows,cols", [(5, 37), (300, 4096), (1024, 1000), (4096, 4096)])
def test_matvec_and_dequant(comp, t, rows, cols):
    ctx = comp.ctx
    rng = np.random.default_rng(rows + cols + t)
    raw = raw16(rng, rows, cols, t).reshape(rows, cols * 2)
    x = rng.standard_normal(cols).astype(np.float32)
    w = ssdllm.Weight.upload(ctx, raw, t, rows, cols)
    try:
        assert np.array_equal(w.download().reshape(raw.shape), raw)
        y = torch.zeros(rows, device=DEV)
        ssdllm.matvec(ctx, w, torch.from_numpy(x).to(DEV), y)
        if (rows * cols) % 8 == 0:
            out = torch.zeros(rows * cols, device=DEV)
            ssdllm.dequantize(ctx, w, out)
        torch.cuda.synchronize()
    finally:
        w.free()
    ref = ora.matvec_quantized(raw, x, rows, cols, t, threads=8)
    wf = ora.dequantize(raw, t, rows * cols)
    if (rows * cols) % 8 == 0:
        assert np.array_equal(out.cpu().numpy(), wf)
    exact = wf.reshape(rows, cols).astype(np.float64) @ x.astype(np.float64)
    got = y.cpu().numpy()
    assert parity(got, ref, exact), (rel_err(got, ref), rel_err(ref, exact))
