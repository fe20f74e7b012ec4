"""Q8_K on the GPU through the C ABI against the CPU oracle (matvec_q8_k_cpu,
src/metal/compute.rs:971-993, pinned in tests/test_oracle_q8k.py with the reference's
known-answer tests): raw bytes (block sums included) round trip, bit-exact dequantization
(d * q), matvecs within rel. error 1e-3 (floor 1e-3 * ||r||_inf, fp64 arbiter)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from _util import parity, rel_err  # noqa: E402

DEV = "cuda:0"
Q8_K = 15


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


def raw_q8k(rng, rows, cols):
    nb = cols // 256
    raw = rng.integers(0, 256, (rows, nb * 292), dtype=np.uint8)
    ds = rng.uniform(1e-4, 1e-3, (rows, nb)).astype(np.float32).view(np.uint8).reshape(rows, nb, 4)
    for b in range(nb):
        raw[:, b * 292:b * 292 + 4] = ds[:, b]
    return raw


def test_upload_download_round_trip_and_dequant_bitexact(ctx):
    rng = np.random.default_rng(111)
    rows, cols = 21, 768
    raw = raw_q8k(rng, rows, cols)
    w = ssdllm.Weight.upload(ctx, raw, Q8_K, rows, cols)
    try:
        assert np.array_equal(w.download().reshape(raw.shape), raw)
        out = torch.zeros(rows * cols, device=DEV)
        ssdllm.dequantize(ctx, w, out)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), ora.dequantize(raw, Q8_K, rows * cols))
    finally:
        w.free()


@pytest.mark.parametrize("rows,cols", [(1, 256), (9, 1280), (300, 4096), (2048, 11008 // 256 * 256)])
def test_matvec_matches_oracle(ctx, rows, cols):
    rng = np.random.default_rng(rows * 19 + cols)
    raw = raw_q8k(rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    w = ssdllm.Weight.upload(ctx, raw, Q8_K, rows, cols)
    try:
        y = torch.zeros(rows, device=DEV)
        ssdllm.matvec(ctx, w, torch.from_numpy(x).to(DEV), y)
        torch.cuda.synchronize()
    finally:
        w.free()
    ref = ora.matvec_quantized(raw, x, rows, cols, Q8_K, threads=8)
    exact = ora.dequantize(raw, Q8_K, rows * cols).reshape(rows, cols).astype(np.float64) @ \
        x.astype(np.float64)
    got = y.cpu().numpy()
    assert parity(got, ref, exact), (rel_err(got, ref), rel_err(ref, exact), rel_err(got, exact))
