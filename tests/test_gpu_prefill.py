"""GPU parity of the batch-prefill GEMM (tcgen05 tensor cores) against the oracle.

ssd_prefill_matmul computes y[t] = W x[t] for a block of prompt tokens at once; the
reference computes the same rows one matvec_quantized call per token inside
batch_prefill_lora (src/inference/transformer.rs:120-250). Each token row is compared with
the oracle's per-token quantized matvec at the parity tolerance (rel. error <= 1e-3 with a
floor of 1e-3 of the row's max; an fp64 product arbitrates where the oracle's own sequential
fp32 sum is what exceeds it)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from _util import parity, rel_err  # noqa: E402

DEV = "cuda:0"


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


@pytest.mark.parametrize("wtype,rows,cols,tokens", [
    (ora.Q4_K, 512, 4096, 128),   # 256-wide tiles
    (ora.Q4_K, 384, 1024, 256),   # 128-wide tiles, two token tiles
    (ora.Q4_0, 256, 2048, 128),
    (ora.Q8_0, 128, 512, 128),
])
def test_prefill_matmul_matches_per_token_matvec(ctx, wtype, rows, cols, tokens):
    rng = np.random.default_rng(rows + cols + tokens)
    wf = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    raw = ora.quantize(wf, wtype)
    w = ssdllm.Weight.upload(ctx, raw, wtype, rows, cols)
    x = rng.standard_normal((tokens, cols)).astype(np.float32)
    y = torch.full((tokens, rows), float("nan"), device=DEV)
    ssdllm.prefill_matmul(ctx, w, torch.from_numpy(x).to(DEV), y)
    torch.cuda.synchronize()
    assert ctx.device_status() == 0
    got = y.cpu().numpy()
    deq = ora.dequantize(raw, wtype, rows * cols).reshape(rows, cols).astype(np.float64)
    worst = 0.0
    for t in range(0, tokens, max(1, tokens // 16)):
        ref = ora.matvec_quantized(raw, x[t], rows, cols, wtype, threads=8)
        exact = deq @ x[t].astype(np.float64)
        assert parity(got[t], ref, exact), (t, rel_err(got[t], ref), rel_err(ref, exact),
                                            rel_err(got[t], exact))
        worst = max(worst, rel_err(got[t], exact))
    assert np.all(np.isfinite(got))
    w.free()
