"""Q6_K on the GPU through the C ABI against the CPU oracle (matvec_q6_k_cpu,
src/metal/compute.rs:752-790, restated in oracle/oracle.c and pinned in
tests/test_oracle_q6k.py).

Bars: the upload repack and the download unpack are exact inverses (raw bytes round
trip); dequantization is bit-exact ((d * scale) * q, the reference's order); the
fp32-accumulated matvecs are within rel. error 1e-3 (floor 1e-3 * ||r||_inf), with an
fp64 arbiter where the oracle's own sequential sum is what differs. Blocks are random
bytes (every bit pattern is a valid Q6_K block) with d in a typical range.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from _util import parity, rel_err  # noqa: E402

TOL = 1e-3
DEV = "cuda:0"
Q6_K = 14


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


def d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, torch.float32)


def raw_q6k(rng, rows, cols):
    nb = cols // 256
    raw = rng.integers(0, 256, (rows, nb * 210), dtype=np.uint8)
    dv = rng.uniform(2e-5, 2e-4, (rows, nb)).astype(np.float16).view(np.uint16)
    for b in range(nb):
        raw[:, b * 210 + 208] = dv[:, b] & 0xFF
        raw[:, b * 210 + 209] = dv[:, b] >> 8
    return raw


def test_upload_download_round_trip_and_dequant_bitexact(ctx):
    rng = np.random.default_rng(71)
    rows, cols = 37, 768
    raw = raw_q6k(rng, rows, cols)
    w = ssdllm.Weight.upload(ctx, raw, Q6_K, rows, cols)
    try:
        assert np.array_equal(w.download().reshape(raw.shape), raw)
        out = torch.zeros(rows * cols, device=DEV)
        ssdllm.dequantize(ctx, w, out)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), ora.dequantize(raw, Q6_K, rows * cols))
    finally:
        w.free()


# (rows, cols): chunk counts below, at and above one 32-chunk step, ragged row counts,
# a 4096-wide layer and a wide row
CASES = [(1, 256), (7, 512), (33, 1280), (300, 4096), (4096, 4096), (1000, 11008 // 256 * 256)]


@pytest.mark.parametrize("rows,cols", CASES)
def test_matvec_matches_oracle(ctx, rows, cols):
    rng = np.random.default_rng(rows * 13 + cols)
    raw = raw_q6k(rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    w = ssdllm.Weight.upload(ctx, raw, Q6_K, rows, cols)
    try:
        y = torch.zeros(rows, device=DEV)
        ssdllm.matvec(ctx, w, d(x), y)
        torch.cuda.synchronize()
    finally:
        w.free()
    ref = ora.matvec_quantized(raw, x, rows, cols, Q6_K, threads=8)
    exact = ora.dequantize(raw, Q6_K, rows * cols).reshape(rows, cols).astype(np.float64) @ \
        x.astype(np.float64)
    got = y.cpu().numpy()
    assert parity(got, ref, exact), (rel_err(got, ref), rel_err(ref, exact), rel_err(got, exact))


def test_matvec_residual_and_swiglu(ctx):
    """The fused epilogues on Q6_K weights: y = base + W x, and SwiGLU over gate / up
    (RMSNorm folded into the prologue)."""
    rng = np.random.default_rng(72)
    E, F = 1024, 2816 // 256 * 256
    raw = raw_q6k(rng, E, E)
    x = rng.standard_normal(E).astype(np.float32)
    base = rng.standard_normal(E).astype(np.float32)
    w = ssdllm.Weight.upload(ctx, raw, Q6_K, E, E)
    wg_raw, wu_raw = raw_q6k(rng, F, E), raw_q6k(rng, F, E)
    G, U = (ssdllm.Weight.upload(ctx, a, Q6_K, F, E) for a in (wg_raw, wu_raw))
    nw = (rng.random(E) + 0.5).astype(np.float32)
    try:
        y = torch.zeros(E, device=DEV)
        ssdllm.matvec_residual(ctx, w, d(x), d(base), y)
        act = torch.zeros(F, device=DEV)
        ssdllm.fused_swiglu(ctx, G, U, d(x), d(nw), 1e-5, act)
        torch.cuda.synchronize()
    finally:
        for t in (w, G, U):
            t.free()
    ref = base + ora.matvec_quantized(raw, x, E, E, Q6_K)
    assert rel_err(y.cpu().numpy(), ref) <= TOL
    _, xn = ora.fused_post_attn_norm(x, np.zeros(E, np.float32), nw, 1e-5)
    ref = ora.silu(ora.matvec_quantized(wg_raw, xn, F, E, Q6_K)) * \
        ora.matvec_quantized(wu_raw, xn, F, E, Q6_K)
    assert rel_err(act.cpu().numpy(), ref) <= TOL


def test_rejects_cols_not_multiple_of_256(ctx):
    rng = np.random.default_rng(73)
    with pytest.raises(ssdllm.SsdError):
        ssdllm.Weight.upload(ctx, rng.integers(0, 256, 210, dtype=np.uint8), Q6_K, 1, 128)
