"""Q5_K on the GPU through the C ABI against the CPU oracle (matvec_q5_k_cpu,
src/metal/compute.rs:845-899, restated in oracle/oracle.c and pinned in
tests/test_oracle_q5k.py with the reference's own known-answer tests).

Bars: raw bytes round trip through upload and download; dequantization bit-exact
(scale * q - min, the reference's order); matvecs within rel. error 1e-3 (floor
1e-3 * ||r||_inf, fp64 arbiter). Blocks are random bytes with d, dmin in a typical range.
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
Q5_K = 13


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


def d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, torch.float32)


def raw_q5k(rng, rows, cols):
    nb = cols // 256
    raw = rng.integers(0, 256, (rows, nb * 176), dtype=np.uint8)
    for off in (0, 2):  # d, dmin
        v = rng.uniform(1e-4, 1e-3, (rows, nb)).astype(np.float16).view(np.uint16)
        raw[:, off::176] = (v & 0xFF).astype(np.uint8)
        raw[:, off + 1::176] = (v >> 8).astype(np.uint8)
    return raw


def test_upload_download_round_trip_and_dequant_bitexact(ctx):
    rng = np.random.default_rng(91)
    rows, cols = 29, 1024
    raw = raw_q5k(rng, rows, cols)
    w = ssdllm.Weight.upload(ctx, raw, Q5_K, rows, cols)
    try:
        assert np.array_equal(w.download().reshape(raw.shape), raw)
        out = torch.zeros(rows * cols, device=DEV)
        ssdllm.dequantize(ctx, w, out)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), ora.dequantize(raw, Q5_K, rows * cols))
    finally:
        w.free()


CASES = [(1, 256), (9, 768), (300, 4096), (4096, 4096), (777, 11008 // 256 * 256)]


@pytest.mark.parametrize("rows,cols", CASES)
def test_matvec_matches_oracle(ctx, rows, cols):
    rng = np.random.default_rng(rows * 17 + cols)
    raw = raw_q5k(rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    w = ssdllm.Weight.upload(ctx, raw, Q5_K, rows, cols)
    try:
        y = torch.zeros(rows, device=DEV)
        ssdllm.matvec(ctx, w, d(x), y)
        torch.cuda.synchronize()
    finally:
        w.free()
    ref = ora.matvec_quantized(raw, x, rows, cols, Q5_K, threads=8)
    exact = ora.dequantize(raw, Q5_K, rows * cols).reshape(rows, cols).astype(np.float64) @ \
        x.astype(np.float64)
    got = y.cpu().numpy()
    assert parity(got, ref, exact), (rel_err(got, ref), rel_err(ref, exact), rel_err(got, exact))


def test_swiglu_and_residual(ctx):
    rng = np.random.default_rng(92)
    E, F = 1024, 2048
    wg_raw, wu_raw, wd_raw = raw_q5k(rng, F, E), raw_q5k(rng, F, E), raw_q5k(rng, E, F)
    G, U = (ssdllm.Weight.upload(ctx, a, Q5_K, F, E) for a in (wg_raw, wu_raw))
    D = ssdllm.Weight.upload(ctx, wd_raw, Q5_K, E, F)
    x = rng.standard_normal(E).astype(np.float32)
    nw = (rng.random(E) + 0.5).astype(np.float32)
    base = rng.standard_normal(E).astype(np.float32)
    try:
        act = torch.zeros(F, device=DEV)
        ssdllm.fused_swiglu(ctx, G, U, d(x), d(nw), 1e-5, act)
        y = torch.zeros(E, device=DEV)
        ssdllm.matvec_residual(ctx, D, act, d(base), y)
        torch.cuda.synchronize()
    finally:
        for t in (G, U, D):
            t.free()
    _, xn = ora.fused_post_attn_norm(x, np.zeros(E, np.float32), nw, 1e-5)
    ref_act = ora.silu(ora.matvec_quantized(wg_raw, xn, F, E, Q5_K)) * \
        ora.matvec_quantized(wu_raw, xn, F, E, Q5_K)
    got_act = act.cpu().numpy()
    assert rel_err(got_act, ref_act) <= TOL
    ref_y = base + ora.matvec_quantized(wd_raw, got_act, E, F, Q5_K)
    assert rel_err(y.cpu().numpy(), ref_y) <= TOL
