"""GPU parity of the three matvec kernels: the tcgen05 integer tensor-core kernel
(matvec_i8.cu, covering cols % 256 == 0; opt-in with SSD_MV_IMPL=i8), the mma.sync
integer tensor-core kernel (matvec_tc.cu, covering cols % 256 == 0, cols >= 2048; opt-in
with SSD_MV_IMPL=tc) and the FMA kernel (matvec.cu, every shape), each forced in turn
with SSD_MV_IMPL=i8 / tc / fma, which the library reads on each call.

Both are checked against the oracle's matvec_quantized (src/metal/compute.rs:680-750,
:904-925) on shapes that exercise the tensor-core kernel's own structure: ragged row
counts (half 16-row tiles, rows past the end), one-unit CTAs, partial last K stages,
wide rows (a shallower TMA stage ring), and x vectors whose 32-element chunks span
very different magnitudes (the per-chunk fixed-point exponent), including all-zero
chunks and chunks whose small elements sit 2^-40 below the chunk maximum. The fused
epilogues (residual, RMSNorm, QKV + RoPE, SwiGLU) run under both kernels too.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from _util import normwise, parity, rel_err  # noqa: E402

TOL = 1e-3
DEV = "cuda:0"
IMPLS = ["i8", "tc", "fma"]


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


@pytest.fixture(params=IMPLS)
def impl(request, monkeypatch):
    monkeypatch.setenv("SSD_MV_IMPL", request.param)
    return request.param


def d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def randw(rng, rows, cols, std=0.02):
    return (rng.standard_normal((rows, cols)) * std).astype(np.float32)


def wild_x(rng, cols):
    """Chunks of 32 with scales from 1e-30 to 1e6, all-zero chunks, and chunks whose
    elements span 2^40 around their maximum."""
    x = rng.standard_normal(cols).astype(np.float32)
    nc = cols // 32
    scales = np.array([1.0, 1e6, 1e-30, 0.0, 3e-3, 1.0, 7.5, 1e-8], np.float32)
    for c in range(nc):
        x[32 * c:32 * c + 32] *= scales[c % len(scales)]
        if c % 5 == 4:  # one large element, the rest far below it
            x[32 * c:32 * c + 32] *= np.float32(2.0 ** -40)
            x[32 * c + (c % 32)] = np.float32(3.0)
    return x


def check_matvec(ctx, wtype, rows, cols, x, seed):
    rng = np.random.default_rng(seed)
    raw = ora.quantize(randw(rng, rows, cols), wtype)
    w = ssdllm.Weight.upload(ctx, raw, wtype, rows, cols)
    y = torch.full((rows,), float("nan"), device=DEV)
    ssdllm.matvec(ctx, w, d(x), y)
    torch.cuda.synchronize()
    ref = ora.matvec_quantized(raw, x, rows, cols, wtype, threads=8)
    exact = ora.dequantize(raw, wtype, rows * cols).reshape(rows, cols).astype(np.float64) @ \
        x.astype(np.float64)
    got = y.cpu().numpy()
    assert np.all(np.isfinite(got))
    assert parity(got, ref, exact), (rel_err(got, ref), rel_err(ref, exact), rel_err(got, exact))
    return got


TC_SHAPES = [
    (ora.Q4_0, 37, 2048),    # 5 units: a half tile, rows past the end
    (ora.Q4_0, 9, 2048),     # two CTAs of one unit (half tiles)
    (ora.Q4_0, 300, 4096),   # fewer units than SMs
    (ora.Q4_0, 2000, 2304),  # several tiles per CTA; last K stage of 8 chunks (2 warps)
    (ora.Q4_0, 1000, 28672),  # wide rows: 112 KB of x, a shallower stage ring
    (ora.Q4_0, 100, 1056),   # not covered by the tensor-core kernel: the FMA kernel
    (ora.Q8_0, 9, 2048),
    (ora.Q8_0, 1200, 2560),  # last K stage of 16 chunks
    (ora.Q4_K, 21, 2048),
    (ora.Q4_K, 3000, 2304),
]


@pytest.mark.parametrize("wtype,rows,cols", TC_SHAPES)
def test_matvec_both_kernels_match_oracle(ctx, impl, wtype, rows, cols):
    rng = np.random.default_rng(rows + cols)
    x = rng.standard_normal(cols).astype(np.float32)
    check_matvec(ctx, wtype, rows, cols, x, seed=rows * 3 + cols)


@pytest.mark.parametrize("wtype", [ora.Q4_0, ora.Q8_0, ora.Q4_K])
def test_matvec_wide_dynamic_range_chunks(ctx, impl, wtype):
    rng = np.random.default_rng(int(wtype))
    rows, cols = 700, 2048
    check_matvec(ctx, wtype, rows, cols, wild_x(rng, cols), seed=11)


@pytest.mark.parametrize("tc_impl", ["i8", "tc"])
def test_tensor_core_kernel_is_deterministic_and_close_to_fma(ctx, monkeypatch, tc_impl):
    """Both tensor-core kernels add their partial sums in a fixed order (the tcgen05 kernel
    across CTAs of a split tile too), so two calls give identical bits."""
    rng = np.random.default_rng(3)
    rows, cols = 8192, 4096
    raw = ora.quantize(randw(rng, rows, cols), ora.Q4_0)
    w = ssdllm.Weight.upload(ctx, raw, ora.Q4_0, rows, cols)
    x = d(rng.standard_normal(cols).astype(np.float32))
    ys = []
    for env in (tc_impl, tc_impl, "fma"):
        monkeypatch.setenv("SSD_MV_IMPL", env)
        y = torch.zeros(rows, device=DEV)
        ssdllm.matvec(ctx, w, x, y)
        torch.cuda.synchronize()
        ys.append(y.cpu().numpy())
    assert np.array_equal(ys[0], ys[1])  # fixed summation order
    assert normwise(ys[0], ys[2]) <= 1e-5  # two fp32 summation orders


def test_fused_epilogues_both_kernels(ctx, impl):
    rng = np.random.default_rng(21)
    E, nh, nkv, hd, pos, theta = 2048, 16, 4, 128, 777, 5e5
    x = rng.standard_normal(E).astype(np.float32)
    nw = (rng.random(E) + 0.5).astype(np.float32)
    # residual + fused RMSNorm matvec
    rows = 2048
    raw = ora.quantize(randw(rng, rows, E), ora.Q4_0)
    w = ssdllm.Weight.upload(ctx, raw, ora.Q4_0, rows, E)
    base = rng.standard_normal(rows).astype(np.float32)
    y = torch.zeros(rows, device=DEV)
    ssdllm.matvec_residual(ctx, w, d(x), d(base), y)
    y2 = torch.zeros(rows, device=DEV)
    ssdllm.fused_rmsnorm_matvec(ctx, w, d(x), d(nw), 1e-5, y2)
    # QKV + RoPE
    wq, wk, wv = (ora.quantize(randw(rng, r, E), ora.Q4_0) for r in (nh * hd, nkv * hd, nkv * hd))
    W = [ssdllm.Weight.upload(ctx, a, ora.Q4_0, a.shape[0], E) for a in (wq, wk, wv)]
    q = torch.zeros(nh * hd, device=DEV)
    k = torch.zeros(nkv * hd, device=DEV)
    v = torch.zeros(nkv * hd, device=DEV)
    ssdllm.fused_qkv_rope(ctx, *W, d(x), d(nw), 1e-5, hd, pos, theta, q, k, v)
    # SwiGLU (gate/up row pairs)
    F = 5632
    wg, wu = (ora.quantize(randw(rng, F, E), ora.Q4_0) for _ in range(2))
    G, U = (ssdllm.Weight.upload(ctx, a, ora.Q4_0, F, E) for a in (wg, wu))
    act = torch.zeros(F, device=DEV)
    ssdllm.fused_swiglu(ctx, G, U, d(x), d(nw), 1e-5, act)
    torch.cuda.synchronize()

    mv = ora.matvec_quantized(raw, x, rows, E, ora.Q4_0)
    assert rel_err(y.cpu().numpy(), base + mv) <= TOL
    ref2 = ora.fused_rmsnorm_linear(x, nw, ora.dequantize(raw, ora.Q4_0, rows * E), rows, E)
    assert rel_err(y2.cpu().numpy(), ref2) <= TOL
    xn = ora.rmsnorm(x, nw, 1e-5)
    rq = ora.rope_multi_head(ora.matvec_quantized(wq, xn, nh * hd, E, ora.Q4_0), hd, nh, pos, theta)
    rk = ora.rope_multi_head(ora.matvec_quantized(wk, xn, nkv * hd, E, ora.Q4_0), hd, nkv, pos,
                             theta)
    rv = ora.matvec_quantized(wv, xn, nkv * hd, E, ora.Q4_0)
    assert rel_err(q.cpu().numpy(), rq) <= TOL
    assert rel_err(k.cpu().numpy(), rk) <= TOL
    assert rel_err(v.cpu().numpy(), rv) <= TOL
    _, xf = ora.fused_post_attn_norm(x, np.zeros(E, np.float32), nw, 1e-5)
    ref = ora.silu(ora.matvec_quantized(wg, xf, F, E, ora.Q4_0)) * \
        ora.matvec_quantized(wu, xf, F, E, ora.Q4_0)
    assert rel_err(act.cpu().numpy(), ref) <= TOL
