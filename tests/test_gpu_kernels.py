"""GPU parity tests: the CUDA kernels through the C ABI vs the CPU oracle.

Bars: bit-exact for quantization, dequantization and the INT8 KV quantizer;
max relative error <= 1e-3 (floor 1e-3*||r||_inf, see _util.rel_err) for the
fp32-accumulated matvecs, norms and attention."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from _util import parity, rel_err  # noqa: E402

TOL = 1e-3
DEV = "cuda:0"


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


def d(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def randw(rng, rows, cols, std=0.02):
    return (rng.standard_normal((rows, cols)) * std).astype(np.float32)


def edge_rows(cols):
    """Rows with the blocks the quantizers treat specially."""
    e = np.zeros((4, cols), np.float32)
    e[1, :] = np.linspace(-1, 1, cols, dtype=np.float32)
    e[2, :] = -3.0
    e[2, 5] = 5.0
    e[3, :] = 1e-6
    return e


# ---------------------------------------------------------------- quantize
@pytest.mark.parametrize("wtype,cols", [(ora.Q4_0, 128), (ora.Q8_0, 96), (ora.Q4_K, 512)])
def test_device_quantizer_matches_oracle_bitwise(ctx, wtype, cols):
    rng = np.random.default_rng(1)
    w = np.concatenate([randw(rng, 60, cols), edge_rows(cols),
                        (rng.standard_normal((4, cols)) * 3).astype(np.float32)])
    ref = ora.quantize(w, wtype)
    out = torch.zeros(ref.size, dtype=torch.uint8, device=DEV)
    ssdllm.quantize(ctx, d(w), wtype, out)
    torch.cuda.synchronize()
    got, exp = out.cpu().numpy(), ref.reshape(-1)
    bad = np.nonzero(got != exp)[0]
    assert bad.size == 0, (bad[:16], got[bad[:8]], exp[bad[:8]])


@pytest.mark.parametrize("wtype", [ora.Q4_0, ora.Q8_0, ora.Q4_K])
def test_synthetic_weights_equal_quantized_synthetic_values(ctx, wtype):
    """ssd_weight_synth == oracle quantizer applied to ssd_synth_f32's values."""
    rows, total_cols, col0, cols = 8, 1024, 256, 512
    vals = torch.zeros(rows, cols, device=DEV)
    ssdllm.synth_f32(ctx, 42, 7, 0.0, 0.02, total_cols, 3, rows, col0, cols, vals)
    w = ssdllm.Weight.synth(ctx, wtype, 42, 7, 0.02, total_cols, 3, rows, col0, cols)
    torch.cuda.synchronize()
    ref = ora.quantize(vals.cpu().numpy(), wtype)
    assert np.array_equal(w.download(), ref.reshape(-1))
    v = vals.cpu().numpy()
    assert abs(v.std() - 0.02) < 0.004 and abs(v.mean()) < 0.004


# ---------------------------------------------------------------- dequant
@pytest.mark.parametrize("wtype,rows,cols", [(ora.Q4_0, 37, 256), (ora.Q8_0, 19, 96),
                                             (ora.Q4_K, 9, 768)])
def test_weight_round_trip_and_dequant_bit_exact(ctx, wtype, rows, cols):
    rng = np.random.default_rng(2)
    raw = ora.quantize(np.concatenate([randw(rng, rows - 4, cols), edge_rows(cols)]), wtype)
    w = ssdllm.Weight.upload(ctx, raw, wtype, rows, cols)
    assert np.array_equal(w.download(), raw.reshape(-1))
    out = torch.zeros(rows * cols, device=DEV)
    ssdllm.dequantize(ctx, w, out)
    torch.cuda.synchronize()
    ref = ora.dequantize(raw, wtype, rows * cols)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


# ---------------------------------------------------------------- matvec
MATVEC_CASES = [
    (ora.Q4_0, 4096, 4096),   # benchmark config 0
    (ora.Q8_0, 11008, 4096),  # config 1 (gate/up)
    (ora.Q8_0, 4096, 11008),  # config 1 (down)
    (ora.Q4_K, 11008, 4096),
    (ora.Q4_K, 4096, 11008),
    (ora.Q4_0, 1, 32),        # one block
    (ora.Q4_0, 33, 96),       # ragged rows, 3 chunks
    (ora.Q8_0, 7, 1056),      # 33 chunks: ragged lane iterations
    (ora.Q4_K, 5, 256),
    (ora.Q4_0, 8192, 28672),  # 70B down_proj width (112 KB of x in shared memory)
]


@pytest.mark.parametrize("wtype,rows,cols", MATVEC_CASES)
def test_matvec_matches_oracle(ctx, wtype, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    raw = ora.quantize(randw(rng, rows, cols), wtype)
    x = rng.standard_normal(cols).astype(np.float32)
    w = ssdllm.Weight.upload(ctx, raw, wtype, rows, cols)
    y = torch.zeros(rows, device=DEV)
    ssdllm.matvec(ctx, w, d(x), y)
    torch.cuda.synchronize()
    ref = ora.matvec_quantized(raw, x, rows, cols, wtype, threads=8)
    exact = ora.dequantize(raw, wtype, rows * cols).reshape(rows, cols).astype(np.float64) @ \
        x.astype(np.float64)
    got = y.cpu().numpy()
    assert parity(got, ref, exact), (rel_err(got, ref), rel_err(ref, exact), rel_err(got, exact))


@pytest.mark.parametrize("wtype,rows,cols", [(ora.Q4_0, 4096, 4096), (ora.Q8_0, 1000, 2048),
                                               (ora.Q4_K, 513, 1024)])
def test_independent_matvecs_equal_ssd_matvec(ctx, wtype, rows, cols):
    """ssd_matvec_independent: a series of launches that do not wait for each other gives
    ssd_matvec's results bit for bit, and a dependent launch after the series sees every
    one of them complete (each independent launch waits for its predecessor at its end)."""
    rng = np.random.default_rng(rows + cols)
    raws = [ora.quantize(randw(rng, rows, cols), wtype) for _ in range(6)]
    ws = [ssdllm.Weight.upload(ctx, r, wtype, rows, cols) for r in raws]
    x = d(rng.standard_normal(cols).astype(np.float32))
    ref = []
    for w in ws:
        y = torch.zeros(rows, device=DEV)
        ssdllm.matvec(ctx, w, x, y)
        ref.append(y)
    torch.cuda.synchronize()
    ctx.set_pdl(True)
    try:
        ys = [torch.full((rows,), float("nan"), device=DEV) for _ in ws]
        for w, y in zip(ws, ys):
            ssdllm.matvec_independent(ctx, w, x, y)
        # dependent: out = W0 x + ys[0], launched right after the series (PDL on)
        out = torch.zeros(rows, device=DEV)
        ssdllm.matvec_residual(ctx, ws[0], x, ys[0], out)
        torch.cuda.synchronize()
    finally:
        ctx.set_pdl(False)
    for y, r in zip(ys, ref):
        assert torch.equal(y, r)
    assert torch.allclose(out, ref[0] + ref[0], rtol=0, atol=0) or \
        rel_err(out.cpu().numpy(), (ref[0] + ref[0]).cpu().numpy()) <= 1e-6
    for w in ws:
        w.free()


def test_matvec_residual_and_fused_norm(ctx):
    rng = np.random.default_rng(3)
    rows, cols = 1000, 2048
    raw = ora.quantize(randw(rng, rows, cols), ora.Q4_0)
    w = ssdllm.Weight.upload(ctx, raw, ora.Q4_0, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    base = rng.standard_normal(rows).astype(np.float32)
    y = torch.zeros(rows, device=DEV)
    ssdllm.matvec_residual(ctx, w, d(x), d(base), y)
    nw = (rng.random(cols) + 0.5).astype(np.float32)
    y2 = torch.zeros(rows, device=DEV)
    ssdllm.fused_rmsnorm_matvec(ctx, w, d(x), d(nw), 1e-5, y2)
    torch.cuda.synchronize()
    mv = ora.matvec_quantized(raw, x, rows, cols, ora.Q4_0)
    assert rel_err(y.cpu().numpy(), base + mv) <= TOL
    # fused_rmsnorm_linear_f32_cpu (compute.rs:557-577) with the dequantized weight
    ref = ora.fused_rmsnorm_linear(x, nw, ora.dequantize(raw, ora.Q4_0, rows * cols), rows, cols)
    assert rel_err(y2.cpu().numpy(), ref) <= TOL


def test_host_slice_matvec_quantized_kats():
    """MetalCompute::matvec_quantized semantics through the host-slice entry point,
    on the reference's own known answers (compute.rs:2347-2381)."""
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    cc = ssdllm.CudaCompute.new(0)
    h = ora.lib().ora_f32_to_f16(1.0)
    q4 = np.array([h & 0xFF, h >> 8] + [0x88] * 16, np.uint8)
    assert abs(cc.matvec_quantized(q4, np.ones(32, np.float32), 1, 32, ora.Q4_0)[0]) < 1e-5
    q8 = np.array([h & 0xFF, h >> 8] + [1] * 32, np.uint8)
    assert abs(cc.matvec_quantized(q8, np.ones(32, np.float32), 1, 32, ora.Q8_0)[0] - 32) < 1e-3
    with pytest.raises(ssdllm.SsdError) as e:  # no silent zeros for unknown types
        cc.matvec_quantized(q4, np.ones(32, np.float32), 1, 32, 99)
    assert e.value.status == 2


def test_shape_errors_are_reported(ctx):
    raw = np.zeros(18, np.uint8)
    with pytest.raises(ssdllm.SsdError) as e:
        ssdllm.Weight.upload(ctx, raw, ora.Q4_0, 1, 48)  # not a block multiple
    assert e.value.status == 3
    with pytest.raises(ssdllm.SsdError):
        ssdllm.Weight.upload(ctx, raw, ora.Q4_K, 1, 32)


# ------------------------------------------------------------ fused matvecs
def test_fused_qkv_rope_matches_oracle(ctx):
    rng = np.random.default_rng(4)
    E, nh, nkv, hd, pos, theta = 1024, 8, 2, 128, 1234, 5e5
    wq, wk, wv = (ora.quantize(randw(rng, r, E), ora.Q4_0) for r in (nh * hd, nkv * hd, nkv * hd))
    W = [ssdllm.Weight.upload(ctx, a, ora.Q4_0, a.shape[0], E) for a in (wq, wk, wv)]
    x = rng.standard_normal(E).astype(np.float32)
    nw = (rng.random(E) + 0.5).astype(np.float32)
    q = torch.zeros(nh * hd, device=DEV)
    k = torch.zeros(nkv * hd, device=DEV)
    v = torch.zeros(nkv * hd, device=DEV)
    ssdllm.fused_qkv_rope(ctx, *W, d(x), d(nw), 1e-5, hd, pos, theta, q, k, v)
    torch.cuda.synchronize()
    xn = ora.rmsnorm(x, nw, 1e-5)
    rq = ora.rope_multi_head(ora.matvec_quantized(wq, xn, nh * hd, E, ora.Q4_0), hd, nh, pos, theta)
    rk = ora.rope_multi_head(ora.matvec_quantized(wk, xn, nkv * hd, E, ora.Q4_0), hd, nkv, pos,
                             theta)
    rv = ora.matvec_quantized(wv, xn, nkv * hd, E, ora.Q4_0)
    assert rel_err(q.cpu().numpy(), rq) <= TOL
    assert rel_err(k.cpu().numpy(), rk) <= TOL
    assert rel_err(v.cpu().numpy(), rv) <= TOL


@pytest.mark.parametrize("wtype", [ora.Q4_0, ora.Q4_K])
def test_fused_swiglu_matches_oracle(ctx, wtype):
    rng = np.random.default_rng(5)
    E, F = 1024, 2816
    wg, wu = (ora.quantize(randw(rng, F, E), wtype) for _ in range(2))
    G, U = (ssdllm.Weight.upload(ctx, a, wtype, F, E) for a in (wg, wu))
    x = rng.standard_normal(E).astype(np.float32)
    nw = (rng.random(E) + 0.5).astype(np.float32)
    act = torch.zeros(F, device=DEV)
    ssdllm.fused_swiglu(ctx, G, U, d(x), d(nw), 1e-5, act)
    torch.cuda.synchronize()
    _, xn = ora.fused_post_attn_norm(x, np.zeros(E, np.float32), nw, 1e-5)
    ref = ora.silu(ora.matvec_quantized(wg, xn, F, E, wtype)) * \
        ora.matvec_quantized(wu, xn, F, E, wtype)
    assert rel_err(act.cpu().numpy(), ref) <= TOL


# ------------------------------------------------------------ elementwise ops
@pytest.mark.parametrize("n", [1, 4, 4096, 8192, 5000])
def test_rmsnorm_and_post_attn_norm(ctx, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    a = rng.standard_normal(n).astype(np.float32)
    w = (rng.random(n) + 0.5).astype(np.float32)
    xd = d(x)
    ssdllm.rmsnorm(ctx, xd, d(w), 1e-5)
    hd, out = d(x), torch.zeros(n, device=DEV)
    ssdllm.fused_post_attn_norm(ctx, hd, d(a), d(w), 1e-5, out)
    torch.cuda.synchronize()
    assert rel_err(xd.cpu().numpy(), ora.rmsnorm(x, w)) <= 1e-5
    h2, o2 = ora.fused_post_attn_norm(x, a, w)
    assert np.array_equal(hd.cpu().numpy(), h2)  # the residual add is a single rounding
    assert rel_err(out.cpu().numpy(), o2) <= 1e-5


@pytest.mark.parametrize("n", [1, 3, 2049, 128256])
def test_softmax_silu(ctx, n):
    rng = np.random.default_rng(n + 1)
    x = (rng.standard_normal(n) * 4).astype(np.float32)
    xd = d(x)
    ssdllm.softmax(ctx, xd)
    sd = d(x)
    ssdllm.silu(ctx, sd)
    torch.cuda.synchronize()
    assert rel_err(xd.cpu().numpy(), ora.softmax(x)) <= TOL
    assert rel_err(sd.cpu().numpy(), ora.silu(x)) <= 1e-5


@pytest.mark.parametrize("pos,theta", [(0, 1e4), (7, 1e4), (2048, 1e4), (4095, 5e5)])
def test_rope(ctx, pos, theta):
    rng = np.random.default_rng(pos)
    hd, nh = 128, 8
    x = rng.standard_normal(hd * nh).astype(np.float32)
    xd = d(x)
    ssdllm.rope(ctx, xd, hd, nh, pos, theta)
    torch.cuda.synchronize()
    assert rel_err(xd.cpu().numpy(), ora.rope_multi_head(x, hd, nh, pos, theta)) <= 1e-5


def test_argmax_last_index_on_ties(ctx):
    v = np.array([0.5, 2.0, -1.0, 2.0, 1.0, 2.0, 0.0], np.float32)
    idx = torch.zeros(1, dtype=torch.int32, device=DEV)
    ssdllm.argmax(ctx, d(v), idx)
    torch.cuda.synchronize()
    assert int(idx.item()) == ora.argmax(v) == 5
    big = np.random.default_rng(0).standard_normal(128256).astype(np.float32)
    big[100] = big[128000] = big.max() + 1
    ssdllm.argmax(ctx, d(big), idx)
    torch.cuda.synchronize()
    assert int(idx.item()) == ora.argmax(big) == 128000
    neg = np.full(10, -3.0, np.float32)
    ssdllm.argmax(ctx, d(neg), idx)
    torch.cuda.synchronize()
    assert int(idx.item()) == 9


# ------------------------------------------------------------ INT8 KV + attention
def test_kv_append_bit_exact(ctx):
    rng = np.random.default_rng(6)
    kvd, n = 1024, 40
    k = rng.standard_normal((n, kvd)).astype(np.float32)
    v = (rng.standard_normal((n, kvd)) * 10).astype(np.float32)
    k[3] = 0.0  # zero row -> scale 0 (quantized_kv_cache.rs:26-31)
    v[5, :] = 0.0
    v[5, 7] = -2.5
    kv = ssdllm.KvCache(ctx, 64, 8, 128)
    kv.append_rows(d(k[:n - 1]), d(v[:n - 1]), 0)
    kv.append(d(k[n - 1]), d(v[n - 1]), n - 1)
    torch.cuda.synchronize()
    kp, vp, ksp, vsp = kv.pointers()
    got = {}
    for name, ptr, dt in (("k", kp, np.int8), ("v", vp, np.int8)):
        a = np.zeros((n, kvd), dt)
        ssdllm.copy_to_host(ctx, a, ptr)
        got[name] = a
    for name, ptr in (("ks", ksp), ("vs", vsp)):
        a = np.zeros(n, np.float32)
        ssdllm.copy_to_host(ctx, a, ptr)
        got[name] = a
    rk, rks = ora.kv_quantize_rows(k)
    rv, rvs = ora.kv_quantize_rows(v)
    assert np.array_equal(got["k"], rk) and np.array_equal(got["v"], rv)
    assert np.array_equal(got["ks"].view(np.uint32), rks.view(np.uint32))
    assert np.array_equal(got["vs"].view(np.uint32), rvs.view(np.uint32))
    with pytest.raises(ssdllm.SsdError):
        kv.append(d(k[0]), d(v[0]), 64)  # beyond capacity
    kv.free()


@pytest.mark.parametrize("n_head,n_kv,hd,seq", [(8, 8, 128, 1), (8, 8, 128, 37),
                                                (8, 2, 128, 129), (16, 2, 64, 300),
                                                (32, 32, 128, 2049), (64, 8, 128, 4096)])
def test_attention_int8_matches_oracle(ctx, n_head, n_kv, hd, seq):
    rng = np.random.default_rng(seq + n_head)
    kvd = n_kv * hd
    kf = rng.standard_normal((seq, kvd)).astype(np.float32)
    vf = rng.standard_normal((seq, kvd)).astype(np.float32)
    q = rng.standard_normal(n_head * hd).astype(np.float32)
    kv = ssdllm.KvCache(ctx, seq, n_kv, hd)
    kv.append_rows(d(kf), d(vf), 0)
    out = torch.zeros(n_head * hd, device=DEV)
    kv.attention(d(q), n_head, seq, out)
    torch.cuda.synchronize()
    k, ks = ora.kv_quantize_rows(kf)
    v, vs = ora.kv_quantize_rows(vf)
    ref = ora.attention_int8(q, k, ks, v, vs, seq, n_head, n_kv, hd)
    exact = attention_fp64(q, k, ks, v, vs, n_head, n_kv, hd)
    got = out.cpu().numpy()
    assert parity(got, ref, exact), (rel_err(got, ref), rel_err(ref, exact), rel_err(got, exact))
    kv.free()


def attention_fp64(q, k, ks, v, vs, n_head, n_kv, hd):
    """fp64 arbiter: the reference's fp32-dequantized K/V rows (key_at / value_at,
    src/inference/quantized_kv_cache.rs:118-130), everything after in float64."""
    kd = (k.astype(np.float32) * ks[:, None]).astype(np.float64)
    vd = (v.astype(np.float32) * vs[:, None]).astype(np.float64)
    g = n_head // n_kv
    out = np.zeros(n_head * hd)
    for h in range(n_head):
        c = (h // g) * hd
        sc = kd[:, c:c + hd] @ q[h * hd:(h + 1) * hd].astype(np.float64) / np.sqrt(hd)
        p = np.exp(sc - sc.max())
        out[h * hd:(h + 1) * hd] = (p / p.sum()) @ vd[:, c:c + hd]
    return out
