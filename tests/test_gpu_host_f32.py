"""The host-slice f32 operators of MetalCompute (src/metal/compute.rs:145-375) and
MetalGpu::feed_forward_f32 (src/metal/gpu.rs:789-838) on the GPU, through the C entry
points a Rust binding calls (CudaCompute: copy in, compute, copy out):

* the reference's own known-answer tests with their inputs and tolerances
  (compute.rs:2292-2310, 3112-3163, 3300-3338, 3399-3530; feed_forward.rs:76-130;
  flash_attention.rs:414-522);
* random inputs against the oracle at rel. error 1e-3 (fp64 arbiter), including windowed,
  GQA, empty-window, long (split) and odd-head_dim attention;
* F32 weights uploaded once (ssd_weight_upload) through the device matvec and the dense
  SwiGLU pair kernel."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from _util import parity, rel_err  # noqa: E402
from test_oracle_f32ops import attn64, ffn64  # noqa: E402

DEV = "cuda:0"


@pytest.fixture(scope="module")
def cc():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.CudaCompute.new(0)


# ------------------------------------------------------------- reference KATs
def test_matvec_kats(cc):
    """compute.rs:2292-2310."""
    y = cc.matvec_f32([1.0, 0.0, 0.0, 1.0], [3.0, 4.0], 2, 2)
    assert abs(y[0] - 3.0) < 1e-6 and abs(y[1] - 4.0) < 1e-6
    y = cc.matvec_f32([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], [1.0, 1.0], 3, 2)
    assert np.all(np.abs(y - [3.0, 7.0, 11.0]) < 1e-6)


def test_fused_qkv_kats(cc):
    """compute.rs:3112-3163."""
    wq = [1.0, 0.0, 0.0, 0.0, 1.0, 0.0]
    wk = [0.0, 1.0, 0.0, 0.0, 0.0, 1.0]
    wv = [1.0, 1.0, 0.0, 0.0, 1.0, 1.0]
    q, k, v = cc.fused_qkv_f32(wq, wk, wv, [2.0, 3.0, 5.0], 2, 2, 3)
    assert np.all(np.abs(q - [2, 3]) < 1e-6) and np.all(np.abs(k - [3, 5]) < 1e-6)
    assert np.all(np.abs(v - [5, 8]) < 1e-6)
    n_embd, q_dim, kv_dim = 16, 8, 4
    wq = (np.arange(q_dim * n_embd) % 11) * 0.1 - 0.5
    wk = (np.arange(kv_dim * n_embd) % 7) * 0.15 - 0.3
    wv = (np.arange(kv_dim * n_embd) % 13) * 0.08 - 0.4
    x = (np.arange(n_embd) % 5) * 0.3 - 0.6
    q, k, v = cc.fused_qkv_f32(wq, wk, wv, x, q_dim, kv_dim, n_embd)
    for w, y, n in ((wq, q, q_dim), (wk, k, kv_dim), (wv, v, kv_dim)):
        sep = ora.matvec_f32(np.asarray(w, np.float32).reshape(n, n_embd), x)
        assert np.all(np.abs(sep - y) < 1e-4)


def test_fused_qkv_rope_kats(cc):
    """compute.rs:3300-3338: position 0 is the identity; q == k == v == the plain matvec."""
    x = np.ones(4, np.float32)
    w = np.full(16, 0.1, np.float32)
    q, k, v = cc.fused_qkv_rope_f32(w, w, w, x, 4, 4, 4, 4, 0, 10000.0)
    plain = ora.matvec_f32(w.reshape(4, 4), x)
    for y in (q, k, v):
        assert np.all(np.abs(y - plain) < 1e-6)


def test_fused_rmsnorm_linear_kats(cc):
    """compute.rs:3399-3455."""
    n_embd, vocab = 8, 4
    x = ((np.arange(n_embd) + 1.0) * 0.1).astype(np.float32)
    nw = np.ones(n_embd, np.float32)
    ow = np.zeros((vocab, n_embd), np.float32)
    for r in range(vocab):
        ow[r, r] = 1.0
    logits = cc.fused_rmsnorm_linear_f32(x, nw, ow, vocab, n_embd)
    expect = ora.matvec_f32(ow, ora.rmsnorm(x, nw, 1e-5))
    assert logits.shape == (vocab,) and np.all(np.abs(logits - expect) < 1e-5)
    n_embd, vocab = 64, 32
    i = np.arange(n_embd)
    x = (((i * 7 + 3) % 13) * 0.1 - 0.5).astype(np.float32)
    nw = (0.5 + (i % 5) * 0.2).astype(np.float32)
    j = np.arange(vocab * n_embd)
    ow = (((j * 11 + 7) % 19) * 0.05 - 0.4).astype(np.float32)
    logits = cc.fused_rmsnorm_linear_f32(x, nw, ow, vocab, n_embd)
    sep = ora.matvec_f32(ow.reshape(vocab, n_embd), ora.rmsnorm(x, nw, 1e-5))
    assert np.all(np.abs(logits - sep) < 1e-4)


def test_fused_post_attn_norm_kats(cc):
    """compute.rs:3457-3530."""
    n = 64
    hidden = (np.arange(n) * 0.1).astype(np.float32)
    attn = ((n - np.arange(n)) * 0.05).astype(np.float32)
    w = (0.8 + (np.arange(n) % 3) * 0.1).astype(np.float32)
    ffn = cc.fused_post_attn_norm_f32(hidden, attn, w, 1e-5)
    expect_h = np.arange(n) * 0.1 + (n - np.arange(n)) * 0.05
    assert np.all(np.abs(hidden - expect_h) < 1e-6)
    inv = 1.0 / np.sqrt(np.sum(hidden.astype(np.float64) ** 2) / n + 1e-5)
    assert np.all(np.abs(ffn - hidden * inv * w) < 1e-5)
    n = 128
    i = np.arange(n)
    h0 = (((i * 7 + 3) % 13) * 0.1 - 0.5).astype(np.float32)
    attn = (((i * 11 + 5) % 17) * 0.08 - 0.3).astype(np.float32)
    w = (0.5 + (i % 5) * 0.2).astype(np.float32)
    hf = h0.copy()
    ffn = cc.fused_post_attn_norm_f32(hf, attn, w, 1e-5)
    hs = h0 + attn
    assert np.all(np.abs(hf - hs) < 1e-6)
    assert np.all(np.abs(ffn - ora.rmsnorm(hs, w, 1e-5)) < 1e-5)


def test_rmsnorm_and_softmax_in_place(cc):
    """compute.rs:193-215 against the oracle; softmax of nothing is a no-op."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal(4096).astype(np.float32)
    w = (rng.random(4096) + 0.5).astype(np.float32)
    ref = ora.rmsnorm(x, w, 1e-5)
    cc.rmsnorm_f32(x, w, 1e-5)
    assert rel_err(x, ref) <= 1e-5
    s = np.array([1.0, 2.0, 3.0], np.float32)
    cc.softmax_f32(s)
    assert abs(s.sum() - 1.0) < 1e-6 and s[2] > s[1] > s[0]
    cc.softmax_f32(np.zeros(0, np.float32))


def test_feed_forward_kats(cc):
    """feed_forward.rs:76-130 (the shapes case and the GPU-vs-CPU case) and n_ff == 0."""
    out = cc.feed_forward_f32(np.ones(4), np.full(32, 0.1), np.full(32, 0.1), np.full(32, 0.1), 4)
    assert np.allclose(out, ora.feed_forward_f32(np.ones(4), np.full(32, 0.1), np.full(32, 0.1),
                                                 np.full(32, 0.1), 4, 8), rtol=1e-5)
    n_embd, n_ff = 64, 2048
    x = (np.arange(n_embd) * 0.01).astype(np.float32)
    i = np.arange(n_ff * n_embd)
    wg = (((i % 17) - 8.0) * 0.001).astype(np.float32)
    wu = (((i % 13) - 6.0) * 0.001).astype(np.float32)
    wd = (((np.arange(n_embd * n_ff) % 11) - 5.0) * 0.001).astype(np.float32)
    out = cc.feed_forward_f32(x, wg, wu, wd, n_embd)
    ref = ora.feed_forward_f32(x, wg, wu, wd, n_embd, n_ff)
    assert parity(out, ref, ffn64(x, wg, wu, wd, n_embd, n_ff))
    assert np.all(cc.feed_forward_f32(np.ones(4), [], [], [], 4) == 0)


def test_flash_attention_reference_cases(cc):
    """flash_attention.rs:414-522: one position returns its V row; the windowed case
    (10 positions, window 5..11) is finite and matches the oracle."""
    rng = np.random.default_rng(5)
    q = rng.standard_normal(8).astype(np.float32)
    k = rng.standard_normal((1, 8)).astype(np.float32)
    v = rng.standard_normal((1, 8)).astype(np.float32)
    assert np.allclose(cc.flash_attention_f32(q, k, v, 2, 2, 4, 1, 0, 1), v.ravel(), atol=1e-6)
    k = rng.standard_normal((10, 8)).astype(np.float32)
    v = rng.standard_normal((10, 8)).astype(np.float32)
    out = cc.flash_attention_f32(q, k, v, 2, 2, 4, 10, 5, 11)
    assert np.all(np.isfinite(out))
    assert rel_err(out, ora.flash_attention_f32(q, k, v, 2, 2, 4, 10, 5, 11)) <= 1e-5


# ------------------------------------------------------------- random vs oracle
@pytest.mark.parametrize("nh,nkv,hd,seq,ws,we", [
    (32, 8, 128, 1, 0, 1), (32, 8, 128, 4096, 0, 4096), (32, 8, 128, 4096, 1000, 3000),
    (8, 2, 64, 300, 17, 250), (4, 4, 80, 40, 0, 100), (2, 1, 256, 700, 5, 700),
    (64, 8, 128, 2048, 2000, 2048), (4, 1, 4, 3, 0, 3), (8, 8, 128, 64, 64, 64),
    (8, 8, 128, 64, 70, 90)])
def test_flash_attention_matches_oracle(cc, nh, nkv, hd, seq, ws, we):
    rng = np.random.default_rng(nh * 7919 + seq + ws)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal((seq, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((seq, nkv * hd)).astype(np.float32)
    out = cc.flash_attention_f32(q, k, v, nh, nkv, hd, seq, ws, we)
    ref = ora.flash_attention_f32(q, k, v, nh, nkv, hd, seq, ws, we)
    if min(we, seq) <= ws:
        assert np.all(out == 0) and np.all(ref == 0)
        return
    assert parity(out, ref, attn64(q, k, v, nh, nkv, hd, seq, ws, we)), rel_err(out, ref)


def test_flash_attention_device_entry_point(cc):
    """ssd_flash_attention_f32 on device pointers over a resident cache, window offset."""
    rng = np.random.default_rng(11)
    nh, nkv, hd, seq, ws, we = 32, 8, 128, 3000, 100, 2900
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal((seq, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((seq, nkv * hd)).astype(np.float32)
    qd, kd, vd = (torch.from_numpy(a).to(DEV) for a in (q, k, v))
    out = torch.zeros(nh * hd, device=DEV)
    ssdllm.check(ssdllm.lib().ssd_flash_attention_f32(
        cc.ctx.h, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), nh, nkv, hd, seq, ws, we,
        out.data_ptr(), torch.cuda.current_stream().cuda_stream))
    ref = ora.flash_attention_f32(q, k, v, nh, nkv, hd, seq, ws, we)
    assert parity(out.cpu().numpy(), ref, attn64(q, k, v, nh, nkv, hd, seq, ws, we))


def test_flash_attention_rejects_bad_shapes(cc):
    q = np.zeros(8, np.float32)
    with pytest.raises(ssdllm.SsdError) as e:
        cc.flash_attention_f32(q, q, q, 2, 3, 4, 1, 0, 1)  # n_head % n_head_kv != 0
    assert e.value.status == 3
    with pytest.raises(ssdllm.SsdError):
        cc.flash_attention_f32(np.zeros(600), np.zeros(600), np.zeros(600), 2, 2, 300, 1, 0, 1)


@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 5), (4096, 4096), (1000, 4100), (3, 11008)])
def test_matvec_f32_matches_oracle(cc, rows, cols):
    rng = np.random.default_rng(rows + cols)
    w = rng.standard_normal((rows, cols)).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    y = cc.matvec_f32(w, x, rows, cols)
    assert parity(y, ora.matvec_f32(w, x), w.astype(np.float64) @ x)


def test_fused_qkv_rope_matches_oracle(cc):
    rng = np.random.default_rng(12)
    E, nh, nkv, hd, pos, theta = 1024, 8, 2, 128, 777, 5e5
    wq = rng.standard_normal((nh * hd, E)).astype(np.float32) * 0.05
    wk = rng.standard_normal((nkv * hd, E)).astype(np.float32) * 0.05
    wv = rng.standard_normal((nkv * hd, E)).astype(np.float32) * 0.05
    x = rng.standard_normal(E).astype(np.float32)
    q, k, v = cc.fused_qkv_rope_f32(wq, wk, wv, x, nh * hd, nkv * hd, E, hd, pos, theta)
    rq = ora.rope_multi_head(ora.matvec_f32(wq, x), hd, nh, pos, theta)
    rk = ora.rope_multi_head(ora.matvec_f32(wk, x), hd, nkv, pos, theta)
    assert rel_err(q, rq) <= 1e-3 and rel_err(k, rk) <= 1e-3
    assert rel_err(v, ora.matvec_f32(wv, x)) <= 1e-3


def test_feed_forward_matches_oracle(cc):
    rng = np.random.default_rng(13)
    E, F = 512, 1376
    x = rng.standard_normal(E).astype(np.float32)
    wg, wu = (rng.standard_normal(F * E).astype(np.float32) * 0.05 for _ in range(2))
    wd = rng.standard_normal(E * F).astype(np.float32) * 0.05
    out = cc.feed_forward_f32(x, wg, wu, wd, E)
    assert parity(out, ora.feed_forward_f32(x, wg, wu, wd, E, F), ffn64(x, wg, wu, wd, E, F))


def test_resident_f32_weight_and_dense_swiglu(cc):
    """F32 weights uploaded once: ssd_matvec, ssd_matvec_residual and ssd_fused_swiglu
    (dense gate / up rows in one pass, norm_w NULL)."""
    ctx = cc.ctx
    rng = np.random.default_rng(14)
    E, F = 1000, 700
    w = rng.standard_normal((F, E)).astype(np.float32)
    u = rng.standard_normal((F, E)).astype(np.float32)
    x = rng.standard_normal(E).astype(np.float32)
    W = ssdllm.Weight.upload(ctx, w.view(np.uint8), 0, F, E)
    U = ssdllm.Weight.upload(ctx, u.view(np.uint8), 0, F, E)
    assert np.array_equal(W.download().view(np.float32).reshape(F, E), w)
    xd = torch.from_numpy(x).to(DEV)
    y = torch.zeros(F, device=DEV)
    ssdllm.matvec(ctx, W, xd, y)
    g64 = w.astype(np.float64) @ x
    assert parity(y.cpu().numpy(), ora.matvec_f32(w, x), g64)
    base = torch.from_numpy(rng.standard_normal(F).astype(np.float32)).to(DEV)
    ssdllm.matvec_residual(ctx, W, xd, base, y)
    assert rel_err(y.cpu().numpy(), base.cpu().numpy() + g64) <= 1e-3
    act = torch.zeros(F, device=DEV)
    ssdllm.check(ssdllm.lib().ssd_fused_swiglu(ctx.h, W.h, U.h, xd.data_ptr(), None,
                                               0.0, act.data_ptr(),
                                               torch.cuda.current_stream().cuda_stream))
    u64 = u.astype(np.float64) @ x
    ref = g64 / (1 + np.exp(-g64)) * u64
    assert rel_err(act.cpu().numpy(), ref) <= 1e-3
