"""16-bit dense weights (F16, BF16) on the GPU against the oracle (matvec_f16_cpu /
matvec_bf16_cpu, src/metal/compute.rs:2250-2285): the reference's own known-answer tests
through the host-pointer entry point (2 x 2 matrices: any column count), bit-exact
dequantization, byte round trip, random matrices within rel. error 1e-3 (fp64 arbiter), the residual epilogue, the refusal
of fused epilogues, and models whose token_embd is F16 / BF16 decoding like the oracle."""
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


def raw16(rng, rows, cols, t, scale=0.05):
    if t == F16:
        return (rng.standard_normal((rows, cols)) * scale).astype(np.float16).view(np.uint8)
    f = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
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


@pytest.mark.parametrize("t,how", [(F16, "config"), (BF16, "set_tensor_typed")])
def test_model_with_16bit_token_embd_decodes_like_oracle(comp, t, how):
    """A Q4_0 model whose token_embd is F16 or BF16 (common in GGUF files), given as the
    config's embd_type or per tensor: 24 greedy tokens equal the oracle's decode loop (a
    near-tie below fp32 reordering noise may end the comparison early)."""
    from test_gpu_model import build_model, make_weights, oracle_layers
    ctx = comp.ctx
    E, nh, nkv, hd, F, vocab, nl = 256, 4, 2, 64, 512, 384, 2
    cfg = dict(n_layers=nl, n_embd=E, n_head=nh, n_head_kv=nkv, head_dim=hd, n_ff=F, vocab=vocab,
               wtype=ora.Q4_0, out_type=ora.Q4_0, embd_type=t if how == "config" else ora.Q4_0,
               kv_capacity=32, theta=1e4, eps=1e-5, tp_rank=0, tp_size=1)
    rng = np.random.default_rng(81 + t)
    layers, glob = make_weights(rng, E, nh, nkv, hd, F, vocab, nl)
    emb_raw = raw16(rng, vocab, E, t, scale=1.0).reshape(vocab, 2 * E)
    glob = dict(glob)
    del glob["token_embd"]
    m = build_model(ctx, cfg, layers, glob)
    try:
        m.set_tensor("token_embd", -1, emb_raw, wtype=None if how == "config" else t)
        m.set_position(0)
        gpu, tok = [], 7
        for _ in range(24):
            tok = m.decode_token(tok, use_graph=True)
            gpu.append(tok)
    finally:
        m.free()
    OL = oracle_layers(cfg, layers)
    emb = ora.dequantize(emb_raw, t, vocab * E).reshape(vocab, E)
    out_w = ora.dequantize(glob["output"], ora.Q4_0, vocab * E).reshape(vocab, E)
    kvd = nkv * hd
    caches = [(np.zeros((32, kvd), np.int8), np.zeros(32, np.float32),
               np.zeros((32, kvd), np.int8), np.zeros(32, np.float32)) for _ in range(nl)]
    tok = 7
    for pos in range(24):
        h = emb[tok].copy()
        for li in range(nl):
            kc, ks, vc, vs = caches[li]
            OL[li].step(h, pos, kc, ks, vc, vs, mode=0, threads=4)
        logits = ora.fused_rmsnorm_linear(h, glob["output_norm"], out_w, vocab, E)
        tok = ora.argmax(logits)
        if gpu[pos] != tok:
            srt = np.sort(logits)
            assert (srt[-1] - srt[-2]) / np.max(np.abs(logits)) < 1e-4, (pos, gpu[pos], tok)
            return


@pytest.mark.parametrize("t", [F16, BF16])
def test_residual_matvec_and_refused_fused_epilogues(comp, t):
    """y = base + W x on 16-bit rows within rel. error 1e-3 of the oracle; the fused RMSNorm /
    SwiGLU prologue + epilogue is not offered for these types and fails with an error
    instead of a wrong result."""
    ctx = comp.ctx
    rng = np.random.default_rng(90 + t)
    rows, cols = 2048, 1024
    raw = raw16(rng, rows, cols, t).reshape(rows, 2 * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    base = rng.standard_normal(rows).astype(np.float32)
    w = ssdllm.Weight.upload(ctx, raw, t, rows, cols)
    try:
        y = torch.zeros(rows, device=DEV)
        ssdllm.matvec_residual(ctx, w, torch.from_numpy(x).to(DEV),
                               torch.from_numpy(base).to(DEV), y)
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        with pytest.raises(ssdllm.SsdError):
            ssdllm.fused_swiglu(ctx, w, w, torch.from_numpy(x).to(DEV),
                                torch.ones(cols, device=DEV), 1e-5,
                                torch.zeros(rows, device=DEV))
        torch.cuda.synchronize()
    finally:
        w.free()
    ref = base + ora.matvec_quantized(raw, x, rows, cols, t, threads=8)
    assert rel_err(got, ref) <= 1e-3
