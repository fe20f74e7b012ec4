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


def test_model_prefill_matches_oracle_token_loop(ctx):
    """Batch prefill of 128 prompt tokens (Q4_K layers, GQA, 2 layers) against the oracle
    running the same tokens one at a time through its layer step (the reference's
    batch_prefill runs the per-token forward_pass math layer by layer): the last token's
    hidden state within the parity tolerance, every INT8 KV row the same to one quantum,
    the greedy next token identical, and decode continuing from it."""
    from test_gpu_model import build_model, make_weights, oracle_layers
    E, nh, nkv, hd, F, V, nl, n = 512, 8, 2, 64, 1024, 256, 2, 128
    cfg = dict(n_layers=nl, n_embd=E, n_head=nh, n_head_kv=nkv, head_dim=hd, n_ff=F, vocab=V,
               wtype=ora.Q4_K, out_type=ora.Q4_0, embd_type=ora.Q4_0, kv_capacity=n + 8,
               theta=5e5, eps=1e-5, tp_rank=0, tp_size=1)
    rng = np.random.default_rng(11)
    layers, glob = make_weights(rng, E, nh, nkv, hd, F, V, nl, wtype=ora.Q4_K)
    m = build_model(ctx, cfg, layers, glob)
    toks = rng.integers(0, V, n).astype(np.int32)
    m.set_position(0)
    nxt = m.prefill(toks)
    assert ctx.device_status() == 0
    hp, _, _ = m.state_ptrs()
    h_gpu = np.zeros(E, np.float32)
    ssdllm.copy_to_host(ctx, h_gpu, hp)
    assert m.position() == n
    after = m.decode_token(nxt, use_graph=False)

    ol = oracle_layers(cfg, layers)
    embf = ora.dequantize(glob["token_embd"], ora.Q4_0, V * E).reshape(V, E)
    outf = ora.dequantize(glob["output"], ora.Q4_0, V * E).reshape(V, E)
    kvd = nkv * hd
    caches = [(np.zeros((n + 8, kvd), np.int8), np.zeros(n + 8, np.float32),
               np.zeros((n + 8, kvd), np.int8), np.zeros(n + 8, np.float32)) for _ in range(nl)]
    for pos in range(n):
        h = embf[toks[pos]].copy()
        for li in range(nl):
            ol[li].step(h, pos, *caches[li], mode=0, threads=8)
    assert rel_err(h_gpu, h) <= 1e-3, rel_err(h_gpu, h)
    logits = ora.fused_rmsnorm_linear(h, glob["output_norm"], outf, V, E)
    assert nxt == ora.argmax(logits), (nxt, ora.argmax(logits))
    from test_gpu_model import read_cache
    for li in range(nl):
        kq, ks, vq, vs = read_cache(ctx, m, li, n, kvd)
        assert np.max(np.abs(kq.astype(int) - caches[li][0][:n].astype(int))) <= 1
        assert np.max(np.abs(vq.astype(int) - caches[li][2][:n].astype(int))) <= 1
    h2 = embf[nxt].copy()
    for li in range(nl):
        ol[li].step(h2, n, *caches[li], mode=0, threads=8)
    assert after == ora.argmax(ora.fused_rmsnorm_linear(h2, glob["output_norm"], outf, V, E))
    m.free()
