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


def test_q6k_model_greedy_decode_matches_oracle(ctx):
    """A model whose layer weights, output head and token embedding are all Q6_K (as in a
    Q6_K GGUF file): 32 greedy tokens equal the oracle's decode loop (a near-tie below
    fp32 reordering noise may end the comparison early)."""
    from test_gpu_model import LAYER_NAMES, build_model, oracle_layers
    E, nh, nkv, hd, F, vocab, nl = 256, 4, 2, 64, 512, 512, 2
    cfg = dict(n_layers=nl, n_embd=E, n_head=nh, n_head_kv=nkv, head_dim=hd, n_ff=F, vocab=vocab,
               wtype=Q6_K, out_type=Q6_K, embd_type=Q6_K, kv_capacity=48, theta=1e4, eps=1e-5,
               tp_rank=0, tp_size=1)
    rng = np.random.default_rng(74)
    shapes = {"attn_q": (nh * hd, E), "attn_k": (nkv * hd, E), "attn_v": (nkv * hd, E),
              "attn_output": (E, E), "ffn_gate": (F, E), "ffn_up": (F, E), "ffn_down": (E, F)}
    layers = []
    for _ in range(nl):
        L = {n: raw_q6k(rng, *s) for n, s in shapes.items()}
        L["attn_norm"] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        L["ffn_norm"] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        layers.append(L)
    glob = {"token_embd": raw_q6k(rng, vocab, E), "output": raw_q6k(rng, vocab, E),
            "output_norm": (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)}
    assert set(LAYER_NAMES) <= set(layers[0])
    m = build_model(ctx, cfg, layers, glob)
    m.set_position(0)
    gpu, t = [], 5
    for _ in range(32):
        t = m.decode_token(t, use_graph=True)
        gpu.append(t)
    m.free()

    OL = oracle_layers(cfg, layers)
    emb = ora.dequantize(glob["token_embd"], Q6_K, vocab * E).reshape(vocab, E)
    out_w = ora.dequantize(glob["output"], Q6_K, vocab * E).reshape(vocab, E)
    kvd = nkv * hd
    caches = [(np.zeros((48, kvd), np.int8), np.zeros(48, np.float32),
               np.zeros((48, kvd), np.int8), np.zeros(48, np.float32)) for _ in range(nl)]
    t = 5
    for pos in range(32):
        h = emb[t].copy()
        for li in range(nl):
            kc, ks, vc, vs = caches[li]
            OL[li].step(h, pos, kc, ks, vc, vs, mode=0, threads=4)
        logits = ora.fused_rmsnorm_linear(h, glob["output_norm"], out_w, vocab, E)
        t = ora.argmax(logits)
        if gpu[pos] != t:
            srt = np.sort(logits)
            assert (srt[-1] - srt[-2]) / np.max(np.abs(logits)) < 1e-4, (pos, gpu[pos], t)
            return


def test_mixed_type_model_greedy_decode_matches_oracle(ctx):
    """Weights of different types per tensor, as GGUF files mix them (the reference
    dispatches each tensor on its own dtype): Q4_K attn_q / attn_k, Q6_K attn_v (its own
    launch), Q4_0 attn_output, Q8_0 gate / up, Q6_K down and output, Q4_K token_embd, set
    through ssd_model_set_tensor_typed. 32 greedy tokens equal the oracle's decode loop."""
    Q4_0, Q8_0, Q4_K = ora.Q4_0, ora.Q8_0, ora.Q4_K
    E, nh, nkv, hd, F, vocab, nl = 256, 4, 2, 64, 512, 512, 2
    cfg = dict(n_layers=nl, n_embd=E, n_head=nh, n_head_kv=nkv, head_dim=hd, n_ff=F, vocab=vocab,
               wtype=Q4_0, out_type=Q4_0, embd_type=Q4_0, kv_capacity=48, theta=1e4, eps=1e-5,
               tp_rank=0, tp_size=1)
    rng = np.random.default_rng(75)
    names = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")
    types = (Q4_K, Q4_K, Q6_K, Q4_0, Q8_0, Q8_0, Q6_K)
    shapes = ((nh * hd, E), (nkv * hd, E), (nkv * hd, E), (E, E), (F, E), (F, E), (E, F))

    def mk(t, s):
        if t == Q6_K:
            return raw_q6k(rng, *s)
        return ora.quantize((rng.standard_normal(s) * 0.02).astype(np.float32), t)

    layers = []
    for _ in range(nl):
        L = {n: mk(t, s) for n, t, s in zip(names, types, shapes)}
        L["attn_norm"] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        L["ffn_norm"] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        layers.append(L)
    emb = ora.quantize(rng.standard_normal((vocab, E)).astype(np.float32), Q4_K)
    out = raw_q6k(rng, vocab, E)
    onorm = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    m = ssdllm.Model(ctx, **cfg)
    try:
        for li, L in enumerate(layers):
            for n, t in zip(names, types):
                m.set_tensor(n, li, L[n], wtype=t)
            m.set_tensor("attn_norm", li, L["attn_norm"])
            m.set_tensor("ffn_norm", li, L["ffn_norm"])
        m.set_tensor("token_embd", -1, emb, wtype=Q4_K)
        m.set_tensor("output", -1, out, wtype=Q6_K)
        m.set_tensor("output_norm", -1, onorm)
        m.set_position(0)
        gpu, t = [], 9
        for _ in range(32):
            t = m.decode_token(t, use_graph=True)
            gpu.append(t)
        # embed, 2 x (QKV, V, attention partial + combine, o_proj, gate/up, down), logits, finalize
        assert m.launches_per_step() == 1 + nl * 7 + 2
    finally:
        m.free()

    OL = [ora.Layer(E, nh, nkv, hd, F, Q4_0, *(L[n] for n in names), L["attn_norm"],
                    L["ffn_norm"], theta=1e4, eps=1e-5, wtypes=list(types)) for L in layers]
    embf = ora.dequantize(emb, Q4_K, vocab * E).reshape(vocab, E)
    outf = ora.dequantize(out, Q6_K, vocab * E).reshape(vocab, E)
    kvd = nkv * hd
    caches = [(np.zeros((48, kvd), np.int8), np.zeros(48, np.float32),
               np.zeros((48, kvd), np.int8), np.zeros(48, np.float32)) for _ in range(nl)]
    t = 9
    for pos in range(32):
        h = embf[t].copy()
        for li in range(nl):
            kc, ks, vc, vs = caches[li]
            OL[li].step(h, pos, kc, ks, vc, vs, mode=0, threads=4)
        logits = ora.fused_rmsnorm_linear(h, onorm, outf, vocab, E)
        t = ora.argmax(logits)
        if gpu[pos] != t:
            srt = np.sort(logits)
            assert (srt[-1] - srt[-2]) / np.max(np.abs(logits)) < 1e-4, (pos, gpu[pos], t)
            return


def test_mixed_types_that_cannot_fuse_are_rejected(ctx):
    """attn_q / attn_k (and ffn_gate / ffn_up) run as one fused launch, so they must share
    a type: a decode step with them differing fails with SSD_ERR_TYPE, not a wrong result."""
    E, nh, nkv, hd, F = 256, 4, 2, 64, 512
    cfg = dict(n_layers=1, n_embd=E, n_head=nh, n_head_kv=nkv, head_dim=hd, n_ff=F, vocab=64,
               wtype=ora.Q4_0, out_type=ora.Q4_0, embd_type=ora.Q4_0, kv_capacity=8, theta=1e4,
               eps=1e-5, tp_rank=0, tp_size=1)
    m = ssdllm.Model(ctx, **cfg)
    try:
        m.synth_weights(seed=3, std=0.02)
        rng = np.random.default_rng(76)
        m.set_tensor("attn_k", 0, raw_q6k(rng, nkv * hd, E), wtype=Q6_K)
        m.set_position(0)
        with pytest.raises(ssdllm.SsdError) as e:
            m.decode_token(1, use_graph=False)
        assert e.value.status == 2  # SSD_ERR_TYPE
    finally:
        m.free()
