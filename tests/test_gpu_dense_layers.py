"""Dense layer weights in the decode engine (tp_size 1): F16, BF16 and F32 attn / FFN / output
tensors, which the reference dispatches like any other type (matvec_f16_cpu /
matvec_bf16_cpu, src/metal/compute.rs:2250-2285; matvec_f32_simd, :378-424). The engine runs
each dense stage as RMSNorm -> matvec(s) -> RoPE or argmax (the fused prologues and epilogues
are the quantized kernels'); 24 greedy tokens must equal the oracle's decode loop
(generate, src/inference/transformer.rs:681-770; a near-tie below fp32 reordering noise may
end the comparison), graph and eager replay must agree, and the launch count is checked."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from _models import LAYER_NAMES, OracleDecoder  # noqa: E402

NEAR_TIE = 1e-4


def to_raw(w, t):
    """f32 rows -> the type's row-major bytes (F16 / BF16 round to nearest even)."""
    w = np.ascontiguousarray(w, np.float32)
    if t == ora.F32:
        return w.view(np.uint8).reshape(w.shape[0], -1)
    if t == ora.F16:
        return w.astype(np.float16).view(np.uint8).reshape(w.shape[0], -1)
    u = w.view(np.uint32).astype(np.uint64)
    b = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return b.view(np.uint8).reshape(w.shape[0], -1)


def dense_weights(rng, E, nh, nkv, hd, F, vocab, n_layers, t):
    shapes = {"attn_q": (nh * hd, E), "attn_k": (nkv * hd, E), "attn_v": (nkv * hd, E),
              "attn_output": (E, nh * hd), "ffn_gate": (F, E), "ffn_up": (F, E),
              "ffn_down": (E, F)}
    layers = []
    for _ in range(n_layers):
        L = {n: to_raw(rng.standard_normal(sh, dtype=np.float32) * np.float32(0.05), t)
             for n, sh in shapes.items()}
        L["attn_norm"] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        L["ffn_norm"] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        layers.append(L)
    emb = rng.standard_normal((vocab, E), dtype=np.float32)
    out = rng.standard_normal((vocab, E), dtype=np.float32) * np.float32(0.05)
    glob = {"token_embd": ora.quantize(emb, ora.Q4_0), "output": to_raw(out, t),
            "output_norm": (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)}
    return layers, glob


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


@pytest.mark.parametrize("t", [ora.F16, ora.BF16, ora.F32])
def test_dense_layers_decode_like_oracle(ctx, t):
    E, nh, nkv, hd, F, vocab, nl, cap = 256, 4, 2, 64, 512, 384, 2, 40
    cfg = dict(n_layers=nl, n_embd=E, n_head=nh, n_head_kv=nkv, head_dim=hd, n_ff=F, vocab=vocab,
               wtype=t, out_type=t, embd_type=ora.Q4_0, kv_capacity=cap, theta=1e4, eps=1e-5,
               tp_rank=0, tp_size=1)
    rng = np.random.default_rng(500 + t)
    layers, glob = dense_weights(rng, E, nh, nkv, hd, F, vocab, nl, t)
    m = ssdllm.Model(ctx, **cfg)
    try:
        for li, L in enumerate(layers):
            for n, a in L.items():
                m.set_tensor(n, li, a)
        for n, a in glob.items():
            m.set_tensor(n, -1, a)
        toks = {}
        for g in (True, False):
            m.set_position(0)
            seq, tok = [], 11
            for _ in range(24):
                tok = m.decode_token(tok, use_graph=g)
                seq.append(tok)
            toks[g] = seq
        assert toks[True] == toks[False]
        # embed, 2 x (norm, Q, K, V, RoPE, attention partial + combine, o_proj, norm,
        # gate/up + SwiGLU, down), norm, logits, argmax, finalize
        assert m.launches_per_step() == 1 + nl * 11 + 3 + 1
    finally:
        m.free()
    ref = OracleDecoder(cfg, layers, glob, cap)
    tok = 11
    for i, g in enumerate(toks[True]):
        tok, margin = ref.step(tok)
        if g != tok:
            assert margin < NEAR_TIE, (i, g, tok, margin)
            break
        tok = g


def test_dense_layers_refused_with_tensor_parallelism():
    cfg = dict(n_layers=1, n_embd=256, n_head=4, n_head_kv=2, head_dim=64, n_ff=512, vocab=384,
               wtype=ora.F16, out_type=ora.Q4_0, embd_type=ora.Q4_0, kv_capacity=16, theta=1e4,
               eps=1e-5, tp_rank=0, tp_size=2)
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    with pytest.raises(ssdllm.SsdError) as e:
        ssdllm.Model(ssdllm.Context(0), **cfg)
    assert e.value.status == 2
