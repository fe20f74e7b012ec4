"""Low-bit layer weights in the decode engine (tp_size 1): Q3_K, Q2_K, IQ4_NL, IQ4_XS, IQ3_XXS,
IQ3_S, IQ2_XXS and IQ2_XS attn / FFN / output tensors, which the reference dispatches like any
other type (matvec_quantized, src/metal/compute.rs:648-675; the row kernels :793-1075,
:1964-2240). The engine runs each stage as RMSNorm -> the low-bit matvec(s) -> RoPE, SwiGLU
or the argmax key (the quantized kernels' fused prologues and epilogues as separate
launches); 16 greedy tokens must equal the oracle's decode loop (generate,
src/inference/transformer.rs:681-770; a near-tie below fp32 reordering noise may end the
comparison), graph and eager replay must agree, and the launch count is checked."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

import _lowbit_kats as K  # noqa: E402
from _models import OracleDecoder  # noqa: E402

NEAR_TIE = 1e-4
E, NH, NKV, HD, F, VOCAB, NL, CAP = 256, 4, 2, 64, 512, 384, 2, 40


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


def lowbit_model(rng, t):
    shapes = {"attn_q": (NH * HD, E), "attn_k": (NKV * HD, E), "attn_v": (NKV * HD, E),
              "attn_output": (E, NH * HD), "ffn_gate": (F, E), "ffn_up": (F, E),
              "ffn_down": (E, F)}
    layers = []
    for _ in range(NL):
        L = {n: K.random_blocks(rng, t, *sh) for n, sh in shapes.items()}
        L["attn_norm"] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        L["ffn_norm"] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        layers.append(L)
    emb = rng.standard_normal((VOCAB, E)).astype(np.float32)
    glob = {"token_embd": ora.quantize(emb, ora.Q4_0), "output": K.random_blocks(rng, t, VOCAB, E),
            "output_norm": (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)}
    return layers, glob


@pytest.mark.parametrize("t", K.LOWBIT)
def test_lowbit_layers_decode_like_oracle(ctx, t):
    cfg = dict(n_layers=NL, n_embd=E, n_head=NH, n_head_kv=NKV, head_dim=HD, n_ff=F, vocab=VOCAB,
               wtype=t, out_type=t, embd_type=ora.Q4_0, kv_capacity=CAP, theta=1e4, eps=1e-5,
               tp_rank=0, tp_size=1)
    rng = np.random.default_rng(700 + t)
    layers, glob = lowbit_model(rng, t)
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
            for _ in range(16):
                tok = m.decode_token(tok, use_graph=g)
                seq.append(tok)
            toks[g] = seq
        assert toks[True] == toks[False]
        # embed, 2 x (norm, Q, K, V, RoPE, attention partial + combine, o_proj, norm, gate,
        # up, SwiGLU, down), norm, logits, argmax, finalize
        assert m.launches_per_step() == 1 + NL * 13 + 3 + 1
        with pytest.raises(ssdllm.SsdError) as e:  # the prefill GEMMs take no low-bit weights
            m.prefill([1] * 128)
        assert e.value.status == 2
    finally:
        m.free()
    ref = OracleDecoder(cfg, layers, glob, CAP)
    tok = 11
    for i, g in enumerate(toks[True]):
        tok, margin = ref.step(tok)
        if g != tok:
            assert margin < NEAR_TIE, (i, g, tok, margin)
            break
        tok = g


def test_lowbit_layers_refused_with_tensor_parallelism(ctx):
    cfg = dict(n_layers=1, n_embd=E, n_head=NH, n_head_kv=NKV, head_dim=HD, n_ff=F, vocab=VOCAB,
               wtype=K.IQ4_XS, out_type=ora.Q4_0, embd_type=ora.Q4_0, kv_capacity=16, theta=1e4,
               eps=1e-5, tp_rank=0, tp_size=2)
    with pytest.raises(ssdllm.SsdError) as e:
        ssdllm.Model(ctx, **cfg)
    assert e.value.status == 2
