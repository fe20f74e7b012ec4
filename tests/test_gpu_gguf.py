"""A decode model loaded from a GGUF file (ssd_gguf_model_config + ssd_model_load_gguf)
decodes exactly like the same weights set tensor by tensor (ssd_model_set_tensor), the
path the oracle parity tests cover; a file without output.weight uses token_embd as the
output head (transformer.rs:690-700)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from gguf_write import llama_metadata, write_gguf  # noqa: E402

L, E, NH, NKV, HD, F, V = 2, 256, 4, 2, 64, 512, 1000


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


def _weights(tied):
    rng = np.random.default_rng(17)
    q = lambda r, c, t: ora.quantize((rng.standard_normal((r, c)) * 0.05).astype(np.float32), t)
    norm = lambda: (rng.random(E) + 0.5).astype(np.float32)
    kvd = NKV * HD
    glob = {"token_embd": (q(V, E, ora.Q8_0), [E, V], ora.Q8_0),
            "output_norm": (norm(), [E], 0)}
    if not tied:
        glob["output"] = (q(V, E, ora.Q4_0), [E, V], ora.Q4_0)
    layers = []
    for _ in range(L):
        layers.append({
            "attn_norm": (norm(), [E], 0), "attn_q": (q(E, E, ora.Q4_0), [E, E], ora.Q4_0),
            "attn_k": (q(kvd, E, ora.Q4_0), [E, kvd], ora.Q4_0),
            "attn_v": (q(kvd, E, ora.Q4_0), [E, kvd], ora.Q4_0),
            "attn_output": (q(E, E, ora.Q4_0), [E, E], ora.Q4_0), "ffn_norm": (norm(), [E], 0),
            "ffn_gate": (q(F, E, ora.Q4_0), [E, F], ora.Q4_0),
            "ffn_up": (q(F, E, ora.Q4_0), [E, F], ora.Q4_0),
            "ffn_down": (q(E, F, ora.Q4_0), [F, E], ora.Q4_0)})
    return glob, layers


def _tokens(m, n=16):
    m.set_position(0)
    t, seq = 3, []
    for _ in range(n):
        t = m.decode_token(t, use_graph=True)
        seq.append(t)
    return seq


@pytest.mark.parametrize("tied", [False, True])
def test_model_from_gguf_decodes_like_set_tensor(ctx, tmp_path, tied):
    glob, layers = _weights(tied)
    tensors = [(f"{n}.weight", dims, t, np.asarray(a).tobytes()) for n, (a, dims, t) in glob.items()]
    for l, ly in enumerate(layers):
        tensors += [(f"blk.{l}.{n}.weight", dims, t, np.asarray(a).tobytes())
                    for n, (a, dims, t) in ly.items()]
    path = str(tmp_path / "tiny.gguf")
    write_gguf(path, llama_metadata(L, E, NH, NKV, F, V, theta=1e4, eps=1e-5), tensors)

    m1 = ssdllm.Model.from_gguf(ctx, path, kv_capacity=32)
    cfg = ssdllm.GgufFile(path).model_config(kv_capacity=32)
    assert cfg["out_type"] == (ora.Q8_0 if tied else ora.Q4_0)
    m2 = ssdllm.Model(ctx, **cfg)
    for n, (a, _, _) in glob.items():
        m2.set_tensor(n, -1, a)
    if tied:
        m2.set_tensor("output", -1, glob["token_embd"][0])
    for l, ly in enumerate(layers):
        for n, (a, _, _) in ly.items():
            m2.set_tensor(n, l, a)
    try:
        t1, t2 = _tokens(m1), _tokens(m2)
        assert t1 == t2
    finally:
        m1.free()
        m2.free()
