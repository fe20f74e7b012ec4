"""SSD -> HBM streaming tier (ssd_stream_*; SsdStreamer / Prefetcher / LayerCache,
src/ssd/streamer.rs:34-80, src/ssd/prefetch.rs:24-67, src/model/cache.rs): a model whose
layer matrices stay in a GGUF file and pass through a budget of HBM layer slots decodes the
same greedy tokens as the same file loaded HBM-resident (ssd_model_load_gguf, itself checked
against the oracle), whatever the budget and lookahead; the cache counters follow the
policy (LRU victims outside the prefetch window, pinned layers never reloaded)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from gguf_write import llama_metadata, write_gguf  # noqa: E402

L, E, NH, NKV, HD, F, V = 6, 256, 4, 2, 64, 512, 1000
STEPS = 12


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


@pytest.fixture(scope="module")
def gguf_path(tmp_path_factory):
    rng = np.random.default_rng(23)
    q = lambda r, c, t: ora.quantize((rng.standard_normal((r, c)) * 0.05).astype(np.float32), t)
    norm = lambda: (rng.random(E) + 0.5).astype(np.float32)
    kvd = NKV * HD
    tensors = [("token_embd.weight", [E, V], ora.Q8_0, q(V, E, ora.Q8_0).tobytes()),
               ("output_norm.weight", [E], 0, norm().tobytes()),
               ("output.weight", [E, V], ora.Q4_0, q(V, E, ora.Q4_0).tobytes())]
    for l in range(L):
        # layers of different types, so the slots are carved per layer (Q4_K at l = 3)
        t = ora.Q4_K if l == 3 else ora.Q4_0
        mats = {"attn_q": (E, E), "attn_k": (kvd, E), "attn_v": (kvd, E),
                "attn_output": (E, E), "ffn_gate": (F, E), "ffn_up": (F, E), "ffn_down": (E, F)}
        tensors.append((f"blk.{l}.attn_norm.weight", [E], 0, norm().tobytes()))
        tensors.append((f"blk.{l}.ffn_norm.weight", [E], 0, norm().tobytes()))
        for n, (r, c) in mats.items():
            tensors.append((f"blk.{l}.{n}.weight", [c, r], t, q(r, c, t).tobytes()))
    path = str(tmp_path_factory.mktemp("stream") / "six_layers.gguf")
    write_gguf(path, llama_metadata(L, E, NH, NKV, F, V, theta=1e4, eps=1e-5), tensors)
    return path


@pytest.fixture(scope="module")
def resident_tokens(ctx, gguf_path):
    m = ssdllm.Model.from_gguf(ctx, gguf_path, kv_capacity=32)
    try:
        m.set_position(0)
        t, seq = 3, []
        for _ in range(STEPS):
            t = m.decode_token(t, use_graph=True)
            seq.append(t)
        return seq
    finally:
        m.free()


def _stream(ctx, path, budget, lookahead):
    cfg = ssdllm.GgufFile(path).model_config(kv_capacity=32)
    m = ssdllm.Model(ctx, **cfg)
    try:
        return m, ssdllm.Stream(m, path, budget, lookahead)
    except Exception:
        m.free()
        raise


def _decode(m, st):
    m.set_position(0)
    t, seq = 3, []
    for _ in range(STEPS):
        t = st.decode_token(t)
        seq.append(t)
    return seq


def _slot_bytes(ctx, path):
    m, st = _stream(ctx, path, 1 << 40, 0)
    try:
        s = st.stats()
        assert s["n_slots"] == L  # a budget above the model: one slot per layer
        return s["slot_bytes"]
    finally:
        st.close()
        m.free()


@pytest.mark.parametrize("slots,lookahead", [(1, 0), (1, 1), (2, 1), (3, 2), (L, 1)])
def test_streamed_decode_equals_resident(ctx, gguf_path, resident_tokens, slots, lookahead):
    sb = _slot_bytes(ctx, gguf_path)
    m, st = _stream(ctx, gguf_path, slots * sb + sb // 2, lookahead)
    try:
        assert _decode(m, st) == resident_tokens
        s = st.stats()
        assert s["n_slots"] == slots
        assert s["hits"] + s["misses"] == STEPS * L
        assert s["loads"] >= s["misses"] + s["prefetch_hits"]  # some prefetches may go unused
        if slots == L:  # everything fits: each layer read once, never evicted
            assert s["loads"] == L and s["evictions"] == 0
        else:  # every layer is read again each step
            assert s["loads"] >= STEPS * L - (slots - 1) and s["evictions"] > 0
        if lookahead and slots > 1:
            assert s["prefetch_hits"] > 0
        if lookahead == 0:
            assert s["prefetch_hits"] == 0
    finally:
        st.close()
        m.free()


def test_pinned_layer_is_loaded_once(ctx, gguf_path, resident_tokens):
    sb = _slot_bytes(ctx, gguf_path)
    m, st = _stream(ctx, gguf_path, 3 * sb, 1)
    try:
        st.pin(0)
        assert _decode(m, st) == resident_tokens
        s = st.stats()
        # layer 0 once (at the pin); layers 1-5 once per step (3 slots, one of them pinned)
        assert s["loads"] == 1 + STEPS * (L - 1)
        st.pin(1)  # two of three slots pinned: one is left for the other layers
        with pytest.raises(ssdllm.SsdError):  # a third would leave none
            st.pin(2)
    finally:
        st.close()
        m.free()


def test_budget_below_one_layer_is_refused(ctx, gguf_path):
    sb = _slot_bytes(ctx, gguf_path)
    cfg = ssdllm.GgufFile(gguf_path).model_config(kv_capacity=32)
    m = ssdllm.Model(ctx, **cfg)
    try:
        with pytest.raises(ssdllm.SsdError) as e:
            ssdllm.Stream(m, gguf_path, sb // 2, 1)
        assert e.value.status == 7  # SSD_ERR_NOMEM
    finally:
        m.free()
