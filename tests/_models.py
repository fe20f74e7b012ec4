"""Toy decoder models and the oracle's greedy decode loop, shared by the decode-engine
parity tests."""
import numpy as np

from oracle import oracle as ora

LAYER_NAMES = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")


def make_weights(rng, E, nh, nkv, hd, F, vocab, n_layers, wtype=ora.Q4_0, out_type=ora.Q4_0):
    shapes = {"attn_q": (nh * hd, E), "attn_k": (nkv * hd, E), "attn_v": (nkv * hd, E),
              "attn_output": (E, nh * hd), "ffn_gate": (F, E), "ffn_up": (F, E),
              "ffn_down": (E, F)}
    layers = []
    for _ in range(n_layers):
        L = {}
        for n, sh in shapes.items():
            wf = rng.standard_normal(sh, dtype=np.float32)
            wf *= np.float32(0.02)
            L[n] = ora.quantize(wf, wtype)
            del wf
        L["attn_norm"] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        L["ffn_norm"] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        layers.append(L)
    emb = rng.standard_normal((vocab, E), dtype=np.float32)
    out = rng.standard_normal((vocab, E), dtype=np.float32)
    out *= np.float32(0.05)
    glob = {"token_embd": ora.quantize(emb, ora.Q4_0), "output": ora.quantize(out, out_type),
            "output_norm": (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)}
    return layers, glob


def build_model(ssdllm, ctx, cfg, layers, glob):
    m = ssdllm.Model(ctx, **cfg)
    for li, L in enumerate(layers):
        for n, a in L.items():
            m.set_tensor(n, li, a)
    for n, a in glob.items():
        m.set_tensor(n, -1, a)
    return m


def oracle_layers(cfg, layers):
    return [ora.Layer(cfg["n_embd"], cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"],
                      cfg["n_ff"], cfg["wtype"], *(L[n] for n in LAYER_NAMES), L["attn_norm"],
                      L["ffn_norm"], theta=cfg["theta"], eps=cfg["eps"]) for L in layers]


class OracleDecoder:
    """generate's token loop (src/inference/transformer.rs:681-770) on the oracle's layer
    step over its own INT8 caches: one decoding request."""

    def __init__(self, cfg, layers, glob, capacity):
        E, vocab = cfg["n_embd"], cfg["vocab"]
        self.cfg, self.glob = cfg, glob
        self.OL = oracle_layers(cfg, layers)
        self.emb = ora.dequantize(glob["token_embd"], ora.Q4_0, vocab * E).reshape(vocab, E)
        self.out_w = ora.dequantize(glob["output"], cfg["out_type"], vocab * E).reshape(vocab, E)
        kvd = cfg["n_head_kv"] * cfg["head_dim"]
        self.caches = [(np.zeros((capacity, kvd), np.int8), np.zeros(capacity, np.float32),
                        np.zeros((capacity, kvd), np.int8), np.zeros(capacity, np.float32))
                       for _ in range(cfg["n_layers"])]
        self.pos = 0

    def step(self, token):
        """Returns (next token, top-2 margin of the logits relative to their max)."""
        cfg = self.cfg
        h = self.emb[token].copy()
        for li, L in enumerate(self.OL):
            kc, ks, vc, vs = self.caches[li]
            L.step(h, self.pos, kc, ks, vc, vs, mode=0, threads=4)
        self.pos += 1
        logits = ora.fused_rmsnorm_linear(h, self.glob["output_norm"], self.out_w, cfg["vocab"],
                                          cfg["n_embd"])
        t = ora.argmax(logits)
        srt = np.sort(logits)
        return t, float((srt[-1] - srt[-2]) / np.max(np.abs(logits)))


def read_cache(ssdllm, ctx, m, layer, n, kvd):
    """The first n rows of one layer's INT8 cache (K, K scales, V, V scales) on the host."""
    kp, vp, ksp, vsp = m.kv(layer).pointers()
    out = []
    for ptr, shape, dt in ((kp, (n, kvd), np.int8), (ksp, (n,), np.float32),
                           (vp, (n, kvd), np.int8), (vsp, (n,), np.float32)):
        a = np.zeros(shape, dt)
        if n:
            ssdllm.copy_to_host(ctx, a, ptr)
        out.append(a)
    return out
