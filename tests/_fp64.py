"""Float64 restatement of one decoder layer over a prompt (the math of forward_pass,
src/inference/transformer.rs:283-399, run for each prompt position as batch_prefill does,
:120-250), used to referee GPU-vs-oracle differences: the oracle sums in fp32 in the
reference's order, and over rows of 14336 terms its own error approaches the 1e-3 bar."""
import numpy as np

from oracle import oracle as ora


def rmsnorm(x, w, eps, order):
    inv = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x * (inv * w) if order == 0 else (x * inv) * w


def rope(x, n_heads, head_dim, positions, theta):
    """Pairs (2i, 2i+1) of every head rotated by pos / theta^(2i/d) (compute.rs:482-506)."""
    out = x.copy()
    i = np.arange(head_dim // 2)
    freq = 1.0 / theta ** (2.0 * i / head_dim)
    ang = positions[:, None] * freq[None, :]
    c, s = np.cos(ang), np.sin(ang)
    for h in range(n_heads):
        a = x[:, h * head_dim + 2 * i]
        b = x[:, h * head_dim + 2 * i + 1]
        out[:, h * head_dim + 2 * i] = a * c - b * s
        out[:, h * head_dim + 2 * i + 1] = a * s + b * c
    return out


def deq(raw, wtype, rows, cols):
    return ora.dequantize(raw, wtype, rows * cols).reshape(rows, cols).astype(np.float64)


def layer_prefill(cfg, L, X, kq, ks, vq, vs):
    """X: [n, E] layer inputs of positions 0..n-1 (fp64); kq/ks/vq/vs: the INT8 cache rows
    of those positions as the implementation under test wrote them (its quantizer's output),
    so the attention reads the same codes. Returns the layer outputs [n, E] in fp64."""
    E, nh, nkv, hd, F = cfg["n_embd"], cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"], cfg["n_ff"]
    wt, eps, theta = cfg["wtype"], cfg["eps"], cfg["theta"]
    n = X.shape[0]
    pos = np.arange(n, dtype=np.float64)
    xn = rmsnorm(X, L["attn_norm"].astype(np.float64), eps, 0)
    q = rope(xn @ deq(L["attn_q"], wt, nh * hd, E).T, nh, hd, pos, theta)
    K = kq.astype(np.float64) * ks.astype(np.float64)[:, None]
    V = vq.astype(np.float64) * vs.astype(np.float64)[:, None]
    g = nh // nkv
    att = np.zeros((n, nh * hd))
    mask = np.triu(np.ones((n, n), bool), 1)
    for h in range(nh):
        kh = K[:, (h // g) * hd:(h // g + 1) * hd]
        vh = V[:, (h // g) * hd:(h // g + 1) * hd]
        s = (q[:, h * hd:(h + 1) * hd] @ kh.T) / np.sqrt(hd)
        s[mask] = -np.inf
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        att[:, h * hd:(h + 1) * hd] = p @ vh
    h1 = X + att @ deq(L["attn_output"], wt, E, nh * hd).T
    hn = rmsnorm(h1, L["ffn_norm"].astype(np.float64), eps, 1)
    gate = hn @ deq(L["ffn_gate"], wt, F, E).T
    up = hn @ deq(L["ffn_up"], wt, F, E).T
    act = gate / (1.0 + np.exp(-gate)) * up
    return h1 + act @ deq(L["ffn_down"], wt, E, F).T
