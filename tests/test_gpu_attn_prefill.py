"""Prompt-batch causal attention (ssd_attention_prefill): the tcgen05 tensor-core kernel
(head_dim 128, queries a multiple of 128) and the per-query split-K kernels
(SSD_PREFILL_ATTN=decode, and the fallback for other shapes) against the oracle's
attention over the INT8 cache (flash_attention.rs:40-143 on quantized_kv_cache.rs:118-130
rows), query i seeing positions 0 .. pos0 + i; an fp64 result arbitrates where the
oracle's own fp32 sums are what exceed the tolerance."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from _util import normwise, parity, rel_err  # noqa: E402

DEV = "cuda:0"


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


def d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def exact_attention(q, kd, vd, n_head, n_kv, hd):
    g = n_head // n_kv
    out = np.zeros(n_head * hd)
    for h in range(n_head):
        c = (h // g) * hd
        sc = kd[:, c:c + hd] @ q[h * hd:(h + 1) * hd].astype(np.float64) / np.sqrt(hd)
        p = np.exp(sc - sc.max())
        out[h * hd:(h + 1) * hd] = (p / p.sum()) @ vd[:, c:c + hd]
    return out


CASES = [  # n_head, n_kv, head_dim, pos0, n_q, V std, q std
    (32, 8, 128, 0, 512, 1.0, 1.0),    # benchmark config 3 shape (Llama-3-8B), fresh prompt
    (8, 2, 128, 100, 256, 1.0, 1.0),   # after 100 cached positions (blocks straddle tiles)
    (16, 16, 128, 0, 128, 1e-3, 1.0),  # no GQA; tiny V values (small V scales)
    (8, 2, 64, 7, 128, 1.0, 1.0),      # head_dim 64: the per-query kernels either way
]


@pytest.mark.parametrize("impl", ["tc", "decode"])
@pytest.mark.parametrize("n_head,n_kv,hd,pos0,n_q,vstd,qstd", CASES + [
    pytest.param(32, 8, 128, 0, 512, 1.0, 2.0, marks=pytest.mark.tc_only)])
def test_prefill_attention_matches_oracle(ctx, monkeypatch, request, impl, n_head, n_kv, hd,
                                          pos0, n_q, vstd, qstd):
    """The last case (q twice as large: a sharper softmax, where the oracle's own fp32
    sums are 6e-4 off an fp64 result) runs on the tensor-core kernel only."""
    if impl == "decode" and request.node.get_closest_marker("tc_only"):
        pytest.skip("sharpened case: tensor-core kernel only")
    if impl == "decode":
        monkeypatch.setenv("SSD_PREFILL_ATTN", "decode")
    else:
        monkeypatch.delenv("SSD_PREFILL_ATTN", raising=False)
    rng = np.random.default_rng(n_head * 7 + pos0 + n_q)
    kvd, L = n_kv * hd, pos0 + n_q
    kf = rng.standard_normal((L, kvd)).astype(np.float32)
    vf = (rng.standard_normal((L, kvd)) * vstd).astype(np.float32)
    q = (rng.standard_normal((n_q, n_head * hd)) * qstd).astype(np.float32)
    kv = ssdllm.KvCache(ctx, L, n_kv, hd)
    try:
        kv.append_rows(d(kf), d(vf), 0)
        out = torch.full((n_q, n_head * hd), float("nan"), device=DEV)
        kv.attention_prefill(d(q), n_head, pos0, out)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
    finally:
        kv.free()
    k, ks = ora.kv_quantize_rows(kf)
    v, vs = ora.kv_quantize_rows(vf)
    kd = (k.astype(np.float32) * ks[:, None]).astype(np.float64)
    vd = (v.astype(np.float32) * vs[:, None]).astype(np.float64)
    assert np.all(np.isfinite(got))
    for i in sorted(set([0, 1, n_q // 3, n_q // 2, n_q - 2, n_q - 1] + list(range(0, n_q, 37)))):
        seq = pos0 + i + 1
        ref = ora.attention_int8(q[i], k[:seq], ks[:seq], v[:seq], vs[:seq], seq, n_head, n_kv, hd)
        ex = exact_attention(q[i], kd[:seq], vd[:seq], n_head, n_kv, hd)
        assert parity(got[i], ref, ex), (i, rel_err(got[i], ref), rel_err(ref, ex), rel_err(got[i], ex))


def test_tensor_core_and_per_query_kernels_agree(ctx, monkeypatch):
    rng = np.random.default_rng(5)
    n_head, n_kv, hd, pos0, n_q = 32, 8, 128, 64, 384
    L = pos0 + n_q
    kv = ssdllm.KvCache(ctx, L, n_kv, hd)
    try:
        kv.append_rows(d(rng.standard_normal((L, n_kv * hd)).astype(np.float32)),
                       d(rng.standard_normal((L, n_kv * hd)).astype(np.float32)), 0)
        q = d(rng.standard_normal((n_q, n_head * hd)).astype(np.float32))
        outs = []
        for env in (None, "decode"):
            if env:
                monkeypatch.setenv("SSD_PREFILL_ATTN", env)
            o = torch.zeros(n_q, n_head * hd, device=DEV)
            kv.attention_prefill(q, n_head, pos0, o)
            torch.cuda.synchronize()
            outs.append(o.cpu().numpy())
    finally:
        kv.free()
    assert normwise(outs[0], outs[1]) <= 1e-5
