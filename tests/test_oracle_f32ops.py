"""CPU pins of the oracle's f32 windowed attention (flash_attention_f32,
src/metal/shaders/kernels.metal:1360-1440 / flash_attention_windowed,
src/inference/flash_attention.rs:146-229) and SwiGLU feed-forward
(src/inference/feed_forward.rs:17-43): the reference's own test inputs with their
assertions, and an fp64 restatement on random inputs."""
import numpy as np
import pytest

from oracle import oracle as ora


def attn64(q, k, v, n_head, n_head_kv, head_dim, seq_len, ws, we):
    q = np.asarray(q, np.float64).reshape(n_head, head_dim)
    k = np.asarray(k, np.float64).reshape(-1, n_head_kv, head_dim)
    v = np.asarray(v, np.float64).reshape(-1, n_head_kv, head_dim)
    end = min(we, seq_len)
    out = np.zeros((n_head, head_dim))
    g = max(n_head // n_head_kv, 1)
    for h in range(n_head):
        if end <= ws:
            continue
        s = k[ws:end, h // g] @ q[h] / np.sqrt(head_dim)
        p = np.exp(s - s.max())
        out[h] = p @ v[ws:end, h // g] / p.sum()
    return out.ravel()


def ffn64(x, wg, wu, wd, n_embd, n_ff):
    x = np.asarray(x, np.float64)
    g = np.asarray(wg, np.float64).reshape(n_ff, n_embd) @ x
    u = np.asarray(wu, np.float64).reshape(n_ff, n_embd) @ x
    return np.asarray(wd, np.float64).reshape(n_embd, n_ff) @ (g / (1 + np.exp(-g)) * u)


def test_single_position_returns_v():
    """One position: softmax of one score is 1, the output is that V row
    (flash_attention.rs:414-457 compares against the standard path on one token)."""
    rng = np.random.default_rng(0)
    q = rng.standard_normal(8).astype(np.float32)
    k = rng.standard_normal(8).astype(np.float32)
    v = rng.standard_normal(8).astype(np.float32)
    out = ora.flash_attention_f32(q, k, v, 2, 2, 4, 1, 0, 1)
    assert np.allclose(out, v, atol=1e-6)


def test_windowed_reference_case_is_finite():
    """flash_attention.rs:491-522: 10 cached tokens of a 2-head, head_dim-4 layer, window
    5..11 (clamped to the 10 positions)."""
    rng = np.random.default_rng(1)
    q = rng.standard_normal(8).astype(np.float32)
    k = rng.standard_normal((10, 8)).astype(np.float32)
    v = rng.standard_normal((10, 8)).astype(np.float32)
    out = ora.flash_attention_f32(q, k, v, 2, 2, 4, 10, 5, 11)
    assert np.all(np.isfinite(out))
    assert np.allclose(out, attn64(q, k, v, 2, 2, 4, 10, 5, 11), rtol=1e-5, atol=1e-6)


def test_large_scores_stay_finite():
    """flash_attention.rs:459-489: inputs of 100 must not overflow the softmax."""
    q = np.full(4, 40.0, np.float32)
    k = np.full((3, 4), 40.0, np.float32)
    v = np.full((3, 4), 2.0, np.float32)
    out = ora.flash_attention_f32(q, k, v, 1, 1, 4, 3, 0, 3)
    assert np.all(np.isfinite(out)) and np.allclose(out, 2.0)


def test_empty_window_gives_zeros():
    """kernels.metal:1430-1438: running_sum 0 -> zeros."""
    q = np.ones(8, np.float32)
    k = np.ones((4, 8), np.float32)
    out = ora.flash_attention_f32(q, k, k, 2, 1, 4, 4, 3, 3)
    assert np.all(out == 0)
    out = ora.flash_attention_f32(q, k, k, 2, 1, 4, 4, 6, 9)
    assert np.all(out == 0)


@pytest.mark.parametrize("nh,nkv,hd,seq,ws,we", [(4, 2, 4, 3, 0, 3), (8, 2, 64, 300, 17, 250),
                                                 (4, 4, 80, 40, 0, 100), (2, 1, 256, 70, 5, 70)])
def test_random_against_fp64(nh, nkv, hd, seq, ws, we):
    rng = np.random.default_rng(nh * 1000 + seq)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal((seq, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((seq, nkv * hd)).astype(np.float32)
    out = ora.flash_attention_f32(q, k, v, nh, nkv, hd, seq, ws, we)
    assert np.allclose(out, attn64(q, k, v, nh, nkv, hd, seq, ws, we), rtol=1e-4, atol=1e-5)


def test_feed_forward_reference_shapes_case():
    """feed_forward.rs:76-88: x = 1, every weight 0.1, n_embd 4, n_ff 8."""
    out = ora.feed_forward_f32(np.ones(4), np.full(32, 0.1), np.full(32, 0.1), np.full(32, 0.1),
                               4, 8)
    g = 0.4
    expect = 8 * 0.1 * (g / (1 + np.exp(-g)) * g)
    assert out.shape == (4,) and np.allclose(out, expect, rtol=1e-6)


def test_feed_forward_reference_metal_case():
    """feed_forward.rs:106-130: the inputs of the GPU-vs-CPU test, n_embd 64, n_ff 2048."""
    n_embd, n_ff = 64, 2048
    x = (np.arange(n_embd) * 0.01).astype(np.float32)
    i = np.arange(n_ff * n_embd)
    wg = (((i % 17) - 8.0) * 0.001).astype(np.float32)
    wu = (((i % 13) - 6.0) * 0.001).astype(np.float32)
    wd = (((np.arange(n_embd * n_ff) % 11) - 5.0) * 0.001).astype(np.float32)
    out = ora.feed_forward_f32(x, wg, wu, wd, n_embd, n_ff)
    assert np.allclose(out, ffn64(x, wg, wu, wd, n_embd, n_ff), rtol=1e-4, atol=1e-9)


def test_feed_forward_empty_ff_gives_zeros():
    """feed_forward.rs:25-28."""
    out = ora.feed_forward_f32(np.ones(4), np.zeros(0), np.zeros(0), np.zeros(0), 4, 0)
    assert np.all(out == 0)
