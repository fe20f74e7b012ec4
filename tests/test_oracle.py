"""Pins the CPU oracle: golden vectors (bit-exact) and the reference's own
known-answer tests, ported from the reference's inline Rust tests (cited)."""
import math
import os

import numpy as np
import pytest

from oracle import oracle as ora

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def f16_bytes(v: float) -> list:
    h = ora.lib().ora_f32_to_f16(v)
    return [h & 0xFF, h >> 8]


# ------------------------------------------------------------ golden vectors
def test_f16_decode_all_codes():
    vals = np.array([ora.lib().ora_f16_to_f32(int(c)) for c in range(65536)], dtype=np.float32)
    ref = GOLD["f16_values"]
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(vals), nan)
    assert np.array_equal(vals[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_f16_encode_round_trip():
    for c in range(0, 65536):
        if (c & 0x7C00) == 0x7C00 and (c & 0x3FF):
            continue  # NaN payloads
        v = ora.lib().ora_f16_to_f32(c)
        assert ora.lib().ora_f32_to_f16(v) == c


@pytest.mark.parametrize("name,wtype", [("q4_0", ora.Q4_0), ("q8_0", ora.Q8_0),
                                        ("q4_k", ora.Q4_K)])
def test_golden_quantize_dequant_matvec(name, wtype):
    w, x = GOLD[f"{name}_w"], GOLD[f"{name}_x"]
    rows, cols = w.shape
    packed = ora.quantize(w, wtype)
    assert np.array_equal(packed.reshape(-1), GOLD[f"{name}_packed"]), "quantizer bytes"
    deq = ora.dequantize(packed, wtype, rows * cols)
    assert np.array_equal(deq.view(np.uint32), GOLD[f"{name}_deq"].view(np.uint32))
    y = ora.matvec_quantized(packed, x, rows, cols, wtype)
    assert np.array_equal(y.view(np.uint32), GOLD[f"{name}_y"].view(np.uint32))
    y4 = ora.matvec_quantized(packed, x, rows, cols, wtype, threads=3)
    assert np.array_equal(y4.view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("name,wtype", [("q4_0", ora.Q4_0), ("q8_0", ora.Q8_0),
                                        ("q4_k", ora.Q4_K)])
def test_golden_edge_blocks(name, wtype):
    packed = ora.quantize(GOLD["edge_w"], wtype)
    assert np.array_equal(packed.reshape(-1), GOLD[f"edge_{name}_packed"])
    deq = ora.dequantize(packed, wtype, 256)
    # all-zero leading block dequantizes to exact zeros
    assert np.all(deq[:32] == 0)


def test_golden_f32_matvec_rmsnorm_kv_argmax():
    y = ora.matvec_f32(GOLD["f32_w"], GOLD["f32_x"])
    assert np.array_equal(y.view(np.uint32), GOLD["f32_y"].view(np.uint32))
    r = ora.rmsnorm(GOLD["rms_x"], GOLD["rms_w"], 1e-5)
    assert np.array_equal(r.view(np.uint32), GOLD["rms_y"].view(np.uint32))
    for i in range(GOLD["kv_x"].shape[0]):
        q, s = ora.kv_quantize(GOLD["kv_x"][i])
        assert np.array_equal(q, GOLD["kv_q"][i])
        assert np.float32(s).view(np.uint32) == GOLD["kv_scale"][i].view(np.uint32)
    assert ora.argmax(GOLD["argmax_v"]) == int(GOLD["argmax_i"][0]) == 5


# ---------------------------------------------- reference known-answer tests
def test_kat_q4_0_all_0x88_is_zero():
    """src/metal/compute.rs:2347-2366"""
    block = np.array(f16_bytes(1.0) + [0x88] * 16, dtype=np.uint8)
    y = ora.matvec_quantized(block, np.ones(32, np.float32), 1, 32, ora.Q4_0)
    assert abs(y[0]) < 1e-5


def test_kat_q8_0_ones_is_32():
    """src/metal/compute.rs:2369-2381"""
    block = np.array(f16_bytes(1.0) + [1] * 32, dtype=np.uint8)
    y = ora.matvec_quantized(block, np.ones(32, np.float32), 1, 32, ora.Q8_0)
    assert abs(y[0] - 32.0) < 1e-3


def test_kat_unsupported_type_returns_zeros():
    """src/metal/compute.rs:672-675 (zeros for unknown types)."""
    y = np.full(4, 7.0, np.float32)
    rc = ora.lib().ora_matvec_quantized(ora._u8(np.zeros(64, np.uint8)),
                                        ora._f(np.ones(32, np.float32)), 4, 32, 99, ora._f(y))
    assert rc == -1 and np.all(y == 0)


def test_kat_rmsnorm():
    """src/metal/compute.rs:2328-2336"""
    x = ora.rmsnorm(np.array([1, 2, 3, 4], np.float32), np.ones(4, np.float32), 1e-5)
    inv = 1.0 / math.sqrt((1 + 4 + 9 + 16) / 4.0 + 1e-5)
    assert abs(x[0] - inv) < 1e-4


def test_kat_softmax():
    """src/metal/compute.rs:2312-2326"""
    x = ora.softmax(np.array([1, 2, 3], np.float32))
    assert abs(x.sum() - 1.0) < 1e-5 and x[2] > x[1] > x[0]
    assert abs(ora.softmax(np.array([42.0], np.float32))[0] - 1.0) < 1e-6


def test_kat_silu():
    """src/metal/compute.rs:2338-2345"""
    x = ora.silu(np.array([0.0, 1.0, -1.0], np.float32))
    assert abs(x[0]) < 1e-6 and x[1] > 0.5 and -0.5 < x[2] < 0.0


def test_kat_fused_residual_rmsnorm():
    """src/metal/compute.rs:3055-3068 and :3071-3093 (fused == separate)."""
    x = ora.fused_residual_rmsnorm(np.array([1, 2, 3], np.float32),
                                   np.array([1, 1, 1], np.float32), np.ones(3, np.float32))
    inv = 1.0 / math.sqrt((4 + 9 + 16) / 3.0 + 1e-5)
    assert np.allclose(x, np.array([2, 3, 4]) * inv, atol=1e-5)
    x0 = np.array([0.5, -1.2, 3.7, 0.1, -2.5, 1.8, 0.3, -0.9], np.float32)
    r = np.array([0.1, 0.3, -0.5, 1.0, 0.2, -0.4, 0.8, 0.6], np.float32)
    w = np.array([1.0, 0.5, 2.0, 1.5, 0.8, 1.2, 0.3, 1.7], np.float32)
    sep = ora.rmsnorm(x0 + r, w)
    fused = ora.fused_residual_rmsnorm(x0, r, w)
    assert np.max(np.abs(sep - fused)) < 1e-5


def test_kat_post_attn_norm_matches_separate():
    """fused_post_attn_norm_f32_cpu (compute.rs:536-555) == add + rmsnorm (:3429-3456)."""
    h = np.array([0.5, -1.0, 2.0, 0.25], np.float32)
    a = np.array([0.1, 0.2, -0.3, 0.4], np.float32)
    w = np.array([1.0, 2.0, 0.5, 1.5], np.float32)
    h2, out = ora.fused_post_attn_norm(h, a, w)
    assert np.array_equal(h2, h + a)
    assert np.max(np.abs(out - ora.rmsnorm(h + a, w))) < 1e-5


def test_kat_fused_rmsnorm_linear_matches_separate():
    """compute.rs:3493-3530: fused norm+linear == rmsnorm then matvec."""
    n, vocab = 16, 8
    x = ((np.arange(n) % 5) * 0.3 - 0.6).astype(np.float32)
    nw = ((np.arange(n) % 3) * 0.2 + 0.8).astype(np.float32)
    ow = ((np.arange(vocab * n) % 11) * 0.1 - 0.5).astype(np.float32).reshape(vocab, n)
    fused = ora.fused_rmsnorm_linear(x, nw, ow, vocab, n)
    sep = ora.matvec_f32(ow, ora.rmsnorm(x, nw))
    assert np.max(np.abs(fused - sep)) < 1e-5


def test_kat_rope_multi_head_matches_single_head():
    """src/metal/compute.rs:3265-3299"""
    hd, nh, pos, theta = 4, 3, 7, 10000.0
    x = ((np.arange(nh * hd) + 1.0) * 0.5).astype(np.float32)
    y = ora.rope_multi_head(x, hd, nh, pos, theta)
    for h in range(nh):
        for i in range(hd // 2):
            freq = np.float32(1.0) / np.float32(math.pow(theta, 2.0 * i / hd))
            ang = np.float32(pos) * freq
            s, c = math.sin(ang), math.cos(ang)
            x0, x1 = x[h * hd + 2 * i], x[h * hd + 2 * i + 1]
            assert abs(y[h * hd + 2 * i] - (x0 * c - x1 * s)) < 1e-5
            assert abs(y[h * hd + 2 * i + 1] - (x0 * s + x1 * c)) < 1e-5


def test_kat_rope_position_zero_identity():
    """src/metal/compute.rs:3301-3314"""
    x = np.arange(1, 9, dtype=np.float32)
    assert np.max(np.abs(ora.rope_multi_head(x, 4, 2, 0, 10000.0) - x)) < 1e-6


def test_kat_kv_int8_round_trip_and_zero():
    """src/inference/quantized_kv_cache.rs:243-268"""
    v = ((np.arange(128) - 64.0) * 0.1).astype(np.float32)
    q, s = ora.kv_quantize(v)
    deq = np.zeros(128, np.float32)
    ora.lib().ora_kv_dequantize(ora._i8(q), s, 128, ora._f(deq))
    assert np.all(np.abs(v - deq) < s + 0.01)
    q0, s0 = ora.kv_quantize(np.zeros(64, np.float32))
    assert s0 == 0.0 and np.all(q0 == 0)


@pytest.mark.parametrize("n_head,n_head_kv", [(4, 4), (8, 2)])
def test_kat_flash_matches_standard_attention(n_head, n_head_kv):
    """src/inference/flash_attention.rs:408-460 and GQA :522 (flash == standard, 1e-4)."""
    rng = np.random.default_rng(3)
    hd, seq = 16, 37
    q = rng.standard_normal(n_head * hd).astype(np.float32)
    kf = rng.standard_normal((seq, n_head_kv * hd)).astype(np.float32)
    vf = rng.standard_normal((seq, n_head_kv * hd)).astype(np.float32)
    k, ks = ora.kv_quantize_rows(kf)
    v, vs = ora.kv_quantize_rows(vf)
    std = ora.attention_int8(q, k, ks, v, vs, seq, n_head, n_head_kv, hd)
    fl = ora.attention_int8(q, k, ks, v, vs, seq, n_head, n_head_kv, hd, flash=True)
    assert np.max(np.abs(std - fl)) < 1e-4


def test_kat_tensor_parallel_shards_match():
    """src/inference/tensor_parallel.rs:156-232: 1 vs 4 shards."""
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((50, 64)) * 0.02).astype(np.float32)
    x = rng.standard_normal(64).astype(np.float32)
    p = ora.quantize(w, ora.Q4_0)
    a = ora.matvec_quantized(p, x, 50, 64, ora.Q4_0, threads=1)
    b = ora.matvec_quantized(p, x, 50, 64, ora.Q4_0, threads=4)
    assert np.array_equal(a, b)


def test_layer_step_modes_agree():
    """forward_pass layer (transformer.rs:312-394): live f32 path vs operator path."""
    rng = np.random.default_rng(11)
    n, nh, nkv, hd, ff, pos = 64, 4, 2, 16, 96, 5

    def qw(r, c):
        return ora.quantize((rng.standard_normal((r, c)) * 0.02).astype(np.float32), ora.Q4_0)

    L = ora.Layer(n, nh, nkv, hd, ff, ora.Q4_0, qw(n, n), qw(nkv * hd, n), qw(nkv * hd, n),
                  qw(n, n), qw(ff, n), qw(ff, n), qw(n, ff),
                  (rng.random(n) + 0.5).astype(np.float32), (rng.random(n) + 0.5).astype(np.float32))
    kvd = nkv * hd
    kc = np.zeros((pos + 1, kvd), np.int8)
    vc = np.zeros((pos + 1, kvd), np.int8)
    ks = np.zeros(pos + 1, np.float32)
    vs = np.zeros(pos + 1, np.float32)
    kq, kss = ora.kv_quantize_rows(rng.standard_normal((pos, kvd)).astype(np.float32))
    vq, vss = ora.kv_quantize_rows(rng.standard_normal((pos, kvd)).astype(np.float32))
    kc[:pos], vc[:pos], ks[:pos], vs[:pos] = kq, vq, kss, vss
    h0 = rng.standard_normal(n).astype(np.float32)
    outs = []
    for mode in (0, 1):
        h = h0.copy()
        L.step(h, pos, kc.copy(), ks.copy(), vc.copy(), vs.copy(), mode=mode, threads=2)
        outs.append(h)
    rel = np.max(np.abs(outs[0] - outs[1])) / np.max(np.abs(outs[0]))
    assert rel < 1e-4
