"""Pins the oracle's Q6_K restatement (matvec_q6_k_cpu, src/metal/compute.rs:752-790).

The reference has no Q6_K known-answer test, so these are derived from the function's own
definition: a pure-Python float32 re-run of its loop (bit-exact: same operation order),
hand-built blocks whose results follow from the layout (ql[128] low nibbles, qh[64] 2-bit
high parts, 16 int8 scales, f16 d at byte 208, q = (high2 << 4 | low4) - 32), and the
element order of both bit fields.
"""
import numpy as np
import pytest

from oracle import oracle as ora


def f16_bytes(v: float) -> list:
    h = ora.lib().ora_f32_to_f16(v)
    return [h & 0xFF, h >> 8]


def block(ql, qh, scales, d):
    b = np.zeros(210, np.uint8)
    b[:128] = ql
    b[128:192] = qh
    b[192:208] = np.asarray(scales, np.int8).view(np.uint8)
    b[208:210] = f16_bytes(d)
    return b


def ref_loop(raw, x, rows, cols):
    """compute.rs:753-790 step by step in float32 (sum += sc * q * x, element order)."""
    f32 = np.float32
    y = np.zeros(rows, np.float32)
    bpr = cols // 256
    for r in range(rows):
        s = f32(0.0)
        for b in range(bpr):
            blk = raw[r, b * 210:(b + 1) * 210]
            d = f32(ora.lib().ora_f16_to_f32(int(blk[208]) | (int(blk[209]) << 8)))
            for sb in range(16):
                sc = f32(d * f32(np.int8(blk[192 + sb].view(np.int8))))
                for j in range(16):
                    idx = sb * 16 + j
                    qlb = int(blk[idx // 2])
                    low4 = (qlb >> 4) & 15 if idx & 1 else qlb & 15
                    high2 = (int(blk[128 + idx // 4]) >> ((idx % 4) * 2)) & 3
                    q = f32(((high2 << 4) | low4) - 32)
                    s = f32(s + f32(f32(sc * q) * x[b * 256 + idx]))
        y[r] = s
    return y


def test_row_bytes():
    assert ora.row_bytes(ora.Q6_K, 256) == 210 and ora.row_bytes(ora.Q6_K, 4096) == 16 * 210


def test_matvec_matches_reference_loop_bitexact():
    rng = np.random.default_rng(61)
    rows, cols = 3, 512
    raw = rng.integers(0, 256, (rows, cols // 256 * 210), dtype=np.uint8)
    for r in range(rows):
        for b in range(cols // 256):
            raw[r, b * 210 + 208:b * 210 + 210] = f16_bytes(float(rng.uniform(0.001, 0.05)))
    x = rng.standard_normal(cols).astype(np.float32)
    y = ora.matvec_quantized(raw, x, rows, cols, ora.Q6_K)
    assert np.array_equal(y, ref_loop(raw, x, rows, cols))


def test_kat_all_zero_weights():
    """low4 = 0, high2 = 2: q = 32 - 32 = 0 everywhere."""
    b = block([0x00] * 128, [0xAA] * 64, [7] * 16, 1.0)
    y = ora.matvec_quantized(b, np.ones(256, np.float32), 1, 256, ora.Q6_K)
    assert y[0] == 0.0


def test_kat_all_ones_sum_256():
    """low4 = 1, high2 = 2: q = 33 - 32 = 1; scale 1, d 1: every weight is 1."""
    b = block([0x11] * 128, [0xAA] * 64, [1] * 16, 1.0)
    y = ora.matvec_quantized(b, np.ones(256, np.float32), 1, 256, ora.Q6_K)
    assert y[0] == 256.0


def test_kat_one_sub_block_scaled():
    """low4 = high2 = 0: q = -32; only sub-block 0 has a scale (2), d = 0.5:
    16 weights of 0.5 * 2 * -32 = -32, the rest 0."""
    sc = [0] * 16
    sc[0] = 2
    b = block([0x00] * 128, [0x00] * 64, sc, 0.5)
    w = ora.dequantize(b, ora.Q6_K, 256)
    assert np.all(w[:16] == -32.0) and np.all(w[16:] == 0.0)
    y = ora.matvec_quantized(b, np.ones(256, np.float32), 1, 256, ora.Q6_K)
    assert y[0] == -512.0


@pytest.mark.parametrize("idx", [0, 1, 5, 6, 31, 32, 127, 128, 255])
def test_element_order_of_both_fields(idx):
    """Element idx takes the low nibble (idx even) or high nibble (odd) of ql[idx / 2] and
    bits 2 (idx % 4) of qh[idx / 4]: set low4 = 5, high2 = 3 for idx alone."""
    ql = np.zeros(128, np.uint8)
    qh = np.full(64, 0xAA, np.uint8)  # high2 = 2 -> q = low4 for every other element
    ql[idx // 2] |= 5 << (4 * (idx & 1))
    sh = 2 * (idx % 4)
    qh[idx // 4] = (int(qh[idx // 4]) & (0xFF ^ (3 << sh))) | (3 << sh)
    w = ora.dequantize(block(ql, qh, [1] * 16, 1.0), ora.Q6_K, 256)
    expect = np.zeros(256, np.float32)
    expect[idx] = (3 << 4 | 5) - 32  # 21
    assert np.array_equal(w, expect)


def test_dequant_agrees_with_matvec():
    rng = np.random.default_rng(62)
    raw = rng.integers(0, 256, (1, 4 * 210), dtype=np.uint8)
    for b in range(4):
        raw[0, b * 210 + 208:b * 210 + 210] = f16_bytes(0.01)
    x = rng.standard_normal(1024).astype(np.float32)
    w = ora.dequantize(raw, ora.Q6_K, 1024)
    y = ora.matvec_quantized(raw, x, 1, 1024, ora.Q6_K)
    assert abs(float(y[0]) - float(np.dot(w.astype(np.float64), x))) <= 1e-4 * np.abs(w * x).sum()


def test_library_row_bytes_matches_oracle():
    """The library's host-side size rule (no GPU needed) agrees with the oracle's."""
    import ssdllm
    for cols in (256, 4096, 11008 // 256 * 256):
        assert ssdllm.row_bytes(ora.Q6_K, cols) == ora.row_bytes(ora.Q6_K, cols)
    assert ssdllm.row_bytes(ora.Q6_K, 128) == 0  # not a whole super-block
