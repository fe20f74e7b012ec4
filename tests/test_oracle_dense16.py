"""Pins the oracle's 16-bit dense matvecs (matvec_f16_cpu src/metal/compute.rs:2272-2285,
matvec_bf16_cpu :2256-2269, bf16_to_f32 :2250-2253) with the reference's own known-answer
tests (compute.rs:2979-3040)."""
import numpy as np

from oracle import oracle as ora


def mv(w, x, rows, cols, t):
    return ora.matvec_quantized(np.array(w, np.uint8), np.array(x, np.float32), rows, cols, t)


def test_kat_bf16_conversion():
    """compute.rs:2979-2984"""
    v = ora.dequantize(np.array([0x80, 0x3F, 0x00, 0xC0, 0x00, 0x00], np.uint8), ora.BF16, 3)
    assert list(v) == [1.0, -2.0, 0.0]


def test_kat_bf16_identity_and_dispatch():
    """compute.rs:2988-3012"""
    y = mv([0x80, 0x3F, 0x00, 0x00, 0x00, 0x00, 0x80, 0x3F], [3.0, 7.0], 2, 2, ora.BF16)
    assert abs(y[0] - 3.0) < 1e-2 and abs(y[1] - 7.0) < 1e-2
    y = mv([0x80, 0x3F, 0x00, 0x40, 0x40, 0x40, 0x80, 0x40], [1.0, 1.0], 2, 2, ora.BF16)
    assert abs(y[0] - 3.0) < 1e-2 and abs(y[1] - 7.0) < 1e-2


def test_kat_f16_identity_and_dispatch():
    """compute.rs:3015-3040"""
    y = mv([0x00, 0x3C, 0x00, 0x00, 0x00, 0x00, 0x00, 0x3C], [5.0, 9.0], 2, 2, ora.F16)
    assert abs(y[0] - 5.0) < 1e-2 and abs(y[1] - 9.0) < 1e-2
    y = mv([0x00, 0x3C, 0x00, 0x40, 0x00, 0x42, 0x00, 0x44], [1.0, 1.0], 2, 2, ora.F16)
    assert abs(y[0] - 3.0) < 1e-2 and abs(y[1] - 7.0) < 1e-2


def test_bf16_matvec_is_sequential_float32():
    rng = np.random.default_rng(121)
    rows, cols = 3, 37
    raw = rng.integers(0, 256, (rows, cols * 2), dtype=np.uint8)
    raw[:, 1::2] = rng.integers(0x3C, 0x40, (rows, cols), dtype=np.uint8)  # moderate exponents
    x = rng.standard_normal(cols).astype(np.float32)
    w = ora.dequantize(raw, ora.BF16, rows * cols).reshape(rows, cols)
    ref = np.zeros(rows, np.float32)
    for r in range(rows):
        s = np.float32(0)
        for c in range(cols):
            s = np.float32(s + np.float32(w[r, c] * x[c]))
        ref[r] = s
    assert np.array_equal(ora.matvec_quantized(raw, x, rows, cols, ora.BF16), ref)
