"""Pins the oracle's Q8_K restatement (matvec_q8_k_cpu, src/metal/compute.rs:971-993) with
the reference's own known-answer tests (compute.rs:2520-2555) and a float32 re-run of its
loop (bit-exact: same operation order)."""
import numpy as np

from oracle import oracle as ora


def block(d, q):
    b = np.zeros(292, np.uint8)
    b[0:4] = np.frombuffer(np.float32(d).tobytes(), np.uint8)
    b[4:260] = np.asarray(q, np.int8).view(np.uint8)
    return b


def test_row_bytes():
    assert ora.row_bytes(ora.Q8_K, 256) == 292 and ora.row_bytes(ora.Q8_K, 4096) == 16 * 292


def test_kat_ones_sum_256():
    """compute.rs:2520-2535: d = 1, every q = 1."""
    y = ora.matvec_quantized(block(1.0, [1] * 256), np.ones(256, np.float32), 1, 256, ora.Q8_K)
    assert abs(y[0] - 256.0) < 1e-3


def test_kat_negative():
    """compute.rs:2538-2555: d = 0.5, every q = -2."""
    y = ora.matvec_quantized(block(0.5, [-2] * 256), np.ones(256, np.float32), 1, 256, ora.Q8_K)
    assert abs(y[0] + 256.0) < 1e-3


def test_matvec_matches_reference_loop_bitexact():
    rng = np.random.default_rng(101)
    rows, cols = 3, 768
    raw = rng.integers(0, 256, (rows, cols // 256 * 292), dtype=np.uint8)
    ds = rng.uniform(1e-3, 1e-2, (rows, cols // 256)).astype(np.float32)
    for r in range(rows):
        for b in range(cols // 256):
            raw[r, b * 292:b * 292 + 4] = np.frombuffer(ds[r, b].tobytes(), np.uint8)
    x = rng.standard_normal(cols).astype(np.float32)
    f32 = np.float32
    ref = np.zeros(rows, np.float32)
    for r in range(rows):
        s = f32(0.0)
        for b in range(cols // 256):
            q = raw[r, b * 292 + 4:b * 292 + 260].view(np.int8)
            for j in range(256):
                s = f32(s + f32(f32(ds[r, b] * f32(q[j])) * x[b * 256 + j]))
        ref[r] = s
    assert np.array_equal(ora.matvec_quantized(raw, x, rows, cols, ora.Q8_K), ref)
    w = ora.dequantize(raw, ora.Q8_K, rows * cols).reshape(rows, cols)
    assert np.array_equal(w[1, 256:512], ds[1, 1] * raw[1, 296:552].view(np.int8).astype(np.float32))
