"""Pins the oracle's Q5_K restatement (matvec_q5_k_cpu, src/metal/compute.rs:845-899).

The reference's own known-answer tests (compute.rs:2400-2412 zero scales, :2435-2455 one
scaled sub-block), a pure-Python float32 re-run of its loop (bit-exact: same operation
order), and the element order of the two bit fields (ql low nibbles per sub-block, qh
high bits at bit idx % 8 of byte idx / 8).
"""
import numpy as np
import pytest

from oracle import oracle as ora


def f16_bytes(v: float) -> list:
    h = ora.lib().ora_f32_to_f16(v)
    return [h & 0xFF, h >> 8]


def scale_min(sc, sb):
    """compute.rs:865-873 (the Q4_K packing)."""
    if sb < 4:
        return sc[sb] & 0x3F, sc[sb + 4] & 0x3F
    return ((sc[sb - 4] >> 6) | ((sc[sb + 4] & 0x0F) << 2),
            (sc[sb] >> 6) | ((sc[sb + 4] >> 4) << 2))


def ref_loop(raw, x, rows, cols):
    """compute.rs:851-897 step by step in float32."""
    f32 = np.float32
    y = np.zeros(rows, np.float32)
    for r in range(rows):
        s = f32(0.0)
        for b in range(cols // 256):
            blk = [int(v) for v in raw[r, b * 176:(b + 1) * 176]]
            d = f32(ora.lib().ora_f16_to_f32(blk[0] | (blk[1] << 8)))
            dmin = f32(ora.lib().ora_f16_to_f32(blk[2] | (blk[3] << 8)))
            sc, qh, ql = blk[4:16], blk[16:48], blk[48:176]
            for sb in range(8):
                s6, m6 = scale_min(sc, sb)
                scale, mn = f32(d * f32(s6)), f32(dmin * f32(m6))
                for j in range(16):
                    i0 = sb * 32 + 2 * j
                    bv = ql[sb * 16 + j]
                    q0 = (bv & 15) | (((qh[i0 // 8] >> (i0 % 8)) & 1) << 4)
                    q1 = ((bv >> 4) & 15) | (((qh[(i0 + 1) // 8] >> ((i0 + 1) % 8)) & 1) << 4)
                    v0 = f32(f32(scale * f32(q0)) - mn)
                    v1 = f32(f32(scale * f32(q1)) - mn)
                    s = f32(s + f32(f32(v0 * x[b * 256 + i0]) + f32(v1 * x[b * 256 + i0 + 1])))
        y[r] = s
    return y


def test_row_bytes():
    assert ora.row_bytes(ora.Q5_K, 256) == 176 and ora.row_bytes(ora.Q5_K, 4096) == 16 * 176


def test_kat_zero_scales_give_zero():
    """compute.rs:2400-2412: d = 1, everything else 0."""
    block = np.zeros(176, np.uint8)
    block[0:2] = f16_bytes(1.0)
    y = ora.matvec_quantized(block, np.ones(256, np.float32), 1, 256, ora.Q5_K)
    assert abs(y[0]) < 1e-5


def test_kat_one_scaled_sub_block_is_32():
    """compute.rs:2435-2455: d = 1, sc[0] = 1, ql of sub-block 0 all 0x11, qh 0."""
    block = np.zeros(176, np.uint8)
    block[0:2] = f16_bytes(1.0)
    block[4] = 0x01
    block[48:64] = 0x11
    y = ora.matvec_quantized(block, np.ones(256, np.float32), 1, 256, ora.Q5_K)
    assert abs(y[0] - 32.0) < 1e-3


def test_matvec_matches_reference_loop_bitexact():
    rng = np.random.default_rng(81)
    rows, cols = 3, 512
    raw = rng.integers(0, 256, (rows, cols // 256 * 176), dtype=np.uint8)
    for r in range(rows):
        for b in range(cols // 256):
            raw[r, b * 176:b * 176 + 2] = f16_bytes(float(rng.uniform(0.001, 0.01)))
            raw[r, b * 176 + 2:b * 176 + 4] = f16_bytes(float(rng.uniform(0.001, 0.01)))
    x = rng.standard_normal(cols).astype(np.float32)
    y = ora.matvec_quantized(raw, x, rows, cols, ora.Q5_K)
    assert np.array_equal(y, ref_loop(raw, x, rows, cols))


@pytest.mark.parametrize("idx", [0, 1, 7, 8, 31, 32, 100, 255])
def test_element_order_of_both_fields(idx):
    """Element idx: nibble (idx odd: high) of ql[16 (idx / 32) + (idx % 32) / 2], high bit
    at bit idx % 8 of qh[idx / 8]. Scale 1 in every sub-block (sc[0..3] = 0x41: low 6 bits
    1 for sub-blocks 0-3, top 2 bits 1 for 4-7; sc[8..11] = 0), d = 1, dmin = 0."""
    block = np.zeros(176, np.uint8)
    block[0:2] = f16_bytes(1.0)
    block[4:8] = 0x41
    block[8:12] = 0x01
    block[48 + (idx // 32) * 16 + (idx % 32) // 2] |= 5 << (4 * (idx & 1))
    block[16 + idx // 8] |= 1 << (idx % 8)
    w = ora.dequantize(block, ora.Q5_K, 256)
    expect = np.zeros(256, np.float32)
    expect[idx] = 16 + 5
    assert np.array_equal(w, expect)
