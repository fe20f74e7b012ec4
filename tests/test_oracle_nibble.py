"""Known answers that pin the oracle's nibble order (the reference ships none: its Q4_0
test, all 0x88 -> 0, gives the same answer under any order). Element 2j of a 32-weight
block is the low nibble of byte j and element 2j+1 its high nibble, as all three statements
of the format in the reference read it (src/metal/compute.rs:693-699,
src/ssd/streamer.rs:167-173, src/metal/shaders/kernels.metal:190-196); Q4_K sub-block sb
reads bytes 16 sb .. 16 sb + 15 the same way (src/metal/compute.rs:718-744). The answers are
derived by hand below; the same blocks run on the GPU in test_gpu_headline.py."""
import numpy as np

from oracle import oracle as ora


def q4_0_block(d, nibbles):
    b = np.zeros(18, np.uint8)
    b[0:2] = np.frombuffer(np.float16(d).tobytes(), np.uint8)
    for j in range(16):
        b[2 + j] = (nibbles[2 * j] & 15) | ((nibbles[2 * j + 1] & 15) << 4)
    return b


def test_q4_0_low_nibble_is_the_even_element():
    # byte 0 = 0x21: element 0 = 1 - 8 = -7, element 1 = 2 - 8 = -6; other nibbles 8 (zero)
    nib = [8] * 32
    nib[0], nib[1] = 1, 2
    raw = np.concatenate([q4_0_block(1.0, nib), q4_0_block(0.5, [9] * 32)]).reshape(2, 18)
    x = np.zeros(32, np.float32)
    x[0], x[1], x[16] = 1.0, 10.0, 1000.0
    y = ora.matvec_quantized(raw, x, 2, 32, ora.Q4_0)
    assert y[0] == -7.0 * 1.0 + -6.0 * 10.0  # -67; a j / j+16 split would read -7
    assert y[1] == np.float32(0.5) * (1.0 + 10.0 + 1000.0)
    deq = ora.dequantize(raw, ora.Q4_0, 64)
    assert deq[0] == -7.0 and deq[1] == -6.0 and deq[16] == 0.0


def test_q4_k_sub_block_bytes_and_nibbles():
    blk = np.zeros(144, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)   # d
    blk[2:4] = np.frombuffer(np.float16(0.0).tobytes(), np.uint8)   # dmin
    blk[4:8] = 1       # 6-bit scales of sub-blocks 0-3 = 1, mins 0 (bytes 8-11 zero)
    blk[12:16] = 0x01  # sub-blocks 4-7: scale (0 >> 6) | (1 << 2) = 4, min 0
    blk[16 + 48] = 0x5A  # sub-block 3, byte 0: elements 96, 97 = 10, 5
    x = np.zeros(256, np.float32)
    x[96], x[97], x[112] = 2.0, 3.0, 100.0
    y = ora.matvec_quantized(blk.reshape(1, 144), x, 1, 256, ora.Q4_K)
    assert y[0] == 10 * 2.0 + 5 * 3.0
    deq = ora.dequantize(blk, ora.Q4_K, 256)
    assert deq[96] == 10.0 and deq[97] == 5.0 and np.count_nonzero(deq) == 2
