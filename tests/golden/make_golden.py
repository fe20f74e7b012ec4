"""Generates tests/golden/golden.npz: golden vectors for the quantized hot path.

An independent pure-Python restatement of the reference's CPU functions (every
float operation done on numpy.float32 scalars in the reference's order), used to
pin the C oracle bit for bit. The reference (Rust) cannot be built or imported
in this environment, and ships no fixtures; these vectors follow its code:

* f16 -> f32 decode (half crate, src/metal/compute.rs:2244-2247), all 65536 codes
* dequantize_q4_0 / dequantize_q8_0 (src/ssd/streamer.rs:128-180)
* Q4_K element formula (src/metal/compute.rs:718-744)
* matvec_q4_0_cpu / matvec_q8_0_cpu / matvec_q4_k_cpu (compute.rs:680-750, :904-925)
* matvec_f32_simd_scalar (compute.rs:390-424), rmsnorm_f32_fast_scalar (:580-588)
* QuantizedVec::quantize (src/inference/quantized_kv_cache.rs:23-41)
* argmax, last index on ties (src/inference/sampler.rs:572-578)
* the builder's Q4_0 / Q8_0 / Q4_K quantizers (inverses of the decoders above)

Run:  python tests/golden/make_golden.py   (seconds; writes golden.npz beside it)
"""
from __future__ import annotations

import math
import os
import struct

import numpy as np

F = np.float32


def f16_to_f32(code: int) -> F:
    return F(struct.unpack("<e", struct.pack("<H", code))[0])


def f32_to_f16(v: F) -> int:
    return struct.unpack("<H", struct.pack("<e", float(v)))[0]  # RNE


def round_half_away(v: F) -> float:
    a = math.floor(abs(float(v)) + 0.5)  # exact in float64 for any float32 v
    return -a if v < 0 else a


# ------------------------------------------------------------- quantizers
def quant_q4_0(x: np.ndarray) -> bytes:
    out = bytearray()
    for b in range(x.size // 32):
        blk = x[b * 32:(b + 1) * 32]
        amax, m = F(0), F(0)
        for v in blk:
            if abs(v) > amax:
                amax, m = abs(v), v
        d = F(m / F(-8))
        idv = F(F(1) / d) if d != 0 else F(0)
        out += struct.pack("<H", f32_to_f16(d))
        for j in range(16):
            qs = []
            for t in range(2):
                tt = F(F(blk[2 * j + t] * idv) + F(8.5))
                q = int(math.floor(float(tt)))
                qs.append(min(15, max(0, q)))
            out.append(qs[0] | (qs[1] << 4))
    return bytes(out)


def quant_q8_0(x: np.ndarray) -> bytes:
    out = bytearray()
    for b in range(x.size // 32):
        blk = x[b * 32:(b + 1) * 32]
        amax = F(0)
        for v in blk:
            amax = max(amax, abs(v))
        d = F(amax / F(127))
        idv = F(F(1) / d) if d != 0 else F(0)
        out += struct.pack("<H", f32_to_f16(d))
        for v in blk:
            q = int(round_half_away(F(v * idv)))
            out += struct.pack("<b", min(127, max(-127, q)))
    return bytes(out)


def quant_q4_k(x: np.ndarray) -> bytes:
    out = bytearray()
    for b in range(x.size // 256):
        blk = x[b * 256:(b + 1) * 256]
        scale, mins = [], []
        for s in range(8):
            lo, hi = F(0), F(0)
            for v in blk[s * 32:(s + 1) * 32]:
                lo = min(lo, v)
                hi = max(hi, v)
            scale.append(F(F(hi - lo) / F(15)))
            mins.append(F(-lo))
        dh = f32_to_f16(F(max(scale) / F(63)))
        mh = f32_to_f16(F(max(mins) / F(63)))
        d, dmin = f16_to_f32(dh), f16_to_f32(mh)
        sc6 = [min(63, max(0, int(round_half_away(F(scale[s] / d))))) if d > 0 else 0
               for s in range(8)]
        m6 = [min(63, max(0, int(round_half_away(F(mins[s] / dmin))))) if dmin > 0 else 0
              for s in range(8)]
        sc = [0] * 12
        for s in range(4):
            sc[s] = (sc6[s] & 0x3F) | ((sc6[s + 4] & 3) << 6)
            sc[s + 4] = (m6[s] & 0x3F) | ((m6[s + 4] & 3) << 6)
            sc[s + 8] = (sc6[s + 4] >> 2) | ((m6[s + 4] >> 2) << 4)
        out += struct.pack("<HH", dh, mh) + bytes(sc)
        for s in range(8):
            es, em = F(d * F(sc6[s])), F(dmin * F(m6[s]))
            for j in range(16):
                qs = []
                for t in range(2):
                    v = blk[s * 32 + 2 * j + t]
                    q = int(round_half_away(F(F(v + em) / es))) if es > 0 else 0
                    qs.append(min(15, max(0, q)))
                out.append(qs[0] | (qs[1] << 4))
    return bytes(out)


# ------------------------------------------------------------- decoders
def q4k_scale_min(sc, sb):
    if sb < 4:
        return sc[sb] & 0x3F, sc[sb + 4] & 0x3F
    return ((sc[sb - 4] >> 6) | ((sc[sb + 4] & 0x0F) << 2),
            (sc[sb] >> 6) | ((sc[sb + 4] >> 4) << 2))


def deq(w: bytes, wtype: int, n: int) -> np.ndarray:
    out = np.zeros(n, dtype=F)
    if wtype == 2:
        for b in range(n // 32):
            blk = w[b * 18:(b + 1) * 18]
            s = f16_to_f32(blk[0] | (blk[1] << 8))
            for j in range(16):
                out[b * 32 + 2 * j] = F(F((blk[2 + j] & 15) - 8) * s)
                out[b * 32 + 2 * j + 1] = F(F((blk[2 + j] >> 4) - 8) * s)
    elif wtype == 8:
        for b in range(n // 32):
            blk = w[b * 34:(b + 1) * 34]
            s = f16_to_f32(blk[0] | (blk[1] << 8))
            for j in range(32):
                out[b * 32 + j] = F(F(struct.unpack("<b", blk[2 + j:3 + j])[0]) * s)
    elif wtype == 12:
        for b in range(n // 256):
            blk = w[b * 144:(b + 1) * 144]
            d = f16_to_f32(blk[0] | (blk[1] << 8))
            dmin = f16_to_f32(blk[2] | (blk[3] << 8))
            sc, qs = blk[4:16], blk[16:]
            for sb in range(8):
                s, m = q4k_scale_min(sc, sb)
                scale, mn = F(d * F(s)), F(dmin * F(m))
                for j in range(16):
                    byte = qs[sb * 16 + j]
                    out[b * 256 + sb * 32 + 2 * j] = F(F(scale * F(byte & 15)) - mn)
                    out[b * 256 + sb * 32 + 2 * j + 1] = F(F(scale * F(byte >> 4)) - mn)
    return out


def matvec(w: bytes, x: np.ndarray, out_dim: int, in_dim: int, wtype: int) -> np.ndarray:
    y = np.zeros(out_dim, dtype=F)
    if wtype == 2:
        rb = in_dim // 32 * 18
        for r in range(out_dim):
            s = F(0)
            for b in range(in_dim // 32):
                blk = w[r * rb + b * 18:r * rb + (b + 1) * 18]
                sc = f16_to_f32(blk[0] | (blk[1] << 8))
                for j in range(16):
                    lo, hi = F((blk[2 + j] & 15) - 8), F((blk[2 + j] >> 4) - 8)
                    s = F(s + F(F(sc * lo) * x[b * 32 + 2 * j]))
                    s = F(s + F(F(sc * hi) * x[b * 32 + 2 * j + 1]))
            y[r] = s
    elif wtype == 8:
        rb = in_dim // 32 * 34
        for r in range(out_dim):
            s = F(0)
            for b in range(in_dim // 32):
                blk = w[r * rb + b * 34:r * rb + (b + 1) * 34]
                sc = f16_to_f32(blk[0] | (blk[1] << 8))
                for j in range(32):
                    q = F(struct.unpack("<b", blk[2 + j:3 + j])[0])
                    s = F(s + F(F(sc * q) * x[b * 32 + j]))
            y[r] = s
    elif wtype == 12:
        rb = in_dim // 256 * 144
        for r in range(out_dim):
            s = F(0)
            for b in range(in_dim // 256):
                blk = w[r * rb + b * 144:r * rb + (b + 1) * 144]
                d = f16_to_f32(blk[0] | (blk[1] << 8))
                dmin = f16_to_f32(blk[2] | (blk[3] << 8))
                sc, qs = blk[4:16], blk[16:]
                for sb in range(8):
                    a, m = q4k_scale_min(sc, sb)
                    scale, mn = F(d * F(a)), F(dmin * F(m))
                    for j in range(16):
                        byte = qs[sb * 16 + j]
                        v0 = F(F(scale * F(byte & 15)) - mn)
                        v1 = F(F(scale * F(byte >> 4)) - mn)
                        xi = b * 256 + sb * 32 + 2 * j
                        s = F(s + F(F(v0 * x[xi]) + F(v1 * x[xi + 1])))
            y[r] = s
    return y


def matvec_f32(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    out_dim, in_dim = w.shape
    y = np.zeros(out_dim, dtype=F)
    for r in range(out_dim):
        acc = [F(0)] * 4
        for c in range(in_dim // 4):
            for t in range(4):
                acc[t] = F(acc[t] + F(w[r, 4 * c + t] * x[4 * c + t]))
        for j in range(in_dim % 4):
            i = in_dim // 4 * 4 + j
            acc[0] = F(acc[0] + F(w[r, i] * x[i]))
        y[r] = F(F(F(acc[0] + acc[1]) + acc[2]) + acc[3])
    return y


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: F) -> np.ndarray:
    ss = F(0)
    for v in x:
        ss = F(ss + F(v * v))
    inv = F(F(1) / F(np.sqrt(F(F(ss / F(x.size)) + eps))))
    return np.array([F(v * F(inv * wi)) for v, wi in zip(x, w)], dtype=F)


def kv_quantize(v: np.ndarray):
    absmax = F(0)
    for a in v:
        absmax = max(absmax, abs(a))
    if absmax == 0:
        return np.zeros(v.size, np.int8), F(0)
    inv = F(F(127) / absmax)
    scale = F(absmax / F(127))
    q = np.array([min(127, max(-127, round_half_away(F(a * inv)))) for a in v], dtype=np.int8)
    return q, scale


def argmax(v: np.ndarray) -> int:
    best = 0
    for i in range(1, v.size):
        if not (v[i] < v[best]):
            best = i
    return best


def main():
    rng = np.random.default_rng(20261201)
    g = {}
    codes = np.arange(65536, dtype=np.uint16)
    g["f16_codes"] = codes
    g["f16_values"] = codes.view(np.float16).astype(np.float32)  # exact widening
    # One seeded case per quantized format: weights N(0, 0.02), x N(0, 1).
    for name, wtype, rows, cols, qf in (("q4_0", 2, 6, 128, quant_q4_0),
                                        ("q8_0", 8, 5, 96, quant_q8_0),
                                        ("q4_k", 12, 4, 512, quant_q4_k)):
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(F)
        x = rng.standard_normal(cols).astype(F)
        packed = b"".join(qf(w[r]) for r in range(rows))
        g[f"{name}_w"] = w
        g[f"{name}_x"] = x
        g[f"{name}_packed"] = np.frombuffer(packed, dtype=np.uint8)
        g[f"{name}_deq"] = deq(packed, wtype, rows * cols)
        g[f"{name}_y"] = matvec(packed, x, rows, cols, wtype)
    # Edge blocks: all-zero block, +/- extreme, a block whose max magnitude is negative.
    edge = np.zeros((1, 256), dtype=F)
    edge[0, 32:64] = np.linspace(-1, 1, 32, dtype=F)
    edge[0, 64:96] = F(-3.0)
    edge[0, 96] = F(5.0)
    edge[0, 128:160] = np.linspace(0.1, 2.0, 32, dtype=F)
    g["edge_w"] = edge
    for name, qf in (("q4_0", quant_q4_0), ("q8_0", quant_q8_0), ("q4_k", quant_q4_k)):
        g[f"edge_{name}_packed"] = np.frombuffer(qf(edge[0]), dtype=np.uint8)
    wf = rng.standard_normal((7, 37)).astype(F)
    xf = rng.standard_normal(37).astype(F)
    g["f32_w"], g["f32_x"], g["f32_y"] = wf, xf, matvec_f32(wf, xf)
    xn = rng.standard_normal(48).astype(F)
    wn = (rng.random(48) + 0.5).astype(F)
    g["rms_x"], g["rms_w"], g["rms_y"] = xn, wn, rmsnorm(xn, wn, F(1e-5))
    kv = rng.standard_normal((3, 64)).astype(F)
    kv[1] = 0
    qs, ss = zip(*(kv_quantize(r) for r in kv))
    g["kv_x"], g["kv_q"], g["kv_scale"] = kv, np.stack(qs), np.array(ss, dtype=F)
    am = np.array([0.5, 2.0, -1.0, 2.0, 1.0, 2.0, 0.0], dtype=F)
    g["argmax_v"], g["argmax_i"] = am, np.array([argmax(am)], dtype=np.int64)
    np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz"),
                        **g)


if __name__ == "__main__":
    main()
