/*
 * oracle.c — CPU restatement of ssd-llm's CPU compute path (TEST INFRASTRUCTURE ONLY).
 *
 * Parity checker for the CUDA backend; never linked into the product library.
 * Compile with -O2 -ffp-contract=off and no fast-math (oracle/Makefile): every
 * multiply and add below is one IEEE float operation in the order the reference
 * writes it (Rust does not contract a*b+c into an FMA).
 * Citations are path:line inside the reference project (quantumnic/ssd-llm).
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ f16 */

/* IEEE binary16 -> binary32, exact for every input (normals, subnormals, inf, NaN).
 * The reference calls half::f16::from_bits(..).to_f32() (src/metal/compute.rs:2244-2247,
 * src/ssd/streamer.rs:140-141), which is this exact conversion. */
float ora_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do {
                man <<= 1;
                e++;
            } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + (127 - 15)) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* binary32 -> binary16, round to nearest even (half::f16::from_f32). */
uint16_t ora_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0));
    int e = (int)exp - 127 + 15;
    if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e;
        uint32_t half_bits = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (half_bits & 1u))) half_bits++;
        return (uint16_t)(sign | half_bits);
    }
    uint32_t half_bits = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (half_bits & 1u))) half_bits++;
    return (uint16_t)(sign | half_bits);
}

static inline float rd_f16(const uint8_t* p) { return ora_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }
static inline void wr_f16(uint8_t* p, uint16_t h) {
    p[0] = (uint8_t)(h & 0xFF);
    p[1] = (uint8_t)(h >> 8);
}

size_t ora_row_bytes(int type, int64_t n) {
    switch (type) {
        case ORA_F32: return (size_t)n * 4;
        case ORA_F16:
        case ORA_BF16: return (size_t)n * 2;
        case ORA_Q4_0: return (size_t)(n / 32) * 18;
        case ORA_Q8_0: return (size_t)(n / 32) * 34;
        case ORA_Q4_K: return (size_t)(n / 256) * 144;
        case ORA_Q5_K: return (size_t)(n / 256) * 176;
        case ORA_Q6_K: return (size_t)(n / 256) * 210;
        case ORA_Q8_K: return (size_t)(n / 256) * 292;
        case ORA_Q2_K:
        case ORA_Q3_K:
        case ORA_IQ4_NL:
        case ORA_IQ4_XS:
        case ORA_IQ3_XXS:
        case ORA_IQ3_S:
        case ORA_IQ2_XXS:
        case ORA_IQ2_XS:
            return (size_t)(n / ora_lowbit_block(type)) * ora_lowbit_block_bytes(type);
        default: return 0;
    }
}

/* ----------------------------------------------------------- quantizers */
/* The reference ships no Q4_0/Q8_0/Q4_K quantizer; these are the builder's
 * quantizers, written as exact inverses of the reference decoders
 * (src/metal/compute.rs:680-750, :904-925). Both the oracle and the GPU consume
 * the same packed bytes, so dequant parity does not depend on these choices. */

/* Q4_0: d = m / -8 where m is the signed value of largest magnitude (first on ties),
 * stored as f16; q = clamp(floor(x * (1/d) + 8.5), 0, 15); element 2j is the low
 * nibble of byte j, element 2j+1 the high nibble (src/metal/compute.rs:693-699). */
void ora_quantize_q4_0(const float* w, int64_t n, uint8_t* out) {
    for (int64_t b = 0; b < n / 32; b++) {
        const float* x = w + b * 32;
        uint8_t* o = out + b * 18;
        float amax = 0.0f, m = 0.0f;
        for (int j = 0; j < 32; j++) {
            float a = fabsf(x[j]);
            if (a > amax) { amax = a; m = x[j]; }
        }
        float d = m / -8.0f;
        float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        wr_f16(o, ora_f32_to_f16(d));
        for (int j = 0; j < 16; j++) {
            float t0 = x[2 * j] * id + 8.5f;
            float t1 = x[2 * j + 1] * id + 8.5f;
            int q0 = (int)floorf(t0), q1 = (int)floorf(t1);
            q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
            q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
            o[2 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

/* Q8_0: d = amax / 127 (f16), q = round_half_away(x * (1/d)). */
void ora_quantize_q8_0(const float* w, int64_t n, uint8_t* out) {
    for (int64_t b = 0; b < n / 32; b++) {
        const float* x = w + b * 32;
        uint8_t* o = out + b * 34;
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) {
            float a = fabsf(x[j]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        wr_f16(o, ora_f32_to_f16(d));
        for (int j = 0; j < 32; j++) {
            int q = (int)roundf(x[j] * id);
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            o[2 + j] = (uint8_t)(int8_t)q;
        }
    }
}

static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Q4_K super-block (256 weights, 144 bytes): f16 d, f16 dmin, 12 bytes of 6-bit
 * (scale, min) pairs, 128 bytes of nibbles (16 per 32-wide sub-block, element 2j
 * low nibble of byte j). Decoder: src/metal/compute.rs:718-744. Per sub-block s:
 * lo = min(0, min x), hi = max(0, max x), scale_s = (hi-lo)/15, min_s = -lo;
 * d = max scale_s / 63, dmin = max min_s / 63 (f16);
 * sc_s = round(scale_s/d), m_s = round(min_s/dmin) (6 bit);
 * q = clamp(round((x + dmin*m_s) / (d*sc_s)), 0, 15). */
void ora_quantize_q4_k(const float* w, int64_t n, uint8_t* out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const float* x = w + b * 256;
        uint8_t* o = out + b * 144;
        float scale[8], mins[8];
        float max_scale = 0.0f, max_min = 0.0f;
        for (int s = 0; s < 8; s++) {
            float lo = 0.0f, hi = 0.0f;
            for (int j = 0; j < 32; j++) {
                float v = x[s * 32 + j];
                if (v < lo) lo = v;
                if (v > hi) hi = v;
            }
            scale[s] = (hi - lo) / 15.0f;
            mins[s] = -lo;
            if (scale[s] > max_scale) max_scale = scale[s];
            if (mins[s] > max_min) max_min = mins[s];
        }
        uint16_t dh = ora_f32_to_f16(max_scale / 63.0f);
        uint16_t mh = ora_f32_to_f16(max_min / 63.0f);
        float d = ora_f16_to_f32(dh), dmin = ora_f16_to_f32(mh);
        wr_f16(o, dh);
        wr_f16(o + 2, mh);
        uint8_t sc6[8], m6[8];
        for (int s = 0; s < 8; s++) {
            sc6[s] = (uint8_t)(d > 0.0f ? clampi((int)roundf(scale[s] / d), 0, 63) : 0);
            m6[s] = (uint8_t)(dmin > 0.0f ? clampi((int)roundf(mins[s] / dmin), 0, 63) : 0);
        }
        uint8_t* sc = o + 4;
        for (int s = 0; s < 4; s++) {
            sc[s] = (uint8_t)((sc6[s] & 0x3F) | ((sc6[s + 4] & 0x3) << 6));
            sc[s + 4] = (uint8_t)((m6[s] & 0x3F) | ((m6[s + 4] & 0x3) << 6));
            sc[s + 8] = (uint8_t)((sc6[s + 4] >> 2) | ((m6[s + 4] >> 2) << 4));
        }
        uint8_t* qs = o + 16;
        for (int s = 0; s < 8; s++) {
            float es = d * (float)sc6[s];
            float em = dmin * (float)m6[s];
            for (int j = 0; j < 16; j++) {
                int q[2];
                for (int t = 0; t < 2; t++) {
                    float v = x[s * 32 + 2 * j + t];
                    q[t] = es > 0.0f ? clampi((int)roundf((v + em) / es), 0, 15) : 0;
                }
                qs[s * 16 + j] = (uint8_t)(q[0] | (q[1] << 4));
            }
        }
    }
}

/* Q4_K 6-bit (scale, min) of sub-block sb: src/metal/compute.rs:725-733. */
static inline void q4k_scale_min(const uint8_t* sc, int sb, uint8_t* s, uint8_t* m) {
    if (sb < 4) {
        *s = sc[sb] & 0x3F;
        *m = sc[sb + 4] & 0x3F;
    } else {
        int si = sb - 4;
        *s = (uint8_t)((sc[si] >> 6) | ((sc[sb + 4] & 0x0F) << 2));
        *m = (uint8_t)((sc[sb] >> 6) | ((sc[sb + 4] >> 4) << 2));
    }
}

/* ---------------------------------------------------------- dequantize */

/* Q6_K super-block (256 weights, 210 bytes) as matvec_q6_k_cpu reads it
 * (src/metal/compute.rs:752-790): ql[128] low nibbles (element idx: byte idx / 2, high
 * nibble when idx is odd), qh[64] 2-bit high parts (byte idx / 4, bits 2 (idx % 4)),
 * 16 int8 scales (one per 16 elements), f16 d at byte 208. q = (high2 << 4 | low4) - 32. */
static int q6k_q(const uint8_t* blk, int idx) {
    const uint8_t ql_byte = blk[idx / 2];
    const int low4 = (idx & 1) ? (ql_byte >> 4) & 0x0F : ql_byte & 0x0F;
    const int high2 = (blk[128 + idx / 4] >> ((idx % 4) * 2)) & 0x03;
    return ((high2 << 4) | low4) - 32;
}

/* Q5_K super-block (256 weights, 176 bytes) as matvec_q5_k_cpu reads it
 * (src/metal/compute.rs:845-899): f16 d, f16 dmin, 12 bytes of 6-bit (scale, min) packed
 * as Q4_K's, qh[32] high bits (element idx: bit idx % 8 of qh[idx / 8]), ql[128] low
 * nibbles (sub-block sb at ql[16 sb], element 2j low / 2j + 1 high nibble of byte j). */
static int q5k_q(const uint8_t* blk, int idx) {
    const uint8_t b = blk[48 + (idx / 32) * 16 + (idx % 32) / 2];
    const int low4 = (idx & 1) ? (b >> 4) & 0x0F : b & 0x0F;
    const int hbit = (blk[16 + idx / 8] >> (idx % 8)) & 1;
    return low4 | (hbit << 4);
}

int ora_dequantize(const uint8_t* w, int type, int64_t n, float* out) {
    if (ora_lowbit_block_bytes(type)) return ora_dequant_lowbit(w, type, n, out);
    switch (type) {
        case ORA_F32: memcpy(out, w, (size_t)n * 4); return 0;
        case ORA_BF16: /* bf16_to_f32 src/metal/compute.rs:2250-2253: bits << 16 */
            for (int64_t i = 0; i < n; i++) {
                const uint32_t b = ((uint32_t)w[2 * i] | ((uint32_t)w[2 * i + 1] << 8)) << 16;
                memcpy(&out[i], &b, 4);
            }
            return 0;
        case ORA_F16: /* src/ssd/streamer.rs:99-106 */
            for (int64_t i = 0; i < n; i++) out[i] = rd_f16(w + 2 * i);
            return 0;
        case ORA_Q8_0: /* dequantize_q8_0 src/ssd/streamer.rs:128-152: q as f32 * scale */
            for (int64_t b = 0; b < n / 32; b++) {
                const uint8_t* blk = w + b * 34;
                float scale = rd_f16(blk);
                for (int j = 0; j < 32; j++) out[b * 32 + j] = (float)(int8_t)blk[2 + j] * scale;
            }
            return 0;
        case ORA_Q4_0: /* dequantize_q4_0 src/ssd/streamer.rs:155-180 */
            for (int64_t b = 0; b < n / 32; b++) {
                const uint8_t* blk = w + b * 18;
                float scale = rd_f16(blk);
                for (int j = 0; j < 16; j++) {
                    uint8_t byte = blk[2 + j];
                    int lo = (int)(byte & 0x0F) - 8;
                    int hi = (int)((byte >> 4) & 0x0F) - 8;
                    out[b * 32 + 2 * j] = (float)lo * scale;
                    out[b * 32 + 2 * j + 1] = (float)hi * scale;
                }
            }
            return 0;
        case ORA_Q8_K: /* element value of matvec_q8_k_cpu src/metal/compute.rs:983-988:
                          f32 d (little-endian), 256 int8, 32 bytes of block sums unused */
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t* blk = w + b * 292;
                float d;
                memcpy(&d, blk, 4);
                for (int j = 0; j < 256; j++) out[b * 256 + j] = d * (float)(int8_t)blk[4 + j];
            }
            return 0;
        case ORA_Q5_K: /* element value of matvec_q5_k_cpu src/metal/compute.rs:863-892 */
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t* blk = w + b * 176;
                const float d = rd_f16(blk), dmin = rd_f16(blk + 2);
                for (int sb = 0; sb < 8; sb++) {
                    uint8_t s, m;
                    q4k_scale_min(blk + 4, sb, &s, &m);
                    const float scale = d * (float)s, min_val = dmin * (float)m;
                    for (int j = 0; j < 32; j++)
                        out[b * 256 + sb * 32 + j] = scale * (float)q5k_q(blk, sb * 32 + j) - min_val;
                }
            }
            return 0;
        case ORA_Q6_K: /* element value of matvec_q6_k_cpu src/metal/compute.rs:768-785 */
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t* blk = w + b * 210;
                const float d = rd_f16(blk + 208);
                for (int sb = 0; sb < 16; sb++) {
                    const float sc = d * (float)(int8_t)blk[192 + sb];
                    for (int j = 0; j < 16; j++)
                        out[b * 256 + sb * 16 + j] = sc * (float)q6k_q(blk, sb * 16 + j);
                }
            }
            return 0;
        case ORA_Q4_K: /* element value of matvec_q4_k_cpu src/metal/compute.rs:718-744 */
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t* blk = w + b * 144;
                float d = rd_f16(blk), dmin = rd_f16(blk + 2);
                const uint8_t* sc = blk + 4;
                const uint8_t* qs = blk + 16;
                for (int sb = 0; sb < 8; sb++) {
                    uint8_t s, m;
                    q4k_scale_min(sc, sb, &s, &m);
                    float scale = d * (float)s;
                    float min_val = dmin * (float)m;
                    for (int j = 0; j < 16; j++) {
                        uint8_t byte_val = qs[sb * 16 + j];
                        out[b * 256 + sb * 32 + 2 * j] = scale * (float)(byte_val & 0x0F) - min_val;
                        out[b * 256 + sb * 32 + 2 * j + 1] =
                            scale * (float)((byte_val >> 4) & 0x0F) - min_val;
                    }
                }
            }
            return 0;
        default: return -1;
    }
}

/* -------------------------------------------------------------- matvecs */

/* matvec_q4_0_cpu src/metal/compute.rs:680-704, one row. */
static float row_q4_0(const uint8_t* w, const float* x, int in_dim, int row) {
    int bpr = in_dim / 32;
    const uint8_t* r = w + (size_t)row * bpr * 18;
    float sum = 0.0f;
    for (int b = 0; b < bpr; b++) {
        const uint8_t* blk = r + (size_t)b * 18;
        float scale = rd_f16(blk);
        int xb = b * 32;
        for (int j = 0; j < 16; j++) {
            uint8_t byte = blk[2 + j];
            int lo = (int)(byte & 0x0F) - 8;
            int hi = (int)((byte >> 4) & 0x0F) - 8;
            sum += scale * (float)lo * x[xb + j * 2];
            sum += scale * (float)hi * x[xb + j * 2 + 1];
        }
    }
    return sum;
}

/* matvec_q8_0_cpu src/metal/compute.rs:904-925, one row. */
static float row_q8_0(const uint8_t* w, const float* x, int in_dim, int row) {
    int bpr = in_dim / 32;
    const uint8_t* r = w + (size_t)row * bpr * 34;
    float sum = 0.0f;
    for (int b = 0; b < bpr; b++) {
        const uint8_t* blk = r + (size_t)b * 34;
        float scale = rd_f16(blk);
        int xb = b * 32;
        for (int j = 0; j < 32; j++) sum += scale * (float)(int8_t)blk[2 + j] * x[xb + j];
    }
    return sum;
}

/* matvec_q4_k_cpu src/metal/compute.rs:707-750, one row. */
static float row_q4_k(const uint8_t* w, const float* x, int in_dim, int row) {
    int bpr = in_dim / 256;
    const uint8_t* r = w + (size_t)row * bpr * 144;
    float sum = 0.0f;
    for (int b = 0; b < bpr; b++) {
        const uint8_t* blk = r + (size_t)b * 144;
        float d = rd_f16(blk), dmin = rd_f16(blk + 2);
        const uint8_t* sc = blk + 4;
        const uint8_t* qs = blk + 16;
        int xb = b * 256;
        for (int sb = 0; sb < 8; sb++) {
            uint8_t s, m;
            q4k_scale_min(sc, sb, &s, &m);
            float scale = d * (float)s;
            float min_val = dmin * (float)m;
            for (int j = 0; j < 16; j++) {
                uint8_t byte_val = qs[sb * 16 + j];
                float v0 = scale * (float)(byte_val & 0x0F) - min_val;
                float v1 = scale * (float)((byte_val >> 4) & 0x0F) - min_val;
                int xi = xb + sb * 32 + j * 2;
                sum += v0 * x[xi] + v1 * x[xi + 1];
            }
        }
    }
    return sum;
}

/* matvec_q8_k_cpu src/metal/compute.rs:971-993, one row: sum += d * q * x. */
static float row_q8_k(const uint8_t* w, const float* x, int in_dim, int row) {
    int bpr = in_dim / 256;
    const uint8_t* r = w + (size_t)row * bpr * 292;
    float sum = 0.0f;
    for (int b = 0; b < bpr; b++) {
        const uint8_t* blk = r + (size_t)b * 292;
        float d;
        memcpy(&d, blk, 4);
        for (int j = 0; j < 256; j++) sum += d * (float)(int8_t)blk[4 + j] * x[b * 256 + j];
    }
    return sum;
}

/* matvec_q5_k_cpu src/metal/compute.rs:845-899, one row: pairs of elements,
 * sum += v0 * x0 + v1 * x1. */
static float row_q5_k(const uint8_t* w, const float* x, int in_dim, int row) {
    int bpr = in_dim / 256;
    const uint8_t* r = w + (size_t)row * bpr * 176;
    float sum = 0.0f;
    for (int b = 0; b < bpr; b++) {
        const uint8_t* blk = r + (size_t)b * 176;
        const float d = rd_f16(blk), dmin = rd_f16(blk + 2);
        for (int sb = 0; sb < 8; sb++) {
            uint8_t s, m;
            q4k_scale_min(blk + 4, sb, &s, &m);
            const float scale = d * (float)s, min_val = dmin * (float)m;
            for (int j = 0; j < 16; j++) {
                const int i0 = sb * 32 + 2 * j;
                const float v0 = scale * (float)q5k_q(blk, i0) - min_val;
                const float v1 = scale * (float)q5k_q(blk, i0 + 1) - min_val;
                sum += v0 * x[b * 256 + i0] + v1 * x[b * 256 + i0 + 1];
            }
        }
    }
    return sum;
}

/* matvec_q6_k_cpu src/metal/compute.rs:752-790, one row: sum += (d * scale) * q * x in
 * element order. */
static float row_q6_k(const uint8_t* w, const float* x, int in_dim, int row) {
    int bpr = in_dim / 256;
    const uint8_t* r = w + (size_t)row * bpr * 210;
    float sum = 0.0f;
    for (int b = 0; b < bpr; b++) {
        const uint8_t* blk = r + (size_t)b * 210;
        const float d = rd_f16(blk + 208);
        for (int sb = 0; sb < 16; sb++) {
            const float sc = d * (float)(int8_t)blk[192 + sb];
            for (int j = 0; j < 16; j++) {
                const int idx = sb * 16 + j;
                sum += sc * (float)q6k_q(blk, idx) * x[b * 256 + idx];
            }
        }
    }
    return sum;
}

/* matvec_bf16_cpu src/metal/compute.rs:2256-2269, one row. */
static float row_bf16(const uint8_t* w, const float* x, int in_dim, int row) {
    const uint8_t* r = w + (size_t)row * in_dim * 2;
    float sum = 0.0f;
    for (int c = 0; c < in_dim; c++) {
        const uint32_t b = ((uint32_t)r[2 * c] | ((uint32_t)r[2 * c + 1] << 8)) << 16;
        float v;
        memcpy(&v, &b, 4);
        sum += v * x[c];
    }
    return sum;
}

/* f16 matvec src/metal/compute.rs:2272-2285, one row. */
static float row_f16(const uint8_t* w, const float* x, int in_dim, int row) {
    const uint8_t* r = w + (size_t)row * in_dim * 2;
    float sum = 0.0f;
    for (int c = 0; c < in_dim; c++) sum += rd_f16(r + 2 * c) * x[c];
    return sum;
}

/* matvec_f32_simd_scalar src/metal/compute.rs:390-424, one row. */
static float row_f32(const float* w, const float* x, int in_dim, int row) {
    const float* r = w + (size_t)row * in_dim;
    int chunks = in_dim / 4, rem = in_dim % 4;
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    for (int c = 0; c < chunks; c++) {
        int j = c * 4;
        s0 += r[j] * x[j];
        s1 += r[j + 1] * x[j + 1];
        s2 += r[j + 2] * x[j + 2];
        s3 += r[j + 3] * x[j + 3];
    }
    int base = chunks * 4;
    for (int j = 0; j < rem; j++) s0 += r[base + j] * x[base + j];
    return s0 + s1 + s2 + s3;
}

void ora_matvec_f32(const float* w, const float* x, int out_dim, int in_dim, float* y) {
    for (int i = 0; i < out_dim; i++) y[i] = row_f32(w, x, in_dim, i);
}

typedef float (*row_fn)(const uint8_t*, const float*, int, int);

/* F32 rows as bytes: the same matvec_f32_simd row (for layers of F32 weights). */
static float row_f32b(const uint8_t* w, const float* x, int in_dim, int row) {
    return row_f32((const float*)w, x, in_dim, row);
}

static row_fn pick_row(int type) {
    switch (type) {
        case ORA_F32: return row_f32b;
        case ORA_Q4_0: return row_q4_0;
        case ORA_Q8_0: return row_q8_0;
        case ORA_Q4_K: return row_q4_k;
        case ORA_Q5_K: return row_q5_k;
        case ORA_Q6_K: return row_q6_k;
        case ORA_Q8_K: return row_q8_k;
        case ORA_F16: return row_f16;
        case ORA_BF16: return row_bf16;
        default: return NULL;
    }
}

typedef struct {
    row_fn fn;
    int type; /* low-bit formats (fn NULL) */
    const uint8_t* w;
    const float* x;
    int in_dim, r0, r1;
    float* y;
} mv_job;

static void mv_rows(const mv_job* j) {
    for (int r = j->r0; r < j->r1; r++) {
        if (j->fn)
            j->y[r] = j->fn(j->w, j->x, j->in_dim, r);
        else
            ora_row_lowbit(j->type, j->w, j->x, j->in_dim, r, &j->y[r]);
    }
}

static void* mv_worker(void* p) {
    mv_rows((const mv_job*)p);
    return NULL;
}

int ora_matvec_quantized_mt(const uint8_t* w, const float* x, int out_dim, int in_dim, int type,
                            float* y, int threads) {
    row_fn fn = pick_row(type);
    if (type == ORA_F32) {
        ora_matvec_f32((const float*)w, x, out_dim, in_dim, y);
        return 0;
    }
    if (!fn && !ora_lowbit_block_bytes(type)) { /* compute.rs:672-675: unsupported -> zeros */
        memset(y, 0, sizeof(float) * (size_t)out_dim);
        return -1;
    }
    if (threads <= 1 || out_dim < 2 * threads) {
        const mv_job j = {fn, type, w, x, in_dim, 0, out_dim, y};
        mv_rows(&j);
        return 0;
    }
    if (threads > 256) threads = 256;
    pthread_t th[256];
    mv_job jobs[256];
    /* row split as in parallel_matvec src/inference/tensor_parallel.rs:47-64 */
    int shard = out_dim / threads, remainder = out_dim % threads, off = 0;
    for (int t = 0; t < threads; t++) {
        int rows = shard + (t < remainder ? 1 : 0);
        jobs[t] = (mv_job){fn, type, w, x, in_dim, off, off + rows, y};
        off += rows;
        pthread_create(&th[t], NULL, mv_worker, &jobs[t]);
    }
    for (int t = 0; t < threads; t++) pthread_join(th[t], NULL);
    return 0;
}

int ora_matvec_quantized(const uint8_t* w, const float* x, int out_dim, int in_dim, int type,
                         float* y) {
    return ora_matvec_quantized_mt(w, x, out_dim, in_dim, type, y, 1);
}

/* ------------------------------------------------------- norms and such */

static float sum_sq(const float* x, int n) { /* x.iter().map(|v| v * v).sum() */
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += x[i] * x[i];
    return s;
}

void ora_rmsnorm(float* x, const float* w, int n, float eps) {
    float ss = sum_sq(x, n);
    float inv_rms = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) x[i] *= inv_rms * w[i];
}

void ora_fused_residual_rmsnorm(float* x, const float* residual, const float* w, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) {
        float val = x[i] + residual[i];
        x[i] = val;
        ss += val * val;
    }
    float inv_rms = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) x[i] *= inv_rms * w[i];
}

void ora_fused_post_attn_norm(float* hidden, const float* attn, const float* w, int n, float eps,
                              float* out) {
    for (int i = 0; i < n; i++) hidden[i] += attn[i];
    float ss = sum_sq(hidden, n);
    float inv_rms = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) out[i] = hidden[i] * inv_rms * w[i];
}

void ora_fused_rmsnorm_linear(const float* x, const float* norm_w, const float* out_w, int vocab,
                              int n_embd, float* logits) {
    float ss = sum_sq(x, n_embd);
    float inv_rms = 1.0f / sqrtf(ss / (float)n_embd + 1e-5f);
    float* xn = (float*)malloc(sizeof(float) * (size_t)n_embd);
    for (int i = 0; i < n_embd; i++) xn[i] = x[i] * inv_rms * norm_w[i];
    ora_matvec_f32(out_w, xn, vocab, n_embd, logits);
    free(xn);
}

void ora_rope_multi_head(float* x, int len, int head_dim, int n_heads, int position, float theta) {
    int half_dim = head_dim / 2;
    for (int h = 0; h < n_heads; h++) {
        int base = h * head_dim;
        for (int i = 0; i < half_dim; i++) {
            float freq = 1.0f / powf(theta, 2.0f * (float)i / (float)head_dim);
            float angle = (float)position * freq;
            float s = sinf(angle), c = cosf(angle);
            int i0 = base + i * 2, i1 = i0 + 1;
            if (i1 < len) {
                float x0 = x[i0], x1 = x[i1];
                x[i0] = x0 * c - x1 * s;
                x[i1] = x0 * s + x1 * c;
            }
        }
    }
}

void ora_softmax(float* x, int n) {
    if (n <= 0) return;
    float mx = -INFINITY;
    for (int i = 0; i < n; i++) mx = fmaxf(mx, x[i]); /* fold(NEG_INFINITY, f32::max) */
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    if (sum > 0.0f) {
        float inv = 1.0f / sum;
        for (int i = 0; i < n; i++) x[i] *= inv;
    }
}

void ora_silu(float* x, int n) {
    for (int i = 0; i < n; i++) x[i] = x[i] / (1.0f + expf(-x[i]));
}

int ora_argmax(const float* v, int n) {
    if (n <= 0) return 0;
    int best = 0;
    for (int i = 1; i < n; i++)
        if (!(v[i] < v[best])) best = i; /* max_by keeps the last of equal maxima */
    return best;
}

/* -------------------------------------------------------------- INT8 KV */

void ora_kv_quantize(const float* v, int n, int8_t* q, float* scale) {
    float absmax = 0.0f;
    for (int i = 0; i < n; i++) absmax = fmaxf(absmax, fabsf(v[i]));
    if (absmax == 0.0f) {
        memset(q, 0, (size_t)n);
        *scale = 0.0f;
        return;
    }
    float inv_scale = 127.0f / absmax;
    *scale = absmax / 127.0f;
    for (int i = 0; i < n; i++) {
        float r = roundf(v[i] * inv_scale); /* Rust f32::round: half away from zero */
        if (r < -127.0f) r = -127.0f;
        if (r > 127.0f) r = 127.0f;
        q[i] = (int8_t)r;
    }
}

void ora_kv_dequantize(const int8_t* q, float scale, int n, float* out) {
    for (int i = 0; i < n; i++) out[i] = (float)q[i] * scale;
}

void ora_attention_int8(const float* q, const int8_t* k, const float* ks, const int8_t* v,
                        const float* vs, int seq_len, int n_head, int n_head_kv, int head_dim,
                        float* out) {
    int kv_dim = n_head_kv * head_dim;
    float scale = 1.0f / sqrtf((float)head_dim);
    int group = n_head / n_head_kv;
    if (group < 1) group = 1;
    float* scores = (float*)malloc(sizeof(float) * (size_t)(seq_len > 0 ? seq_len : 1));
    float* kh = (float*)malloc(sizeof(float) * (size_t)head_dim);
    for (int h = 0; h < n_head; h++) {
        int kv_h = h / group;
        const float* qh = q + (size_t)h * head_dim;
        for (int p = 0; p < seq_len; p++) { /* key_at + dot, attention.rs:208-214 */
            ora_kv_dequantize(k + (size_t)p * kv_dim + (size_t)kv_h * head_dim, ks[p], head_dim, kh);
            float dot = 0.0f;
            for (int d = 0; d < head_dim; d++) dot += qh[d] * kh[d];
            scores[p] = dot * scale;
        }
        ora_softmax(scores, seq_len);
        for (int d = 0; d < head_dim; d++) { /* attention.rs:219-229, value_at(pos)[d] */
            float weighted = 0.0f;
            for (int p = 0; p < seq_len; p++) {
                float vd = (float)v[(size_t)p * kv_dim + (size_t)kv_h * head_dim + d] * vs[p];
                weighted += scores[p] * vd;
            }
            out[(size_t)h * head_dim + d] = weighted;
        }
    }
    free(kh);
    free(scores);
}

void ora_flash_attention_int8(const float* q, const int8_t* k, const float* ks, const int8_t* v,
                              const float* vs, int seq_len, int n_head, int n_head_kv,
                              int head_dim, float* out) {
    int kv_dim = n_head_kv * head_dim;
    float scale = 1.0f / sqrtf((float)head_dim);
    int group = n_head / n_head_kv;
    if (group < 1) group = 1;
    float* acc = (float*)malloc(sizeof(float) * (size_t)head_dim);
    float* kh = (float*)malloc(sizeof(float) * (size_t)head_dim);
    float* vh = (float*)malloc(sizeof(float) * (size_t)head_dim);
    for (int h = 0; h < n_head; h++) {
        int kv_h = h / group;
        const float* qh = q + (size_t)h * head_dim;
        float running_max = -INFINITY, running_sum = 0.0f;
        for (int d = 0; d < head_dim; d++) acc[d] = 0.0f;
        for (int p = 0; p < seq_len; p++) {
            ora_kv_dequantize(k + (size_t)p * kv_dim + (size_t)kv_h * head_dim, ks[p], head_dim, kh);
            float dot = 0.0f; /* 4-wide unroll, flash_attention.rs:90-102 */
            int chunks = head_dim / 4, rem = head_dim % 4;
            for (int c = 0; c < chunks; c++) {
                int b = c * 4;
                dot += qh[b] * kh[b] + qh[b + 1] * kh[b + 1] + qh[b + 2] * kh[b + 2] +
                       qh[b + 3] * kh[b + 3];
            }
            for (int i = chunks * 4; i < chunks * 4 + rem; i++) dot += qh[i] * kh[i];
            float score = dot * scale;
            ora_kv_dequantize(v + (size_t)p * kv_dim + (size_t)kv_h * head_dim, vs[p], head_dim, vh);
            if (score > running_max) {
                float correction = expf(running_max - score);
                running_sum *= correction;
                for (int d = 0; d < head_dim; d++) acc[d] *= correction;
                running_max = score;
            }
            float weight = expf(score - running_max);
            running_sum += weight;
            for (int d = 0; d < head_dim; d++) acc[d] += weight * vh[d];
        }
        for (int d = 0; d < head_dim; d++) out[(size_t)h * head_dim + d] = 0.0f;
        if (running_sum > 0.0f) {
            float inv_sum = 1.0f / running_sum;
            for (int d = 0; d < head_dim; d++) out[(size_t)h * head_dim + d] = acc[d] * inv_sum;
        }
    }
    free(vh);
    free(kh);
    free(acc);
}

/* Windowed attention over f32 K/V rows [pos][n_head_kv * head_dim]: the shader
 * flash_attention_f32 (src/metal/shaders/kernels.metal:1360-1440) and its CPU twin
 * flash_attention_windowed (src/inference/flash_attention.rs:146-229). Positions
 * [window_start, min(window_end, seq_len)) in order; 4-wide unrolled q.k as the shader
 * (kernels.metal:1399-1407); a head whose window is empty gets zeros (:1430-1438). */
void ora_flash_attention_f32(const float* q, const float* k, const float* v, int n_head,
                             int n_head_kv, int head_dim, int seq_len, int window_start,
                             int window_end, float* out) {
    int kv_dim = n_head_kv * head_dim;
    int group = n_head_kv > 0 ? n_head / n_head_kv : 1;
    if (group < 1) group = 1;
    float scale = 1.0f / sqrtf((float)head_dim);
    int end = window_end < seq_len ? window_end : seq_len;
    float* acc = (float*)malloc(sizeof(float) * (size_t)(head_dim > 0 ? head_dim : 1));
    for (int h = 0; h < n_head; h++) {
        int kv_h = h / group;
        const float* qh = q + (size_t)h * head_dim;
        float running_max = -INFINITY, running_sum = 0.0f;
        for (int d = 0; d < head_dim; d++) acc[d] = 0.0f;
        for (int p = window_start; p < end; p++) {
            const float* kh = k + (size_t)p * kv_dim + (size_t)kv_h * head_dim;
            const float* vh = v + (size_t)p * kv_dim + (size_t)kv_h * head_dim;
            int hd4 = (head_dim / 4) * 4;
            float dot = 0.0f;
            for (int d = 0; d < hd4; d += 4)
                dot += qh[d] * kh[d] + qh[d + 1] * kh[d + 1] + qh[d + 2] * kh[d + 2] +
                       qh[d + 3] * kh[d + 3];
            for (int d = hd4; d < head_dim; d++) dot += qh[d] * kh[d];
            float score = dot * scale;
            if (score > running_max) {
                float correction = expf(running_max - score);
                running_sum *= correction;
                for (int d = 0; d < head_dim; d++) acc[d] *= correction;
                running_max = score;
            }
            float weight = expf(score - running_max);
            running_sum += weight;
            for (int d = 0; d < head_dim; d++) acc[d] += weight * vh[d];
        }
        for (int d = 0; d < head_dim; d++)
            out[(size_t)h * head_dim + d] = running_sum > 0.0f ? acc[d] * (1.0f / running_sum) : 0.0f;
    }
    free(acc);
}

/* SwiGLU feed-forward (src/inference/feed_forward.rs:17-43): act = silu(W_gate x) * (W_up x),
 * out = W_down act, each product by matvec_f32_simd (compute.rs:390-424). n_ff == 0 gives
 * zeros (:25-28). */
void ora_feed_forward_f32(const float* x, const float* w_gate, const float* w_up,
                          const float* w_down, int n_embd, int n_ff, float* out) {
    if (n_ff <= 0) {
        for (int i = 0; i < n_embd; i++) out[i] = 0.0f;
        return;
    }
    float* g = (float*)malloc(sizeof(float) * (size_t)n_ff);
    float* u = (float*)malloc(sizeof(float) * (size_t)n_ff);
    ora_matvec_f32(w_gate, x, n_ff, n_embd, g);
    ora_silu(g, n_ff);
    ora_matvec_f32(w_up, x, n_ff, n_embd, u);
    for (int i = 0; i < n_ff; i++) g[i] *= u[i];
    ora_matvec_f32(w_down, g, n_embd, n_ff, out);
    free(u);
    free(g);
}

/* ----------------------------------------------------------- layer step */

/* Matvec in one of the two reference CPU paths. Mode 0 (the live path of
 * forward_pass): the weights are dequantized to f32 (src/ssd/streamer.rs:34-66)
 * and multiplied by matvec_f32_simd (compute.rs:390-424); dequant is elementwise
 * and exact, so dequantizing row by row gives the same bits. Mode 1: the
 * operator path matvec_quantized_cpu (compute.rs:648-677). */
typedef struct {
    const uint8_t* w;
    const float* x;
    int in_dim, wtype, r0, r1, mode;
    float* y;
} lmv_job;

static void* lmv_worker(void* p) {
    lmv_job* j = (lmv_job*)p;
    size_t rb = ora_row_bytes(j->wtype, j->in_dim);
    if (j->mode == 0) {
        float* row = (float*)malloc(sizeof(float) * (size_t)j->in_dim);
        for (int r = j->r0; r < j->r1; r++) {
            ora_dequantize(j->w + (size_t)r * rb, j->wtype, j->in_dim, row);
            j->y[r] = row_f32(row, j->x, j->in_dim, 0);
        }
        free(row);
    } else {
        row_fn fn = pick_row(j->wtype);
        for (int r = j->r0; r < j->r1; r++) {
            if (fn)
                j->y[r] = fn(j->w, j->x, j->in_dim, r);
            else  /* low-bit: the reference's matvec_*_cpu row (compute.rs:793-1075, 1964-2240) */
                ora_row_lowbit(j->wtype, j->w, j->x, j->in_dim, r, &j->y[r]);
        }
    }
    return NULL;
}

static void layer_matvec(const uint8_t* w, int wtype, const float* x, int out_dim, int in_dim,
                         float* y, int mode, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (out_dim < 2 * threads) threads = 1;
    pthread_t th[256];
    lmv_job jobs[256];
    int shard = out_dim / threads, remainder = out_dim % threads, off = 0;
    for (int t = 0; t < threads; t++) {
        int rows = shard + (t < remainder ? 1 : 0);
        jobs[t] = (lmv_job){w, x, in_dim, wtype, off, off + rows, mode, y};
        off += rows;
        if (threads == 1)
            lmv_worker(&jobs[t]);
        else
            pthread_create(&th[t], NULL, lmv_worker, &jobs[t]);
    }
    if (threads > 1)
        for (int t = 0; t < threads; t++) pthread_join(th[t], NULL);
}

static int layer_wtype(const ora_layer* L, int i) {
    return L->wtypes[i] >= 0 ? L->wtypes[i] : L->wtype;
}

int ora_layer_step(const ora_layer* L, float* hidden, int position, int8_t* k_cache,
                   float* k_scales, int8_t* v_cache, float* v_scales, int matvec_mode,
                   int threads) {
    int n = L->n_embd, hd = L->head_dim;
    int q_dim = L->n_head * hd, kv_dim = L->n_head_kv * hd, ff = L->n_ff;
    if (q_dim != n) return -1;
    /* every type the row kernels or the low-bit row decoder read (ora_row_bytes > 0) */
    for (int i = 0; i < 7; i++)
        if (!pick_row(layer_wtype(L, i)) && ora_row_bytes(layer_wtype(L, i), 256) == 0) return -1;
    float* attn_in = (float*)malloc(sizeof(float) * (size_t)n);
    float* q = (float*)malloc(sizeof(float) * (size_t)q_dim);
    float* k = (float*)malloc(sizeof(float) * (size_t)kv_dim);
    float* v = (float*)malloc(sizeof(float) * (size_t)kv_dim);
    float* attn = (float*)malloc(sizeof(float) * (size_t)n);
    float* attn_out = (float*)malloc(sizeof(float) * (size_t)n);
    float* ffn_in = (float*)malloc(sizeof(float) * (size_t)n);
    float* gate = (float*)malloc(sizeof(float) * (size_t)ff);
    float* up = (float*)malloc(sizeof(float) * (size_t)ff);
    float* down = (float*)malloc(sizeof(float) * (size_t)n);

    /* 1. pre-attention RMSNorm: transformer.rs:323-326 (eps 1e-5, :576-579) */
    memcpy(attn_in, hidden, sizeof(float) * (size_t)n);
    ora_rmsnorm(attn_in, L->attn_norm, n, L->eps);
    /* 2. fused QKV + RoPE: fused_qkv_rope_f32_cpu compute.rs:509-529 */
    layer_matvec(L->wq, layer_wtype(L, 0), attn_in, q_dim, n, q, matvec_mode, threads);
    layer_matvec(L->wk, layer_wtype(L, 1), attn_in, kv_dim, n, k, matvec_mode, threads);
    layer_matvec(L->wv, layer_wtype(L, 2), attn_in, kv_dim, n, v, matvec_mode, threads);
    ora_rope_multi_head(q, q_dim, hd, L->n_head, position, L->theta);
    ora_rope_multi_head(k, kv_dim, hd, L->n_head_kv, position, L->theta);
    /* kv_cache.append: QuantizedLayerKvCache::append quantized_kv_cache.rs:107-110 */
    ora_kv_quantize(k, kv_dim, k_cache + (size_t)position * kv_dim, &k_scales[position]);
    ora_kv_quantize(v, kv_dim, v_cache + (size_t)position * kv_dim, &v_scales[position]);
    /* attention over positions 0..=position: attention.rs:198-236 */
    ora_attention_int8(q, k_cache, k_scales, v_cache, v_scales, position + 1, L->n_head,
                       L->n_head_kv, hd, attn);
    layer_matvec(L->wo, layer_wtype(L, 3), attn, n, n, attn_out, matvec_mode, threads);
    /* 3. residual + FFN norm: fused_post_attn_norm_f32_cpu compute.rs:536-555 */
    ora_fused_post_attn_norm(hidden, attn_out, L->ffn_norm, n, L->eps, ffn_in);
    /* 4. SwiGLU FFN: feed_forward feed_forward.rs:17-44 */
    layer_matvec(L->w_gate, layer_wtype(L, 4), ffn_in, ff, n, gate, matvec_mode, threads);
    ora_silu(gate, ff);
    layer_matvec(L->w_up, layer_wtype(L, 5), ffn_in, ff, n, up, matvec_mode, threads);
    for (int i = 0; i < ff; i++) gate[i] *= up[i];
    layer_matvec(L->w_down, layer_wtype(L, 6), gate, n, ff, down, matvec_mode, threads);
    /* 5. residual: transformer.rs:369-371 */
    for (int i = 0; i < n; i++) hidden[i] += down[i];

    free(attn_in); free(q); free(k); free(v); free(attn);
    free(attn_out); free(ffn_in); free(gate); free(up); free(down);
    return 0;
}
