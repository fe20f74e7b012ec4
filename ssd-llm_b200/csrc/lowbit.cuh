// lowbit.cuh — device decoders of the reference's low-bit formats, kept in the reference's
// own block layouts (matvec_q3_k_cpu ... matvec_iq2_xs_cpu, src/metal/compute.rs:793-1075,
// 1964-2240): Q3_K (256 weights in 110 B), Q2_K (84 B), IQ4_NL (32 in 18 B), IQ4_XS (148 B),
// IQ3_XXS (98 B), IQ3_S (110 B), IQ2_XXS (66 B), IQ2_XS (74 B).
//
// lowbit_group() gives the 32 weights of one 32-element group of a block, each the product
// of its factors in the reference's left-to-right order, one rounding per product
// (__fmul_rn / __fsub_rn: no contraction), so ssd_dequantize is bit-exact with the
// reference's element values. KSIGNS_IQ2XS (compute.rs:1964) is i with bit 7 = parity(i).
#pragma once
#include "common.cuh"

#define SSD_IQ_DATA static __device__ const
#include "iq_grids.h"
#undef SSD_IQ_DATA

namespace ssd {

// IQ4_NL_QUANTS (compute.rs:997-999)
__device__ __forceinline__ float iq4nl_value(int i) {
    const int8_t t[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
    return (float)t[i];
}
__device__ __forceinline__ uint32_t ksigns_iq2xs(uint32_t i) {
    return i | ((uint32_t)(__popc(i) & 1) << 7);
}
__device__ __forceinline__ float lb_f16(const uint8_t* p) {
    return f16_bits_to_f32((uint16_t)(p[0] | (p[1] << 8)));
}
__device__ __forceinline__ uint32_t lb_u32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
__device__ __forceinline__ float lb_sign(uint32_t signs, int j) {
    return (signs >> j) & 1u ? -1.0f : 1.0f;
}

// The 32 weights of group g (elements 32g .. 32g + 31) of the block at blk.
template <int T>
__device__ __forceinline__ void lowbit_group(const uint8_t* __restrict__ blk, int g, float (&w)[32]) {
    if constexpr (T == SSD_TYPE_Q3_K) {  // compute.rs:796-840
        const uint8_t* hmask = blk;
        const uint8_t* qs = blk + 32;
        const uint8_t* sc = blk + 96;
        const float d = lb_f16(blk + 108);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int sb = 2 * g + h;
            const int low4 = (sc[sb / 2] >> ((sb & 1) * 4)) & 0x0F;
            const int hi2 = (sc[8 + sb / 4] >> ((sb % 4) * 2)) & 0x03;
            int s = low4 | (hi2 << 4);
            if (s >= 32) s -= 64;
            const float sc_f = __fmul_rn(d, (float)s);
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int idx = sb * 16 + j;
                const int low2 = (qs[idx / 4] >> ((idx % 4) * 2)) & 0x03;
                const int hbit = (hmask[idx / 8] >> (idx % 8)) & 1;
                w[h * 16 + j] = __fmul_rn(sc_f, (float)((low2 | (hbit << 2)) - 4));
            }
        }
    } else if constexpr (T == SSD_TYPE_Q2_K) {  // compute.rs:930-966: scale * q - min
        const float d = lb_f16(blk), dmin = lb_f16(blk + 2);
        const uint8_t* sc = blk + 4;
        const uint8_t* qs = blk + 20;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int sb = 2 * g + h;
            const float scale = __fmul_rn(d, (float)(sc[sb] & 0x0F));
            const float mn = __fmul_rn(dmin, (float)((sc[sb] >> 4) & 0x0F));
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int idx = sb * 16 + j;
                const float q = (float)((qs[idx / 4] >> ((idx % 4) * 2)) & 0x03);
                w[h * 16 + j] = __fsub_rn(__fmul_rn(scale, q), mn);
            }
        }
    } else if constexpr (T == SSD_TYPE_IQ4_NL) {  // compute.rs:1004-1030 (one group per block)
        const float d = lb_f16(blk);
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const uint8_t b = blk[2 + j];
            w[2 * j] = __fmul_rn(d, iq4nl_value(b & 0x0F));
            w[2 * j + 1] = __fmul_rn(d, iq4nl_value(b >> 4));
        }
    } else if constexpr (T == SSD_TYPE_IQ4_XS) {  // compute.rs:1034-1075
        const float d = lb_f16(blk);
        const uint32_t sh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8);
        const uint32_t slw = (uint32_t)blk[4 + (g / 2) * 2] | ((uint32_t)blk[5 + (g / 2) * 2] << 8);
        const int sl = (g % 2 == 0) ? (int)(slw & 0x0F) : (int)((slw >> 4) & 0x0F);
        const int shb = (int)((sh >> (2 * g)) & 0x03);
        const float ds = __fmul_rn(d, (float)(sl | (shb << 4)) - 32.0f);
        const uint8_t* q = blk + 20 + g * 16;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            w[2 * j] = __fmul_rn(ds, iq4nl_value(q[j] & 0x0F));
            w[2 * j + 1] = __fmul_rn(ds, iq4nl_value(q[j] >> 4));
        }
    } else if constexpr (T == SSD_TYPE_IQ3_XXS) {  // compute.rs:1983-2036
        const float d = lb_f16(blk);
        const uint8_t* qs = blk + 2;
        const uint32_t aux = lb_u32(qs + 64 + g * 4);
        const float db = __fmul_rn(__fmul_rn(d, 0.5f + (float)(aux >> 28)), 0.5f);
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t signs = ksigns_iq2xs((aux >> (7 * l)) & 127u);
            const uint32_t c0 = kIq3xxsGrid[qs[g * 8 + 2 * l]], c1 = kIq3xxsGrid[qs[g * 8 + 2 * l + 1]];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                w[l * 8 + j] = __fmul_rn(__fmul_rn(db, (float)kIq3xxsVals[(c0 >> (3 * j)) & 7]),
                                         lb_sign(signs, j));
                w[l * 8 + j + 4] = __fmul_rn(
                    __fmul_rn(db, (float)kIq3xxsVals[(c1 >> (3 * j)) & 7]), lb_sign(signs, j + 4));
            }
        }
    } else if constexpr (T == SSD_TYPE_IQ3_S) {  // compute.rs:2042-2131
        const float d = lb_f16(blk);
        const uint8_t* qs = blk + 2;
        const uint8_t* qh = qs + 64;
        const uint8_t* sg = qh + 8;
        const uint8_t sbyte = (qh + 40)[g / 2];
        const float db = __fmul_rn(d, (float)(1 + 2 * (int)((g % 2 == 0) ? (sbyte & 0x0F) : (sbyte >> 4))));
        const int q8 = qh[g];
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const int e0 = qs[g * 8 + 2 * l] | ((q8 << (8 - 2 * l)) & 256);
            const int e1 = qs[g * 8 + 2 * l + 1] | ((q8 << (7 - 2 * l)) & 256);
            const uint32_t c0 = kIq3sGrid[e0], c1 = kIq3sGrid[e1];
            const uint32_t signs = sg[g * 4 + l];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                w[l * 8 + j] = __fmul_rn(__fmul_rn(db, (float)kIq3sVals[(c0 >> (3 * j)) & 7]),
                                         lb_sign(signs, j));
                w[l * 8 + j + 4] = __fmul_rn(__fmul_rn(db, (float)kIq3sVals[(c1 >> (3 * j)) & 7]),
                                             lb_sign(signs, j + 4));
            }
        }
    } else if constexpr (T == SSD_TYPE_IQ2_XXS) {  // compute.rs:2137-2186
        const float d = lb_f16(blk);
        const uint8_t* gp = blk + 2 + g * 8;
        const uint32_t a1 = lb_u32(gp + 4);
        const float db = __fmul_rn(__fmul_rn(d, 0.5f + (float)(a1 >> 28)), 0.25f);
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t signs = ksigns_iq2xs((a1 >> (7 * l)) & 127u);
            const uint32_t c = kIq2xxsGrid[gp[l]];
#pragma unroll
            for (int j = 0; j < 8; j++)
                w[l * 8 + j] = __fmul_rn(__fmul_rn(db, (float)kIq2Vals[(c >> (2 * j)) & 3]),
                                         lb_sign(signs, j));
        }
    } else {  // IQ2_XS, compute.rs:2192-2240
        const float d = lb_f16(blk);
        const uint8_t* qs = blk + 2;
        const uint8_t sb = qs[64 + g / 2];
        const float db = __fmul_rn(__fmul_rn(d, 0.5f + (float)((g % 2 == 0) ? (sb & 0x0F) : (sb >> 4))), 0.25f);
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t v = (uint32_t)qs[(g * 4 + l) * 2] | ((uint32_t)qs[(g * 4 + l) * 2 + 1] << 8);
            const uint32_t signs = ksigns_iq2xs(v >> 9);
            const uint32_t c = kIq2xsGrid[v & 511u];
#pragma unroll
            for (int j = 0; j < 8; j++)
                w[l * 8 + j] = __fmul_rn(__fmul_rn(db, (float)kIq2Vals[(c >> (2 * j)) & 3]),
                                         lb_sign(signs, j));
        }
    }
}

// Runtime dispatch of lowbit_group (dequantize path).
__device__ __forceinline__ void lowbit_group_any(int type, const uint8_t* blk, int g, float (&w)[32]) {
    switch (type) {
        case SSD_TYPE_Q3_K: lowbit_group<SSD_TYPE_Q3_K>(blk, g, w); break;
        case SSD_TYPE_Q2_K: lowbit_group<SSD_TYPE_Q2_K>(blk, g, w); break;
        case SSD_TYPE_IQ4_NL: lowbit_group<SSD_TYPE_IQ4_NL>(blk, g, w); break;
        case SSD_TYPE_IQ4_XS: lowbit_group<SSD_TYPE_IQ4_XS>(blk, g, w); break;
        case SSD_TYPE_IQ3_XXS: lowbit_group<SSD_TYPE_IQ3_XXS>(blk, g, w); break;
        case SSD_TYPE_IQ3_S: lowbit_group<SSD_TYPE_IQ3_S>(blk, g, w); break;
        case SSD_TYPE_IQ2_XXS: lowbit_group<SSD_TYPE_IQ2_XXS>(blk, g, w); break;
        default: lowbit_group<SSD_TYPE_IQ2_XS>(blk, g, w); break;
    }
}

}  // namespace ssd
