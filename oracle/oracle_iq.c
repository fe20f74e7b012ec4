/*
 * oracle_iq.c — CPU restatement of the reference's low-bit formats (TEST INFRASTRUCTURE ONLY):
 * Q3_K, Q2_K, IQ4_NL, IQ4_XS, IQ3_XXS, IQ3_S, IQ2_XXS, IQ2_XS in the reference's own block
 * layouts (src/metal/compute.rs:793-1075, 1964-2240). Built into the oracle library with
 * oracle.c (same flags: one IEEE float op per Rust float op, no contraction).
 *
 * Each row function walks the elements in the reference's loop order and adds
 * w * x[idx] to one fp32 sum, where w is the product of the element's factors in the
 * reference's left-to-right order (for Q2_K, scale * q - min). The dequantize functions
 * give the same w per element in element order.
 *
 * The lattice grids come from the library's iq_grids.h (16-bit codes; its SHA-256 over the
 * expanded tables is pinned by tests/test_oracle_iq.py); the sign table KSIGNS_IQ2XS
 * (compute.rs:1964) is i with bit 7 = parity(i).
 */
#include <string.h>

#include "oracle.h"
#include "../ssd-llm_b200/csrc/iq_grids.h"

static inline float f16(const uint8_t* p) { return ora_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }
static inline uint32_t u32le(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static inline uint8_t ksigns(uint32_t i) {
    uint32_t p = i;
    p ^= p >> 4;
    p ^= p >> 2;
    p ^= p >> 1;
    return (uint8_t)(i | ((p & 1u) << 7));
}
/* byte j of a grid entry */
static inline int g_iq2xxs(int e, int j) { return kIq2Vals[(kIq2xxsGrid[e] >> (2 * j)) & 3]; }
static inline int g_iq2xs(int e, int j) { return kIq2Vals[(kIq2xsGrid[e] >> (2 * j)) & 3]; }
static inline int g_iq3xxs(int e, int j) { return kIq3xxsVals[(kIq3xxsGrid[e] >> (3 * j)) & 7]; }
static inline int g_iq3s(int e, int j) { return kIq3sVals[(kIq3sGrid[e] >> (3 * j)) & 7]; }
static inline float sgn(uint8_t signs, int j) { return (signs >> j) & 1 ? -1.0f : 1.0f; }

/* IQ4_NL_QUANTS, compute.rs:997-999 */
static const float kIq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                 1,    13,   25,  38,  53,  69,  89,  113};

size_t ora_lowbit_block_bytes(int type) {
    switch (type) {
        case ORA_Q2_K: return 84;
        case ORA_Q3_K: return 110;
        case ORA_IQ4_NL: return 18;
        case ORA_IQ4_XS: return 148;
        case ORA_IQ3_XXS: return 98;
        case ORA_IQ3_S: return 110;
        case ORA_IQ2_XXS: return 66;
        case ORA_IQ2_XS: return 74;
        default: return 0;
    }
}
int ora_lowbit_block(int type) { return type == ORA_IQ4_NL ? 32 : 256; }

/* The weight values of one block, element order, written through `emit(idx, w)` in the
 * reference's loop order (the order its matvec adds them). */
typedef void (*emit_fn)(void* ctx, int idx, float w);

static void blk_q3_k(const uint8_t* blk, emit_fn emit, void* c) { /* compute.rs:796-840 */
    const uint8_t* hmask = blk;
    const uint8_t* qs = blk + 32;
    const uint8_t* sc = blk + 96;
    const float d = f16(blk + 108);
    for (int sb = 0; sb < 16; sb++) {
        const int low4 = (sc[sb / 2] >> ((sb & 1) * 4)) & 0x0F;
        const int hi2 = (sc[8 + sb / 4] >> ((sb % 4) * 2)) & 0x03;
        int s = low4 | (hi2 << 4);
        if (s >= 32) s -= 64;
        const float sc_f = d * (float)s;
        for (int j = 0; j < 16; j++) {
            const int idx = sb * 16 + j;
            const int low2 = (qs[idx / 4] >> ((idx % 4) * 2)) & 0x03;
            const int hbit = (hmask[idx / 8] >> (idx % 8)) & 1;
            const int q = (low2 | (hbit << 2)) - 4;
            emit(c, idx, sc_f * (float)q);
        }
    }
}

static void blk_q2_k(const uint8_t* blk, emit_fn emit, void* c) { /* compute.rs:930-966 */
    const float d = f16(blk), dmin = f16(blk + 2);
    const uint8_t* sc = blk + 4;
    const uint8_t* qs = blk + 20;
    for (int sb = 0; sb < 16; sb++) {
        const float scale = d * (float)(sc[sb] & 0x0F);
        const float min_val = dmin * (float)((sc[sb] >> 4) & 0x0F);
        for (int j = 0; j < 16; j++) {
            const int idx = sb * 16 + j;
            const float q = (float)((qs[idx / 4] >> ((idx % 4) * 2)) & 0x03);
            emit(c, idx, scale * q - min_val);
        }
    }
}

static void blk_iq4_nl(const uint8_t* blk, emit_fn emit, void* c) { /* compute.rs:1004-1030 */
    const float d = f16(blk);
    for (int j = 0; j < 16; j++) {
        const uint8_t b = blk[2 + j];
        emit(c, 2 * j, d * kIq4nl[b & 0x0F]);
        emit(c, 2 * j + 1, d * kIq4nl[(b >> 4) & 0x0F]);
    }
}

static void blk_iq4_xs(const uint8_t* blk, emit_fn emit, void* c) { /* compute.rs:1034-1075 */
    const float d = f16(blk);
    const uint32_t sh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8);
    for (int sb = 0; sb < 8; sb++) {
        const uint32_t slw = (uint32_t)blk[4 + (sb / 2) * 2] | ((uint32_t)blk[5 + (sb / 2) * 2] << 8);
        const int sl = sb % 2 == 0 ? (int)(slw & 0x0F) : (int)((slw >> 4) & 0x0F);
        const int shb = (int)((sh >> (2 * sb)) & 0x03);
        const float scale = (float)(sl | (shb << 4)) - 32.0f;
        const uint8_t* q = blk + 20 + sb * 16;
        for (int j = 0; j < 16; j++) {
            emit(c, sb * 32 + 2 * j, d * scale * kIq4nl[q[j] & 0x0F]);
            emit(c, sb * 32 + 2 * j + 1, d * scale * kIq4nl[(q[j] >> 4) & 0x0F]);
        }
    }
}

static void blk_iq3_xxs(const uint8_t* blk, emit_fn emit, void* c) { /* compute.rs:1983-2036 */
    const float d = f16(blk);
    const uint8_t* qs = blk + 2;
    for (int ib = 0; ib < 8; ib++) {
        const uint32_t aux = u32le(qs + 64 + ib * 4);
        const float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
        for (int l = 0; l < 4; l++) {
            const uint8_t signs = ksigns((aux >> (7 * l)) & 127);
            const int e0 = qs[ib * 8 + 2 * l], e1 = qs[ib * 8 + 2 * l + 1];
            for (int j = 0; j < 4; j++) {
                emit(c, ib * 32 + l * 8 + j, db * (float)g_iq3xxs(e0, j) * sgn(signs, j));
                emit(c, ib * 32 + l * 8 + j + 4, db * (float)g_iq3xxs(e1, j) * sgn(signs, j + 4));
            }
        }
    }
}

static void blk_iq3_s(const uint8_t* blk, emit_fn emit, void* c) { /* compute.rs:2042-2131 */
    const float d = f16(blk);
    const uint8_t* qs = blk + 2;
    const uint8_t* qh = qs + 64;
    const uint8_t* signs = qh + 8;
    const uint8_t* scales = signs + 32;
    for (int ib = 0; ib < 8; ib += 2) {
        const uint8_t sbyte = scales[ib / 2];
        const float dbs[2] = {d * (float)(1 + 2 * (int)(sbyte & 0x0F)),
                              d * (float)(1 + 2 * (int)(sbyte >> 4))};
        for (int h = 0; h < 2; h++) {
            const int g = ib + h;
            const int q8 = qh[g];
            for (int l = 0; l < 4; l++) {
                const int e0 = qs[g * 8 + 2 * l] | ((q8 << (8 - 2 * l)) & 256);
                const int e1 = qs[g * 8 + 2 * l + 1] | ((q8 << (7 - 2 * l)) & 256);
                const uint8_t sb = signs[g * 4 + l];
                for (int j = 0; j < 4; j++) {
                    emit(c, g * 32 + l * 8 + j, dbs[h] * (float)g_iq3s(e0, j) * sgn(sb, j));
                    emit(c, g * 32 + l * 8 + j + 4, dbs[h] * (float)g_iq3s(e1, j) * sgn(sb, j + 4));
                }
            }
        }
    }
}

static void blk_iq2_xxs(const uint8_t* blk, emit_fn emit, void* c) { /* compute.rs:2137-2186 */
    const float d = f16(blk);
    for (int ib = 0; ib < 8; ib++) {
        const uint8_t* g = blk + 2 + ib * 8;
        const uint32_t a1 = u32le(g + 4);
        const float db = d * (0.5f + (float)(a1 >> 28)) * 0.25f;
        for (int l = 0; l < 4; l++) {
            const uint8_t signs = ksigns((a1 >> (7 * l)) & 127);
            for (int j = 0; j < 8; j++)
                emit(c, ib * 32 + l * 8 + j, db * (float)g_iq2xxs(g[l], j) * sgn(signs, j));
        }
    }
}

static void blk_iq2_xs(const uint8_t* blk, emit_fn emit, void* c) { /* compute.rs:2192-2240 */
    const float d = f16(blk);
    const uint8_t* qs = blk + 2;
    const uint8_t* scales = qs + 64;
    for (int ib = 0; ib < 8; ib++) {
        const uint8_t sb = scales[ib / 2];
        const int nib = ib % 2 == 0 ? (sb & 0x0F) : (sb >> 4);
        const float db = d * (0.5f + (float)nib) * 0.25f;
        for (int l = 0; l < 4; l++) {
            const uint32_t v = (uint32_t)qs[(ib * 4 + l) * 2] | ((uint32_t)qs[(ib * 4 + l) * 2 + 1] << 8);
            const int e = (int)(v & 511);
            const uint8_t signs = ksigns(v >> 9);
            for (int j = 0; j < 8; j++)
                emit(c, ib * 32 + l * 8 + j, db * (float)g_iq2xs(e, j) * sgn(signs, j));
        }
    }
}

static void (*pick_blk(int type))(const uint8_t*, emit_fn, void*) {
    switch (type) {
        case ORA_Q3_K: return blk_q3_k;
        case ORA_Q2_K: return blk_q2_k;
        case ORA_IQ4_NL: return blk_iq4_nl;
        case ORA_IQ4_XS: return blk_iq4_xs;
        case ORA_IQ3_XXS: return blk_iq3_xxs;
        case ORA_IQ3_S: return blk_iq3_s;
        case ORA_IQ2_XXS: return blk_iq2_xxs;
        case ORA_IQ2_XS: return blk_iq2_xs;
        default: return NULL;
    }
}

typedef struct {
    const float* x;
    float sum;
} dot_ctx;
static void emit_dot(void* c, int idx, float w) {
    dot_ctx* d = (dot_ctx*)c;
    d->sum += w * d->x[idx];
}
typedef struct {
    float* out;
} store_ctx;
static void emit_store(void* c, int idx, float w) { ((store_ctx*)c)->out[idx] = w; }

/* One row of the reference's matvec for a low-bit type; returns -1 for other types. */
int ora_row_lowbit(int type, const uint8_t* w, const float* x, int in_dim, int row, float* y) {
    void (*blk)(const uint8_t*, emit_fn, void*) = pick_blk(type);
    if (!blk) return -1;
    const int bs = ora_lowbit_block(type);
    const size_t bb = ora_lowbit_block_bytes(type);
    const int bpr = in_dim / bs;
    const uint8_t* r = w + (size_t)row * bpr * bb;
    dot_ctx c = {x, 0.0f};
    for (int b = 0; b < bpr; b++) {
        c.x = x + (size_t)b * bs;
        blk(r + (size_t)b * bb, emit_dot, &c);
    }
    *y = c.sum;
    return 0;
}

int ora_dequant_lowbit(const uint8_t* w, int type, int64_t n, float* out) {
    void (*blk)(const uint8_t*, emit_fn, void*) = pick_blk(type);
    if (!blk) return -1;
    const int bs = ora_lowbit_block(type);
    const size_t bb = ora_lowbit_block_bytes(type);
    for (int64_t b = 0; b < n / bs; b++) {
        store_ctx c = {out + b * bs};
        blk(w + b * bb, emit_store, &c);
    }
    return 0;
}
