// matvec.cu — fused GGUF dequant-matvec (Q4_0 / Q8_0 / Q4_K) for sm_100a.
//
// Replaces matvec_quantized (src/metal/compute.rs:157-191) and its Metal kernels
// matvec_q4_0 / matvec_q4_k / matvec_q8_0 (src/metal/shaders/kernels.metal:166-273,
// :575-604), whose CPU forms are src/metal/compute.rs:680-750 and :904-925.
//
// Design (HBM-bound streaming, batch 1):
//  * A warp owns R consecutive output rows; lane l owns the 32-wide chunks
//    c = l, l+32, ... of those rows. Each chunk is one aligned 16-byte (Q4_0, Q4_K)
//    or 2x16-byte (Q8_0) vector load, so a warp reads 512 contiguous bytes per row.
//    Loads run one register stage (U chunks per row) ahead of the arithmetic and
//    across row-group boundaries; the first stage is issued before
//    griddepcontrol.wait, so under programmatic dependent launch (PDL) it overlaps
//    the previous kernel's tail.
//  * The kernel is persistent: x is staged once per CTA by TMA into shared memory
//    with the 128-byte swizzle (chunk c's 16-byte unit u at unit u ^ (c & 7)), so
//    the 8 float4 reads of a chunk are bank-conflict free across a quarter warp; the
//    residual add and RMSNorm are applied there.
//  * Exact decode with one logic op per weight ("denormal decode"): masking a
//    quantized field in place, w & (0xF << s), and reading the word as an fp32 gives
//    the denormal q * 2^(s-149) exactly (s <= 16 keeps q * 2^s below 2^23). x is
//    staged pre-multiplied by 2^(85-s) for each element's field position s, so one
//    FFMA adds q * x * 2^-64 to the chunk sum, and the epilogue multiplies by 2^64.
//    All scalings are powers of two, so the arithmetic is the fp32 dot product of the
//    exact integers q with x; only fp32 FMA rounding remains. Offsets are folded in
//    by chunk sums of x: sum (q-8) x = sum q x - 8 X (Q4_0), sum q x - 128 X for
//    Q8_0 read as unsigned q+128, and scale * sum q x - min * X for Q4_K.
//  * Epilogues fuse what follows the matvec in the decode step: residual add,
//    SwiGLU, RoPE on Q/K, or argmax (LAST index on ties, sampler.rs:572-578).
#include <cstring>
#include <type_traits>

#include "matvec_dev.cuh"

namespace ssd {

// Field positions and the matching power-of-two pre-scale of x. Element k of a
// 32-bit word sits at bit 4k (nibbles: element 2j = low nibble of byte j,
// src/metal/compute.rs:693-699) or 8k (Q8_0 bytes). Fields above bit 16 are first
// shifted down (by 12 for nibbles, 16 for bytes) so that every decoded value is a
// denormal.
constexpr int kScaleBias = 85;         // x'' = x * 2^(85 - s); products carry 2^-64
constexpr float kUnscale = 18446744073709551616.0f;  // 2^64
__host__ __device__ constexpr int nib_pos(int k) { return k <= 4 ? 4 * k : 4 * k - 12; }
__host__ __device__ constexpr int byte_pos(int k) { return (k & 1) * 8; }

__device__ __forceinline__ float den(uint32_t bits) { return __uint_as_float(bits); }

template <int FMT>
struct Chunk;
template <>
struct Chunk<SSD_TYPE_Q4_0> {
    uint4 q;
    uint32_t d;
};
template <>
struct Chunk<SSD_TYPE_Q8_0> {
    uint4 q0, q1;
    uint32_t d;
};
template <>
struct Chunk<SSD_TYPE_Q4_K> {
    uint4 q;
    uint4 m;
};
template <>
struct Chunk<SSD_TYPE_Q5_K> {
    uint4 q0, q1;  // 32 bytes q ^ 0x80, q = low4 | hbit << 4
    uint4 m;       // the super-block header (as Q4_K)
};
template <>
struct Chunk<SSD_TYPE_Q8_K> {
    uint4 q0, q1;  // 32 int8
    uint32_t m;    // f32 d of the super-block
};
template <>
struct Chunk<SSD_TYPE_Q6_K> {
    uint4 q0, q1;  // 32 signed bytes q - 32
    uint32_t m;    // int8 scale of elements 0-15, of 16-31, f16 d
};

// Byte pointers of one row of the library layout (see ssd_weight in common.cuh).
template <int FMT, int MAP>
__device__ __forceinline__ void row_ptr(const MvArgs& a, int R, int v, const uint8_t*& qs,
                                        const uint8_t*& meta) {
    int seg, lr;
    map_row<MAP>(a, R, v, seg, lr);
    const size_t nc = (size_t)(a.cols >> 5);
    const uint8_t* q = seg == 0 ? a.qs[0] : (seg == 1 ? a.qs[1] : a.qs[2]);
    const uint8_t* m = seg == 0 ? a.meta[0] : (seg == 1 ? a.meta[1] : a.meta[2]);
    if constexpr (FMT == SSD_TYPE_Q4_0) {
        qs = q + (size_t)lr * nc * 16;
        meta = m + (size_t)lr * nc * 2;
    } else if constexpr (FMT == SSD_TYPE_Q8_0) {
        qs = q + (size_t)lr * nc * 32;
        meta = m + (size_t)lr * nc * 2;
    } else if constexpr (FMT == SSD_TYPE_Q6_K || FMT == SSD_TYPE_Q8_K) {
        qs = q + (size_t)lr * nc * 32;
        meta = m + (size_t)lr * nc * 4;
    } else if constexpr (FMT == SSD_TYPE_Q5_K) {
        qs = q + (size_t)lr * nc * 32;
        meta = m + (size_t)lr * (nc >> 3) * 16;
    } else {
        qs = q + (size_t)lr * nc * 16;
        meta = m + (size_t)lr * (nc >> 3) * 16;
    }
}

// ---- cp.async staging of weights. Each lane copies its own chunks of a stage into
// its own 16-byte slots of the warp's ring and later reads them back, so completion
// only needs the thread's own cp.async.wait_group (Q4_K / Q5_K headers: the group's
// first lane copies, a __syncwarp after the wait publishes it to the other 7).
// Ring slot sizes per (row, chunk): payload QB bytes, metadata MB bytes (Q4_0 / Q8_0:
// the aligned 4-byte word holding the chunk's f16 d; Q4_K / Q5_K: the super-block's 16
// bytes, one slot per group of 8 lanes).
template <int FMT>
struct Slot {
    static constexpr int QB =
        FMT == SSD_TYPE_Q8_0 || FMT == SSD_TYPE_Q6_K || FMT == SSD_TYPE_Q5_K ||
                FMT == SSD_TYPE_Q8_K
            ? 32
            : 16;
    static constexpr int MB = FMT == SSD_TYPE_Q4_K || FMT == SSD_TYPE_Q5_K ? 16 : 4;
    // Q4_K / Q5_K: the 8 lanes of a group read chunks of one super-block, so its 16-byte
    // header is copied once per group (by the group's first lane) into a slot they share
    static constexpr bool HDR = MB == 16;
    static constexpr int MSLOT = HDR ? 4 * 16 : 32 * MB;  // metadata bytes per (row, step)
};
template <int FMT, int R, int U>
__host__ __device__ constexpr int stage_bytes() {
    return R * U * (32 * Slot<FMT>::QB + Slot<FMT>::MSLOT);
}

// Issues the copies of chunk step u of a stage for one row into the shared addresses
// qdst / mdst. qp / mp point at this lane's chunk of the stage's first step
// (tail-clamped by the caller); for Q4_0 / Q8_0 mp is the aligned 4-byte word holding
// the chunk's f16 d.
__device__ __forceinline__ void cp_async16_s(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4_s(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
template <int FMT>
__device__ __forceinline__ void issue_chunk(uint32_t qdst, uint32_t mdst, const uint8_t* qp,
                                            const uint8_t* mp, bool copy_hdr) {
    cp_async16_s(qdst, qp);
    if constexpr (Slot<FMT>::QB == 32) cp_async16_s(qdst + 16, qp + 16);
    if constexpr (Slot<FMT>::HDR) {
        if (copy_hdr) cp_async16_s(mdst, mp);
    } else {
        cp_async4_s(mdst, mp);
    }
}

// Reads one (row, chunk) slot back: qsrc = payload slot, msrc = metadata slot (for
// Q4_0 / Q8_0 already offset to the f16 d inside the copied 4-byte word).
template <int FMT>
__device__ __forceinline__ void read_chunk(Chunk<FMT>& k, const uint8_t* qsrc, const uint8_t* msrc) {
    if constexpr (FMT == SSD_TYPE_Q4_0) {
        k.q = *reinterpret_cast<const uint4*>(qsrc);
        k.d = *reinterpret_cast<const uint16_t*>(msrc);
    } else if constexpr (FMT == SSD_TYPE_Q8_0) {
        k.q0 = *reinterpret_cast<const uint4*>(qsrc);
        k.q1 = *reinterpret_cast<const uint4*>(qsrc + 16);
        k.d = *reinterpret_cast<const uint16_t*>(msrc);
    } else if constexpr (FMT == SSD_TYPE_Q6_K || FMT == SSD_TYPE_Q8_K) {
        k.q0 = *reinterpret_cast<const uint4*>(qsrc);
        k.q1 = *reinterpret_cast<const uint4*>(qsrc + 16);
        k.m = *reinterpret_cast<const uint32_t*>(msrc);
    } else if constexpr (FMT == SSD_TYPE_Q5_K) {
        k.q0 = *reinterpret_cast<const uint4*>(qsrc);
        k.q1 = *reinterpret_cast<const uint4*>(qsrc + 16);
        k.m = *reinterpret_cast<const uint4*>(msrc);
    } else {
        k.q = *reinterpret_cast<const uint4*>(qsrc);
        k.m = *reinterpret_cast<const uint4*>(msrc);
    }
}
// Bytes by which the stage pointers advance per chunk step of 32 chunks.
template <int FMT>
__host__ __device__ constexpr int q_step() {
    return Slot<FMT>::QB * 32;
}
// Scale bytes per chunk (Q4_K: 16 B per 8 chunks) and per chunk step of 32 chunks.
template <int FMT>
__host__ __device__ constexpr int m_chunk() {
    return FMT == SSD_TYPE_Q6_K || FMT == SSD_TYPE_Q8_K ? 4 : 2;
}
template <int FMT>
__host__ __device__ constexpr int m_step() { return 32 * m_chunk<FMT>(); }
// Q4_0 / Q8_0 copy the aligned word holding a chunk's 2-byte d: the half to read varies.
template <int FMT>
__host__ __device__ constexpr bool has_doff() { return FMT == SSD_TYPE_Q4_0 || FMT == SSD_TYPE_Q8_0; }
// Per-chunk bias sums staged beside x'': one per chunk, Q6_K one per 16-element half.
template <int FMT>
__host__ __device__ constexpr int csum_per_chunk() { return FMT == SSD_TYPE_Q6_K ? 2 : 1; }
// Offset of lane l's chunk l within a row (qs, meta).
template <int FMT>
__device__ __forceinline__ size_t q_lane(int l) { return (size_t)l * Slot<FMT>::QB; }
template <int FMT>
__device__ __forceinline__ size_t m_lane(int l) {
    return Slot<FMT>::MB == 16 ? (size_t)(l >> 3) * 16 : (size_t)l * m_chunk<FMT>();
}

__device__ __forceinline__ uint32_t word_of(const uint4& q, int m) {
    return m == 0 ? q.x : (m == 1 ? q.y : (m == 2 ? q.z : q.w));
}

// Two x'' units of 16 bytes as four fp32 pairs {a01, a23} at shared address addr + OFF.
template <int OFF>
__device__ __forceinline__ void lds_x(uint32_t addr, uint64_t& a01, uint64_t& a23) {
    asm volatile("ld.shared.v2.b64 {%0, %1}, [%2+%3];" : "=l"(a01), "=l"(a23) : "r"(addr), "n"(OFF));
}
__device__ __forceinline__ float sum_f2(uint64_t p) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(p));
    return lo + hi;
}

// acc (an fp32 pair: even, odd elements) += the 8 nibbles of word w times x'' elements
// 0..7 of the word, given as pairs (0,1) (2,3) (4,5) (6,7). Each nibble is masked in
// place and read as a denormal; nibbles 5-7 come from w >> 12. Two fp32 FMAs per
// fma.rn.f32x2, each rounded exactly as fmaf; denormal operands are not flushed. FIRST:
// the chunk's first word starts the pair (multiply, no accumulate).
template <bool FIRST>
__device__ __forceinline__ void nib_word(uint64_t& acc, uint32_t w, uint64_t x01, uint64_t x23,
                                         uint64_t x45, uint64_t x67) {
    if constexpr (FIRST)
        asm(
            "{\n\t"
            ".reg .b32 t0, t1, t2, t3, t4, t5, t6, t7, w2;\n\t"
            ".reg .b64 p0, p1, p2, p3;\n\t"
            "and.b32 t0, %1, 0x0000000F;\n\t"
            "and.b32 t1, %1, 0x000000F0;\n\t"
            "mov.b64 p0, {t0, t1};\n\t"
            "mul.rn.f32x2 %0, p0, %2;\n\t"
            "and.b32 t2, %1, 0x00000F00;\n\t"
            "and.b32 t3, %1, 0x0000F000;\n\t"
            "mov.b64 p1, {t2, t3};\n\t"
            "fma.rn.f32x2 %0, p1, %3, %0;\n\t"
            "shr.u32 w2, %1, 12;\n\t"
            "and.b32 t4, %1, 0x000F0000;\n\t"
            "and.b32 t5, w2, 0x00000F00;\n\t"
            "mov.b64 p2, {t4, t5};\n\t"
            "fma.rn.f32x2 %0, p2, %4, %0;\n\t"
            "and.b32 t6, w2, 0x0000F000;\n\t"
            "and.b32 t7, w2, 0x000F0000;\n\t"
            "mov.b64 p3, {t6, t7};\n\t"
            "fma.rn.f32x2 %0, p3, %5, %0;\n\t"
            "}"
            : "=&l"(acc)
            : "r"(w), "l"(x01), "l"(x23), "l"(x45), "l"(x67));
    else
        asm(
            "{\n\t"
            ".reg .b32 t0, t1, t2, t3, t4, t5, t6, t7, w2;\n\t"
            ".reg .b64 p0, p1, p2, p3;\n\t"
            "and.b32 t0, %1, 0x0000000F;\n\t"
            "and.b32 t1, %1, 0x000000F0;\n\t"
            "mov.b64 p0, {t0, t1};\n\t"
            "fma.rn.f32x2 %0, p0, %2, %0;\n\t"
            "and.b32 t2, %1, 0x00000F00;\n\t"
            "and.b32 t3, %1, 0x0000F000;\n\t"
            "mov.b64 p1, {t2, t3};\n\t"
            "fma.rn.f32x2 %0, p1, %3, %0;\n\t"
            "shr.u32 w2, %1, 12;\n\t"
            "and.b32 t4, %1, 0x000F0000;\n\t"
            "and.b32 t5, w2, 0x00000F00;\n\t"
            "mov.b64 p2, {t4, t5};\n\t"
            "fma.rn.f32x2 %0, p2, %4, %0;\n\t"
            "and.b32 t6, w2, 0x0000F000;\n\t"
            "and.b32 t7, w2, 0x000F0000;\n\t"
            "mov.b64 p3, {t6, t7};\n\t"
            "fma.rn.f32x2 %0, p3, %5, %0;\n\t"
            "}"
            : "+l"(acc)
            : "r"(w), "l"(x01), "l"(x23), "l"(x45), "l"(x67));
}

// acc += the 4 signed bytes of word w (read as unsigned q + 128: one LOP3 per byte does
// the mask and the sign flip) times x'' pairs (0,1) (2,3); bytes 2-3 via w >> 16.
template <bool FIRST>
__device__ __forceinline__ void byte_word(uint64_t& acc, uint32_t w, uint64_t x01, uint64_t x23) {
    if constexpr (FIRST)
        asm(
            "{\n\t"
            ".reg .b32 t0, t1, t2, t3, w2;\n\t"
            ".reg .b64 p0, p1;\n\t"
            "lop3.b32 t0, %1, 0x000000FF, 0x00000080, 0x6A;\n\t"
            "lop3.b32 t1, %1, 0x0000FF00, 0x00008000, 0x6A;\n\t"
            "mov.b64 p0, {t0, t1};\n\t"
            "mul.rn.f32x2 %0, p0, %2;\n\t"
            "shr.u32 w2, %1, 16;\n\t"
            "lop3.b32 t2, w2, 0x000000FF, 0x00000080, 0x6A;\n\t"
            "lop3.b32 t3, w2, 0x0000FF00, 0x00008000, 0x6A;\n\t"
            "mov.b64 p1, {t2, t3};\n\t"
            "fma.rn.f32x2 %0, p1, %3, %0;\n\t"
            "}"
            : "=&l"(acc)
            : "r"(w), "l"(x01), "l"(x23));
    else
        asm(
            "{\n\t"
            ".reg .b32 t0, t1, t2, t3, w2;\n\t"
            ".reg .b64 p0, p1;\n\t"
            "lop3.b32 t0, %1, 0x000000FF, 0x00000080, 0x6A;\n\t"
            "lop3.b32 t1, %1, 0x0000FF00, 0x00008000, 0x6A;\n\t"
            "mov.b64 p0, {t0, t1};\n\t"
            "fma.rn.f32x2 %0, p0, %2, %0;\n\t"
            "shr.u32 w2, %1, 16;\n\t"
            "lop3.b32 t2, w2, 0x000000FF, 0x00000080, 0x6A;\n\t"
            "lop3.b32 t3, w2, 0x0000FF00, 0x00008000, 0x6A;\n\t"
            "mov.b64 p1, {t2, t3};\n\t"
            "fma.rn.f32x2 %0, p1, %3, %0;\n\t"
            "}"
            : "+l"(acc)
            : "r"(w), "l"(x01), "l"(x23));
}

// acc[r] = sum over a 16-byte nibble chunk of q * x''. The chunk's x'' unit u is at
// shared address xq[u] + XOFF (x'' pre-scaled per field position, see nib_pos).
template <int R, int XOFF>
__device__ __forceinline__ void nib_dot(const uint32_t (&xq)[8], const uint4 (&q)[R],
                                        uint64_t (&acc)[R]) {
#pragma unroll
    for (int m = 0; m < 4; m++) {
        uint64_t x01, x23, x45, x67;
        lds_x<XOFF>(xq[2 * m], x01, x23);
        lds_x<XOFF>(xq[2 * m + 1], x45, x67);
#pragma unroll
        for (int r = 0; r < R; r++) {
            if (m == 0)
                nib_word<true>(acc[r], word_of(q[r], m), x01, x23, x45, x67);
            else
                nib_word<false>(acc[r], word_of(q[r], m), x01, x23, x45, x67);
        }
    }
}

// Per-chunk data staged next to x'': csum[c] = bias term of the chunk, already scaled
// by 2^-64: -8 X (Q4_0), -128 X (Q8_0), X (Q4_K), X = sum of the chunk's x. b = csum of
// this chunk; the chunk's x'' unit u is at shared address xq[u] + XOFF.
template <int FMT, int R, int XOFF>
__device__ __forceinline__ void compute_chunk(const Chunk<FMT> (&ch)[R], const uint32_t (&xq)[8],
                                              float b, float b2, int lane, float (&acc)[R]) {
    uint64_t eo[R];
    if constexpr (FMT == SSD_TYPE_Q4_0) {
        uint4 q[R];
#pragma unroll
        for (int r = 0; r < R; r++) q[r] = ch[r].q;
        nib_dot<R, XOFF>(xq, q, eo);
#pragma unroll
        for (int r = 0; r < R; r++)
            acc[r] = fmaf(f16_bits_to_f32((uint16_t)ch[r].d), sum_f2(eo[r]) + b, acc[r]);
    } else if constexpr (FMT == SSD_TYPE_Q8_0) {
#pragma unroll
        for (int m = 0; m < 8; m++) {  // unit m = elements 4m..4m+3
            uint64_t x01, x23;
            lds_x<XOFF>(xq[m], x01, x23);
#pragma unroll
            for (int r = 0; r < R; r++) {
                const uint32_t w = word_of(m < 4 ? ch[r].q0 : ch[r].q1, m & 3);
                if (m == 0)
                    byte_word<true>(eo[r], w, x01, x23);
                else
                    byte_word<false>(eo[r], w, x01, x23);
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++)
            acc[r] = fmaf(f16_bits_to_f32((uint16_t)ch[r].d), sum_f2(eo[r]) + b, acc[r]);
    } else if constexpr (FMT == SSD_TYPE_Q8_K) {  // Q8_0's decode, f32 d per super-block
#pragma unroll
        for (int m = 0; m < 8; m++) {
            uint64_t x01, x23;
            lds_x<XOFF>(xq[m], x01, x23);
#pragma unroll
            for (int r = 0; r < R; r++) {
                const uint32_t w = word_of(m < 4 ? ch[r].q0 : ch[r].q1, m & 3);
                if (m == 0)
                    byte_word<true>(eo[r], w, x01, x23);
                else
                    byte_word<false>(eo[r], w, x01, x23);
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = fmaf(__uint_as_float(ch[r].m), sum_f2(eo[r]) + b, acc[r]);
    } else if constexpr (FMT == SSD_TYPE_Q6_K) {
        // signed bytes q - 32 decoded as Q8_0's (q + 128 read unsigned); elements 0-15 and
        // 16-31 have their own scale, so each half has its own pair and bias (b, b2):
        // sum (d * sc_h) * q * x = (d * sc_h) * (sum q x) per half (compute.rs:768-785)
        uint64_t eh[R];
#pragma unroll
        for (int m = 0; m < 8; m++) {  // unit m = elements 4m..4m+3
            uint64_t x01, x23;
            lds_x<XOFF>(xq[m], x01, x23);
#pragma unroll
            for (int r = 0; r < R; r++) {
                const uint32_t w = word_of(m < 4 ? ch[r].q0 : ch[r].q1, m & 3);
                if (m == 0)
                    byte_word<true>(eo[r], w, x01, x23);
                else if (m < 4)
                    byte_word<false>(eo[r], w, x01, x23);
                else if (m == 4)
                    byte_word<true>(eh[r], w, x01, x23);
                else
                    byte_word<false>(eh[r], w, x01, x23);
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++) {
            const uint32_t mw = ch[r].m;
            const float d = f16_bits_to_f32((uint16_t)(mw >> 16));
            const float s0 = __fmul_rn(d, (float)(int)(int8_t)(mw & 0xFF));
            const float s1 = __fmul_rn(d, (float)(int)(int8_t)((mw >> 8) & 0xFF));
            acc[r] = fmaf(s1, sum_f2(eh[r]) + b2, fmaf(s0, sum_f2(eo[r]) + b, acc[r]));
        }
    } else if constexpr (FMT == SSD_TYPE_Q5_K) {
        // bytes q ^ 0x80 decoded as Q8_0's (q read back unsigned), then Q4_K's per
        // sub-block scale and min: sum (scale q - min) x = scale sum q x - min X
#pragma unroll
        for (int m = 0; m < 8; m++) {
            uint64_t x01, x23;
            lds_x<XOFF>(xq[m], x01, x23);
#pragma unroll
            for (int r = 0; r < R; r++) {
                const uint32_t w = word_of(m < 4 ? ch[r].q0 : ch[r].q1, m & 3);
                if (m == 0)
                    byte_word<true>(eo[r], w, x01, x23);
                else
                    byte_word<false>(eo[r], w, x01, x23);
            }
        }
        const float X = b;
        const int sb = lane & 7, sh = 8 * (sb & 3);
        const uint32_t sa = sb < 4 ? 0u : 6u, ma = sb < 4 ? 63u : 3u, m8 = sb < 4 ? 0u : 15u;
#pragma unroll
        for (int r = 0; r < R; r++) {
            const uint4 m = ch[r].m;
            const float d = f16_bits_to_f32((uint16_t)(m.x & 0xFFFF));
            const float dmin = f16_bits_to_f32((uint16_t)(m.x >> 16));
            const uint32_t yb = m.y >> sh, zb = m.z >> sh, wb = m.w >> sh;
            const uint32_t s6 = ((yb >> sa) & ma) | ((wb & m8) << 2);
            const uint32_t m6 = ((zb >> sa) & ma) | (((wb >> 4) & m8) << 2);
            const float scale = __fmul_rn(d, (float)s6);
            const float mn = __fmul_rn(dmin, (float)m6);
            acc[r] = fmaf(-mn, X, fmaf(scale, sum_f2(eo[r]), acc[r]));
        }
    } else {  // Q4_K: this lane's sub-block index is c & 7 == lane & 7
        uint4 q[R];
#pragma unroll
        for (int r = 0; r < R; r++) q[r] = ch[r].q;
        nib_dot<R, XOFF>(xq, q, eo);
        const float X = b;
        // 6-bit scale / min of sub-block sb (src/metal/compute.rs:725-733): sb < 4 takes the
        // low 6 bits of header bytes 4 + sb / 8 + sb; sb >= 4 their top 2 bits joined with
        // the low / high nibble of byte 12 + sb - 4. Branch-free with lane-constant shifts
        // and masks (sb = lane & 7 differs within each group of 8 lanes).
        const int sb = lane & 7, sh = 8 * (sb & 3);
        const uint32_t sa = sb < 4 ? 0u : 6u, ma = sb < 4 ? 63u : 3u, m8 = sb < 4 ? 0u : 15u;
#pragma unroll
        for (int r = 0; r < R; r++) {
            const uint4 m = ch[r].m;
            const float d = f16_bits_to_f32((uint16_t)(m.x & 0xFFFF));
            const float dmin = f16_bits_to_f32((uint16_t)(m.x >> 16));
            const uint32_t yb = m.y >> sh, zb = m.z >> sh, wb = m.w >> sh;
            const uint32_t s6 = ((yb >> sa) & ma) | ((wb & m8) << 2);
            const uint32_t m6 = ((zb >> sa) & ma) | (((wb >> 4) & m8) << 2);
            // sum((scale*q - min) x) = scale * sum(q x) - min * X
            const float scale = __fmul_rn(d, (float)s6);
            const float mn = __fmul_rn(dmin, (float)m6);
            acc[r] = fmaf(-mn, X, fmaf(scale, sum_f2(eo[r]), acc[r]));
        }
    }
}

// Shared-memory plan of one CTA (offsets from a 1024-byte aligned base): the staged
// x'' (TMA destination, swizzled), the per-chunk bias sums, reduction scratch, the
// TMA barrier, and one weight ring of n_stages stages per warp: 4 for the 16-warp CTAs
// that own an SM, 3 for the 8-warp CTAs sized so that two CTAs fit on an SM (the next
// kernel's CTAs can then start their weight prefetch beside the previous kernel's).
template <int NW>
__host__ __device__ constexpr int n_stages() { return NW >= 16 ? 4 : 3; }
struct SmemPlan {
    int nc, xrows;  // chunks, staged rows (multiple of kVecBoxRows)
    size_t xs, csum, red, bar, rope, ring, total;
};
__host__ __device__ inline SmemPlan smem_plan(int cols, int nw, int ring_per_warp,
                                              int csum_per_chunk = 1) {
    SmemPlan p;
    p.nc = cols >> 5;
    p.xrows = (p.nc + kVecBoxRows - 1) / kVecBoxRows * kVecBoxRows;
    size_t o = 0;
    p.xs = o;
    o += (size_t)p.xrows * 128;
    p.csum = o;
    o += ((size_t)p.nc * 4 * csum_per_chunk + 15) & ~(size_t)15;
    p.red = o;
    o += 64 * 4 + (size_t)nw * 8;
    p.bar = o;
    o += 16;
    p.rope = o;
    o += (size_t)kMaxRopePairs * 8;
    o = (o + 127) & ~(size_t)127;
    p.ring = o;
    o += (size_t)nw * ring_per_warp;
    p.total = o + 1024;  // alignment slack
    return p;
}

// Power-of-two pre-scale of element position k (0..7) within a 32-bit word.
template <int FMT>
__device__ __forceinline__ float pos_scale(int k) {
    const int s = Slot<FMT>::QB == 32 ? byte_pos(k & 3) : nib_pos(k);
    return __uint_as_float((uint32_t)(127 + kScaleBias - s) << 23);
}

// Persistent fused dequant-matvec. Grid = resident CTAs (or fewer for small matrices);
// CTA b owns the contiguous row-groups (R rows) [b n_rg / G, (b + 1) n_rg / G) (G = gridDim.x;
// counts differ by at most one), its warps taking them round robin. A "stage" is U chunk steps (32 chunks each) of the R rows of one row-group;
// each warp keeps kStages - 1 stages of copies in flight in its shared-memory ring,
// the first ones issued before griddepcontrol.wait.
template <int FMT, int EPI, int R, int U, int NW>
__global__ void __launch_bounds__(NW * 32, NW >= 16 ? 1 : 2)
    k_matvec(const MvArgs a, const __grid_constant__ CUtensorMap tm_x) {
    constexpr int kStages = n_stages<NW>();
    constexpr int SB = stage_bytes<FMT, R, U>();
    constexpr int QB = Slot<FMT>::QB, MB = Slot<FMT>::MB;
    static_assert(U == 1 || U == 2, "chunk steps per stage");
    constexpr int kMap = epi_map(EPI);  // launch_matvec checks a.map against it
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const SmemPlan P = smem_plan(a.cols, NW, kStages * SB, csum_per_chunk<FMT>());
    float4* xs4 = reinterpret_cast<float4*>(base + P.xs);
    float* csum = reinterpret_cast<float*>(base + P.csum);
    float* red = reinterpret_cast<float*>(base + P.red);
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(base + P.red + 256);
    // EPI_PEERS: the CTA's output rows collect in the `red` region (free after the prologue)
    // when they fit, then go out as contiguous stores
    float* peer_buf = red;
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + P.bar);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint8_t* ring = base + P.ring + (size_t)warp * (kStages * SB);
    const int nc = P.nc;
    const int iters = (nc + 31) >> 5;     // chunk iterations per lane per row
    const int spr = (iters + U - 1) / U;  // stages per row-group
    const int n_rg = (a.rows + R - 1) / R;
    // Every SM gets floor or ceil of n_rg / gridDim.x row-groups, as one contiguous range. The
    // SM's issue rate bounds these kernels, so an even share per SM (its warps finish at
    // different times) is what balances the tail; dealing per warp gave some SMs twice as
    // many. Contiguous rows let the peer epilogue store a CTA's outputs as whole lines.
    const int rg_lo = (int)((long long)n_rg * blockIdx.x / gridDim.x);
    const int rg_hi = (int)((long long)n_rg * (blockIdx.x + 1) / gridDim.x);
    const int wg = rg_lo + warp;
    const int my_rg = wg < rg_hi ? (rg_hi - 1 - wg) / NW + 1 : 0;
    const bool peer_buffered = EPI == EPI_PEERS && (rg_hi - rg_lo) * R <= (64 * 4 + NW * 8) / 4;
    const int total = my_rg * spr;  // stages this warp computes

    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }

    // ---- issue cursor: row-group lrg, stage lst; lq / lm = this lane's chunk of the
    // stage in each row (rows past the end alias the last row; their sums are dropped).
    // Steps whose chunks run past the row (the tail of a row whose chunk count is not a
    // multiple of 32*U) re-read the lane's last chunk; compute skips those chunks.
    int lrg = wg, lst = 0, issued = 0;
    const uint8_t* lq[R];
    const uint8_t* lm[R];
    // largest c < nc with c = lane (mod 32); lanes with no chunk at all (nc < 32) use 0
    const int last_c = lane < nc ? nc - 1 - ((nc - 1 - lane) & 31) : 0;
    auto set_rows = [&]() {
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int v = min(lrg * R + r, a.rows - 1);
            const uint8_t *q0, *m0;
            row_ptr<FMT, kMap>(a, R, v, q0, m0);
            lq[r] = q0 + q_lane<FMT>(lane < nc ? lane : 0);
            lm[r] = m0 + m_lane<FMT>(lane < nc ? lane : 0);
            // Q4_0 / Q8_0: the aligned 4-byte word holding the d (stays aligned: the
            // pointer advances by multiples of 64 bytes)
            if constexpr (has_doff<FMT>())
                lm[r] = reinterpret_cast<const uint8_t*>((uintptr_t)lm[r] & ~(uintptr_t)3);
        }
    };
    if (lrg < rg_hi) set_rows();
    const bool any_tail = nc % (32 * U) != 0 || nc < 32;
    // this lane's slots: payload at ring_q + stage + (r*U+u)*32*QB, metadata at
    // ring_m + stage + (r*U+u)*MSLOT (compile-time offsets from two lane pointers; Q4_K /
    // Q5_K lanes point at their group's shared header slot)
    uint8_t* const ring_q = ring + (size_t)lane * QB;
    uint8_t* const ring_m = ring + (size_t)R * U * 32 * QB +
                            (Slot<FMT>::HDR ? (size_t)(lane >> 3) * 16 : (size_t)lane * MB);
    const bool copy_hdr = (lane & 7) == 0;
    const uint32_t ring_qs = smem_u32(ring_q), ring_ms = smem_u32(ring_m);  // copy targets
    int ist = 0;  // byte offset of the stage being issued
    auto issue = [&]() {  // the next stage into the ring, then commit
        if (issued < total) {
            if (!any_tail || (lst + 1) * U * 32 <= nc) {
#pragma unroll
                for (int r = 0; r < R; r++) {
#pragma unroll
                    for (int u = 0; u < U; u++)
                        issue_chunk<FMT>(ring_qs + ist + (r * U + u) * 32 * QB,
                                         ring_ms + ist + (r * U + u) * Slot<FMT>::MSLOT,
                                         lq[r] + u * q_step<FMT>(), lm[r] + u * m_step<FMT>(),
                                         copy_hdr);
                }
            } else {  // tail stage: chunks past the row end re-read the lane's last chunk
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int cu = lane + 32 * (lst * U + u);
                    const int cp = (lane < nc ? lane : 0) + 32 * (lst * U + u);
                    // chunk-index step back to last_c: the same stride per chunk index in
                    // qs (16 or 32 B) and 2 B in meta (Q4_K: 16 B per 8 chunks, dc a
                    // multiple of 32)
                    const long long dc = cu < nc ? 0 : (long long)(last_c - cp);
#pragma unroll
                    for (int r = 0; r < R; r++)
                        issue_chunk<FMT>(ring_qs + ist + (r * U + u) * 32 * QB,
                                         ring_ms + ist + (r * U + u) * Slot<FMT>::MSLOT,
                                         lq[r] + u * q_step<FMT>() + dc * (q_step<FMT>() / 32),
                                         lm[r] + u * m_step<FMT>() + dc * m_chunk<FMT>(),
                                         copy_hdr);
                }
            }
#pragma unroll
            for (int r = 0; r < R; r++) {
                lq[r] += U * q_step<FMT>();
                lm[r] += U * m_step<FMT>();
            }
            issued++;
            ist = ist + SB == kStages * SB ? 0 : ist + SB;
            if (++lst == spr) {
                lst = 0;
                lrg += NW;
                if (lrg < rg_hi) set_rows();
            }
        }
        cp_commit();  // one group per call, empty or not: wait_group counts stay uniform
    };
    // Weights never depend on the previous kernel: fill the ring before waiting.
#pragma unroll
    for (int k = 0; k < kStages - 1; k++) issue();
    __syncthreads();  // barrier initialised
    float2* rope_tab = reinterpret_cast<float2*>(base + P.rope);
    // finish: chunk bias sum (8 consecutive threads hold one chunk's 8 units) and the
    // per-position power-of-two pre-scale, in place
    auto finish = [&](int i, int c, int ph, float4 v, unsigned gmask) {
        float t = (v.x + v.y) + (v.z + v.w);
        t += __shfl_xor_sync(gmask, t, 1);
        t += __shfl_xor_sync(gmask, t, 2);
        if constexpr (FMT == SSD_TYPE_Q6_K) {  // per 16-element half: units 0-3, 4-7
            if ((i & 3) == 0) csum[2 * c + ((i >> 2) & 1)] = -128.0f * __fmul_rn(t, 1.0f / kUnscale);
        } else {
            t += __shfl_xor_sync(gmask, t, 4);
            if ((i & 7) == 0) {
                const float X = __fmul_rn(t, 1.0f / kUnscale);
                csum[c] = FMT == SSD_TYPE_Q4_0 ? -8.0f * X
                          : (FMT == SSD_TYPE_Q8_0 || FMT == SSD_TYPE_Q8_K) ? -128.0f * X
                                                                           : X;
            }
        }
        // word position of v.x
        const int k0 = Slot<FMT>::QB == 32 ? 0 : 4 * (i & 1);
        v.x = __fmul_rn(v.x, pos_scale<FMT>(k0 + 0));
        v.y = __fmul_rn(v.y, pos_scale<FMT>(k0 + 1));
        v.z = __fmul_rn(v.z, pos_scale<FMT>(k0 + 2));
        v.w = __fmul_rn(v.w, pos_scale<FMT>(k0 + 3));
        xs4[ph] = v;
    };
    if (!mv_prologue<NW * 32, EPI>(a, &tm_x, base + P.xs, nc, P.xrows, red, bar, rope_tab, finish)) {
        cp_wait<0>();
        if (a.x_ready) pdl_wait();
        return;
    }

    float acc[R];
#pragma unroll
    for (int r = 0; r < R; r++) acc[r] = 0.0f;
    unsigned long long best = 0ull;
    int crg = wg, cst = 0;  // compute cursor
    // byte offset of the f16 d inside its copied aligned 4-byte word: the half of
    // byte offset 2 * (row * nc + c) in the segment, c = lane (mod 2)
    int doff[R];
    auto set_doff = [&]() {
#pragma unroll
        for (int r = 0; r < R; r++) {
            int seg, lr;
            map_row<kMap>(a, R, min(crg * R + r, a.rows - 1), seg, lr);
            doff[r] = (((lr & 1) * (nc & 1) + lane) & 1) * 2;
        }
    };
    if (has_doff<FMT>() && crg < rg_hi) set_doff();
    int cst_off = 0;  // byte offset of the stage being computed
    // this lane's shared address of x'' unit u of its chunk c = lane (mod 32): row c of
    // 128 bytes, unit u at slot u ^ (c & 7) = u ^ (lane & 7); chunk c + 32 t is 4096 t
    // bytes further
    uint32_t xp[8];
#pragma unroll
    for (int u = 0; u < 8; u++) xp[u] = smem_u32(xs4) + lane * 128 + ((u ^ (lane & 7)) << 4);

    for (int k = 0; k < total; k++) {
        cp_wait<kStages - 2>();  // this thread's copies of stage k have landed
        // the group's shared header was copied by its first lane: make it visible
        if constexpr (Slot<FMT>::HDR) __syncwarp();
        const uint8_t* sq = ring_q + cst_off;
        const uint8_t* sm = ring_m + cst_off;
        uint32_t xst[8];  // x'' units of this stage's first chunk step
#pragma unroll
        for (int u = 0; u < 8; u++) xst[u] = xp[u] + (uint32_t)cst * (U * 4096);
        const float* cs = csum + (lane + 32 * U * cst) * csum_per_chunk<FMT>();
        auto do_u = [&](auto uc) {  // chunk step u (a compile-time constant)
            constexpr int u = decltype(uc)::value;
            Chunk<FMT> ch[R];
#pragma unroll
            for (int r = 0; r < R; r++)
                read_chunk<FMT>(ch[r], sq + (r * U + u) * 32 * QB,
                                sm + (r * U + u) * Slot<FMT>::MSLOT + (has_doff<FMT>() ? doff[r] : 0));
            constexpr int CPC = csum_per_chunk<FMT>();
            compute_chunk<FMT, R, u * 4096>(ch, xst, cs[32 * u * CPC], CPC == 2 ? cs[32 * u * CPC + 1] : 0.0f,
                                            lane, acc);
        };
        using U0 = std::integral_constant<int, 0>;
        using U1 = std::integral_constant<int, (U > 1 ? 1 : 0)>;
        if (!any_tail || (cst + 1) * U * 32 <= nc) {
            do_u(U0{});
            if constexpr (U > 1) do_u(U1{});
        } else {
            if (lane + 32 * (cst * U) < nc) do_u(U0{});
            if constexpr (U > 1)
                if (lane + 32 * (cst * U + 1) < nc) do_u(U1{});
        }
        cst_off = cst_off + SB == kStages * SB ? 0 : cst_off + SB;
        issue();  // refill the buffer of stage k - 1 (this thread is done reading it)
        if (++cst != spr) continue;
        // row-group finished: reduce across the warp and run the epilogue
        cst = 0;
        const int v0 = crg * R;
        crg += NW;
        if (has_doff<FMT>() && crg < rg_hi) set_doff();
        float res[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            res[r] = __fmul_rn(warp_sum(acc[r]), kUnscale);
            acc[r] = 0.0f;
        }
        if constexpr (EPI == EPI_STORE || EPI == EPI_RESID) {
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int row = v0 + r;
                if (lane == r && row < a.rows)
                    a.y[row] = (EPI == EPI_RESID) ? __fadd_rn(a.base[row], res[r]) : res[r];
            }
        } else if constexpr (EPI == EPI_PEERS) {  // partial rows, sent at the end (below)
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int row = v0 + r;
                if (row < a.rows) {
                    if (peer_buffered) {
                        if (lane == r) peer_buf[row - rg_lo * R] = res[r];
                    } else if (lane < a.ar_out_n) {
                        a.ar_out[lane][row] = res[r];
                    }
                }
            }
        } else if constexpr (EPI == EPI_SWIGLU) {  // rows: R/2 gate rows, then R/2 up rows
            constexpr int H = R / 2;
            if (lane < H && v0 < a.rows) {
                float g = res[0], up = res[H];
#pragma unroll
                for (int j = 1; j < H; j++)
                    if (lane == j) {
                        g = res[j];
                        up = res[H + j];
                    }
                // silu(v) = v / (1 + exp(-v)), then gate *= up (feed_forward.rs:31-39,
                // compute.rs:641-645)
                const float si = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
                a.y[(v0 / R) * H + lane] = __fmul_rn(si, up);
            }
        } else if constexpr (EPI == EPI_QKV_ROPE) {  // adjacent pairs (v0+2p, v0+2p+1)
            if (lane < R / 2 && v0 < a.rows) {
                int seg, lr;
                map_row<kMap>(a, R, v0 + 2 * lane, seg, lr);
                float x0 = res[0], x1 = res[1];
#pragma unroll
                for (int p = 1; p < R / 2; p++)
                    if (lane == p) {
                        x0 = res[2 * p];
                        x1 = res[2 * p + 1];
                    }
                if (seg < 2) rope_apply(x0, x1, rope_tab[(lr % a.head_dim) >> 1]);
                float* dst = seg == 0 ? a.y : (seg == 1 ? a.y_k : a.y_v);
                dst[lr] = x0;
                dst[lr + 1] = x1;
            }
        } else {  // EPI_ARGMAX
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int row = v0 + r;
                if (row < a.rows) {
                    if (a.y && lane == r) a.y[row] = res[r];
                    const unsigned long long kk = argmax_key(res[r], (uint32_t)(row + a.index_offset));
                    best = kk > best ? kk : best;
                }
            }
        }
    }
    cp_wait<0>();

    if constexpr (EPI == EPI_PEERS) {
        if (peer_buffered) {  // this CTA's contiguous rows, as whole lines to every rank
            __syncthreads();
            const int row0 = rg_lo * R, nrow = min(rg_hi * R, a.rows) - row0;
            for (int p = 0; p < a.ar_out_n; p++)
                for (int i = tid; i < nrow; i += NW * 32) a.ar_out[p][row0 + i] = peer_buf[i];
        }
        peers_publish(a);  // then the last CTA raises the flags on every rank
    }

    if constexpr (EPI == EPI_ARGMAX) {
        if (lane == 0) keys[warp] = best;
        __syncthreads();
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int w = 0; w < NW; w++) b = keys[w] > b ? keys[w] : b;
            if (b) atomicMax(a.argmax_key, b);
        }
    }
    if (a.x_ready) pdl_wait();  // an independent launch ends after its predecessor
}

// --------------------------------------------------------------- host side

struct Cfg {
    int R, U, NW;
};

// SSD_MV_CONFIG="R,U,NW" selects a tiling of the instantiated set for every matvec
// (tuning sweeps); unset, launch_fmt_epi picks one by shape.
static Cfg env_cfg() {
    static Cfg c = [] {
        Cfg d{0, 0, 0};
        const char* s = getenv("SSD_MV_CONFIG");
        if (s) {
            int r, u, nw;
            if (sscanf(s, "%d,%d,%d", &r, &u, &nw) == 3) d = Cfg{r, u, nw};
        }
        return d;
    }();
    return c;
}

template <int FMT, int EPI, int R, int U, int NW>
static int launch_t(ssd_ctx* ctx, const MvArgs& a, cudaStream_t s, bool pdl) {
    auto kern = k_matvec<FMT, EPI, R, U, NW>;
    const SmemPlan P =
        smem_plan(a.cols, NW, n_stages<NW>() * stage_bytes<FMT, R, U>(), csum_per_chunk<FMT>());
    SSD_REQ(P.total <= ctx->smem_optin, SSD_ERR_SHAPE,
            "cols %d too large for shared-memory staging (%zu bytes)", a.cols, P.total);
    int nb = 0;
    SSD_TRY(occupancy(ctx, kern, NW * 32, P.total, &nb));
    const int n_rg = (a.rows + R - 1) / R;
    const int need = (n_rg + NW - 1) / NW;
    const int grid = need < ctx->num_sms * nb ? need : ctx->num_sms * nb;
    CUtensorMap mx;
    SSD_TRY(encode_vec_map(&mx, a.x, a.cols));
    SSD_CK(launch_pdl(kern, dim3(grid), dim3(NW * 32), P.total, s, pdl, a, mx));
    return SSD_OK;
}

// Tiling by shape. Rows per warp R = 4 (x reads from shared memory shared by 4 rows)
// unless that leaves fewer than ~16 warps per SM, then R = 2. Q4_0 keeps two chunk
// steps per register stage (U = 2); Q8_0 (32-byte chunks) and Q4_K (16 more bytes of
// super-block metadata per chunk) one, which keeps them spill-free. 8 warps per CTA
// while two CTAs' x staging fits in shared memory, else 16 (one CTA per SM).
// Tiling by shape: R = 2 rows per warp, U = 2 chunk steps per stage (Q4_0; one for the
// wider Q8_0 / Q4_K slots), kStages = 4 ring stages per warp. 16 warps per CTA (one
// CTA per SM, one copy of x'' per SM) when their rings fit beside x'' in shared
// memory; for very wide rows Q4_0 first halves its stage (U = 1) to keep 16 warps;
// else 8 warps.
template <int FMT, int EPI>
static int launch_fmt_epi(ssd_ctx* ctx, const MvArgs& a, cudaStream_t s, bool pdl) {
    constexpr int U = FMT == SSD_TYPE_Q4_0 || FMT == SSD_TYPE_Q4_K ? 2 : 1;
    const Cfg c = env_cfg();
    if (c.R) {  // tuning: any instantiated (R, U, NW)
        if (c.U == U && c.NW == 8 && c.R == 2) return launch_t<FMT, EPI, 2, U, 8>(ctx, a, s, pdl);
        if (c.U == U && c.NW == 8 && c.R == 4) return launch_t<FMT, EPI, 4, U, 8>(ctx, a, s, pdl);
        if (c.U == U && c.NW == 16 && c.R == 2) return launch_t<FMT, EPI, 2, U, 16>(ctx, a, s, pdl);
        if (c.U == U && c.NW == 16 && c.R == 4) return launch_t<FMT, EPI, 4, U, 16>(ctx, a, s, pdl);
        if constexpr (U == 2) {
            if (c.U == 1 && c.NW == 8 && c.R == 4) return launch_t<FMT, EPI, 4, 1, 8>(ctx, a, s, pdl);
            if (c.U == 1 && c.NW == 16 && c.R == 4) return launch_t<FMT, EPI, 4, 1, 16>(ctx, a, s, pdl);
            if (c.U == 1 && c.NW == 16 && c.R == 2) return launch_t<FMT, EPI, 2, 1, 16>(ctx, a, s, pdl);
        }
        set_error("SSD_MV_CONFIG=%d,%d,%d is not an instantiated tiling", c.R, c.U, c.NW);
        return SSD_ERR_ARG;
    }
    static const bool coresident = [] {
        const char* e = getenv("SSD_MV_COAL");
        return e && e[0] == '1';
    }();
    if (coresident &&
        2 * (smem_plan(a.cols, 8, n_stages<8>() * stage_bytes<FMT, 2, U>(), csum_per_chunk<FMT>())
                 .total +
             1024) <=
            ctx->smem_per_sm)
        return launch_t<FMT, EPI, 2, U, 8>(ctx, a, s, pdl);
    const int ring = n_stages<16>() * stage_bytes<FMT, 2, U>();
    if (smem_plan(a.cols, 16, ring, csum_per_chunk<FMT>()).total <= ctx->smem_optin)
        return launch_t<FMT, EPI, 2, U, 16>(ctx, a, s, pdl);
    if constexpr (U == 2) {  // wide rows (x'' over 100 KB): halve the stage, keep 16 warps
        if (smem_plan(a.cols, 16, n_stages<16>() * stage_bytes<FMT, 2, 1>()).total <=
            ctx->smem_optin)
            return launch_t<FMT, EPI, 2, 1, 16>(ctx, a, s, pdl);
    }
    return launch_t<FMT, EPI, 2, U, 8>(ctx, a, s, pdl);
}

template <int FMT>
static int launch_fmt(ssd_ctx* ctx, int epi, const MvArgs& a, cudaStream_t s, bool pdl) {
    switch (epi) {
        case EPI_STORE: return launch_fmt_epi<FMT, EPI_STORE>(ctx, a, s, pdl);
        case EPI_RESID: return launch_fmt_epi<FMT, EPI_RESID>(ctx, a, s, pdl);
        case EPI_SWIGLU: return launch_fmt_epi<FMT, EPI_SWIGLU>(ctx, a, s, pdl);
        case EPI_QKV_ROPE: return launch_fmt_epi<FMT, EPI_QKV_ROPE>(ctx, a, s, pdl);
        case EPI_ARGMAX: return launch_fmt_epi<FMT, EPI_ARGMAX>(ctx, a, s, pdl);
        case EPI_PEERS: return launch_fmt_epi<FMT, EPI_PEERS>(ctx, a, s, pdl);
        default: set_error("bad epilogue %d", epi); return SSD_ERR_ARG;
    }
}

static inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// Dense rows: F16 / BF16 (matvec_f16_cpu / matvec_bf16_cpu, src/metal/compute.rs:2250-2285)
// and F32 (matvec_f32_simd, :378-424). Each CTA takes a contiguous, balanced range of output
// rows (counts differ by at most one between CTAs, so no half-empty second pass over a few
// leftover rows), kDenseRows weight rows at a time: its 256 threads split the columns
// (thread t owns the 16 bytes at element EPL*t of every 256*EPL-element step, EPL = 8 for
// 16-bit and 4 for f32 elements, when cols % EPL == 0; single columns otherwise), x is
// loaded once per step for all rows of the group, each warp sums its share, and thread i
// adds the 8 warp partials of row i in warp order. y = W x, or base + W x; with EPI_SWIGLU
// the group's rows are gate r, up r, gate r+1, up r+1 (qs[0], qs[1]) and output r is
// silu(gate r) * up r (the fused_swiglu_f32 shader, kernels.metal:1475-1500).
constexpr int kDenseRows = 4;

template <int DT>
__device__ __forceinline__ float dense_elem(const void* base, size_t i) {
    if (DT == SSD_TYPE_F32) return __ldg(reinterpret_cast<const float*>(base) + i);
    const uint32_t h = __ldg(reinterpret_cast<const uint16_t*>(base) + i);
    return DT == SSD_TYPE_BF16 ? __uint_as_float(h << 16) : f16_bits_to_f32((uint16_t)h);
}

// The 16 bytes q as EPL consecutive elements.
template <int DT>
__device__ __forceinline__ void dense_unpack(const uint4 q, float* f) {
    if (DT == SSD_TYPE_F32) {
        f[0] = __uint_as_float(q.x);
        f[1] = __uint_as_float(q.y);
        f[2] = __uint_as_float(q.z);
        f[3] = __uint_as_float(q.w);
    } else {
        const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            f[2 * j] = DT == SSD_TYPE_BF16 ? __uint_as_float(u[j] << 16)
                                           : f16_bits_to_f32((uint16_t)(u[j] & 0xFFFFu));
            f[2 * j + 1] = DT == SSD_TYPE_BF16 ? __uint_as_float(u[j] & 0xFFFF0000u)
                                               : f16_bits_to_f32((uint16_t)(u[j] >> 16));
        }
    }
}

template <int DT, int EPI>
__global__ void __launch_bounds__(256) k_matvec_dense(const MvArgs a) {
    constexpr int ESZ = DT == SSD_TYPE_F32 ? 4 : 2;
    constexpr int EPL = 16 / ESZ;
    constexpr bool SW = EPI == EPI_SWIGLU;
    constexpr int OUT = SW ? kDenseRows / 2 : kDenseRows;  // outputs per group
    __shared__ float part[8][kDenseRows];
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n_out = SW ? a.seg_rows[0] : a.rows;
    const int r0 = (int)((int64_t)n_out * blockIdx.x / gridDim.x);
    const int r1 = (int)((int64_t)n_out * (blockIdx.x + 1) / gridDim.x);
    const bool vec = (a.cols % EPL) == 0;
    const char* wb0 = reinterpret_cast<const char*>(a.qs[0]);
    const char* wb1 = reinterpret_cast<const char*>(SW ? a.qs[1] : a.qs[0]);
    for (int g = r0; g < r1; g += OUT) {
        const int nr = r1 - g < OUT ? r1 - g : OUT;
        const char* w[kDenseRows];
#pragma unroll
        for (int i = 0; i < kDenseRows; i++) {  // rows past the range re-read the last one
            const int o = i / (SW ? 2 : 1);
            const int row = g + (o < nr ? o : nr - 1);
            w[i] = (SW && (i & 1) ? wb1 : wb0) + (size_t)row * a.cols * ESZ;
        }
        float s[kDenseRows];
#pragma unroll
        for (int i = 0; i < kDenseRows; i++) s[i] = 0.0f;
        if (vec) {
            for (int c = EPL * threadIdx.x; c < a.cols; c += 256 * EPL) {
                uint4 q[kDenseRows];
#pragma unroll
                for (int i = 0; i < kDenseRows; i++)
                    q[i] = __ldg(reinterpret_cast<const uint4*>(w[i] + (size_t)c * ESZ));
                float xv[EPL];
#pragma unroll
                for (int j = 0; j < EPL; j += 4) {
                    const float4 t = __ldg(reinterpret_cast<const float4*>(a.x + c + j));
                    xv[j] = t.x;
                    xv[j + 1] = t.y;
                    xv[j + 2] = t.z;
                    xv[j + 3] = t.w;
                }
#pragma unroll
                for (int i = 0; i < kDenseRows; i++) {
                    float f[EPL];
                    dense_unpack<DT>(q[i], f);
#pragma unroll
                    for (int j = 0; j < EPL; j++) s[i] = fmaf(f[j], xv[j], s[i]);
                }
            }
        } else {
            for (int c = threadIdx.x; c < a.cols; c += 256) {
                const float xv = a.x[c];
#pragma unroll
                for (int i = 0; i < kDenseRows; i++) s[i] = fmaf(dense_elem<DT>(w[i], c), xv, s[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < kDenseRows; i++) {
            const float v = warp_sum(s[i]);
            if (lane == 0) part[warp][i] = v;
        }
        __syncthreads();
        if (threadIdx.x < kDenseRows) {
            float t = part[0][threadIdx.x];
#pragma unroll
            for (int k = 1; k < 8; k++) t += part[k][threadIdx.x];
            part[0][threadIdx.x] = t;
        }
        __syncthreads();
        if (threadIdx.x < nr) {
            const int row = g + threadIdx.x;
            if (SW) {
                // silu(v) = v / (1 + exp(-v)), then gate *= up (feed_forward.rs:31-39)
                const float gt = part[0][2 * threadIdx.x], up = part[0][2 * threadIdx.x + 1];
                a.y[row] = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up);
            } else {
                const float t = part[0][threadIdx.x];
                a.y[row] = EPI == EPI_RESID ? __fadd_rn(a.base[row], t) : t;
            }
        }
        __syncthreads();
    }
}

template <int DT, int EPI>
static int launch_dense_epi(ssd_ctx* ctx, const MvArgs& a, cudaStream_t s, bool pdl) {
    static int per_sm = 0;  // resident CTAs per SM (same on every device of one build)
    if (per_sm == 0) {
        int n = 0;
        SSD_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_matvec_dense<DT, EPI>, 256, 0));
        per_sm = n > 0 ? n : 1;
    }
    const int full = ctx->num_sms * per_sm;
    const int n_out = EPI == EPI_SWIGLU ? a.seg_rows[0] : a.rows;
    const int grid = n_out < full ? n_out : full;
    SSD_CK(launch_pdl(k_matvec_dense<DT, EPI>, dim3(grid), dim3(256), 0, s, pdl, a));
    return SSD_OK;
}

template <int DT>
static int launch_dense(ssd_ctx* ctx, int epi, const MvArgs& a, cudaStream_t s, bool pdl) {
    switch (epi) {
        case EPI_RESID: return launch_dense_epi<DT, EPI_RESID>(ctx, a, s, pdl);
        case EPI_SWIGLU: return launch_dense_epi<DT, EPI_SWIGLU>(ctx, a, s, pdl);
        default: return launch_dense_epi<DT, EPI_STORE>(ctx, a, s, pdl);
    }
}

static bool is_dense(int type) {
    return type == SSD_TYPE_F16 || type == SSD_TYPE_BF16 || type == SSD_TYPE_F32;
}

int launch_matvec(ssd_ctx* ctx, int type, int epi, const MvArgs& a0, cudaStream_t s, bool pdl) {
    MvArgs a = a0;
    if (!a.status) a.status = ctx->dev_status;
    if (is_lowbit(type)) return launch_matvec_lowbit(ctx, type, epi, a, s, pdl);
    if (is_dense(type)) {
        SSD_REQ(a.rows > 0 && a.cols > 0, SSD_ERR_SHAPE, "empty matrix");
        SSD_REQ(a.x && a.y && ((uintptr_t)a.x & 15) == 0, SSD_ERR_ARG,
                "x and y must be non-null, x 16-byte aligned");
        SSD_REQ(((epi == EPI_STORE && a.map == MAP_PLAIN) ||
                 (epi == EPI_RESID && a.map == MAP_PLAIN && a.base) ||
                 (epi == EPI_SWIGLU && a.map == MAP_SWIGLU && a.qs[1] &&
                  a.rows == 2 * a.seg_rows[0])) &&
                    !a.x_add && !a.norm_w && a.ar_in_n == 0,
                SSD_ERR_ARG, "dense weights: plain, residual or un-normed SwiGLU matvec only");
        if (type == SSD_TYPE_F32) return launch_dense<SSD_TYPE_F32>(ctx, epi, a, s, pdl);
        return type == SSD_TYPE_BF16 ? launch_dense<SSD_TYPE_BF16>(ctx, epi, a, s, pdl)
                                     : launch_dense<SSD_TYPE_F16>(ctx, epi, a, s, pdl);
    }
    SSD_REQ(a.cols > 0 && a.cols % 32 == 0, SSD_ERR_SHAPE, "cols %d not a multiple of 32", a.cols);
    SSD_REQ(a.rows > 0, SSD_ERR_SHAPE, "no rows");
    // x, x_add, x_writeback and norm_w are read by TMA / written as float4
    SSD_REQ(a.x && al16(a.x) && al16(a.x_add) && al16(a.x_writeback) && al16(a.norm_w),
            SSD_ERR_ARG, "vector inputs must be non-null and 16-byte aligned");
    SSD_REQ(epi == EPI_ARGMAX ? a.argmax_key != nullptr
                              : (epi == EPI_PEERS ? a.ar_out_n > 0 : a.y != nullptr),
            SSD_ERR_ARG, "null output");
    SSD_REQ(a.ar_in_n >= 0 && a.ar_in_n <= kMaxPeers && a.ar_out_n >= 0 &&
                a.ar_out_n <= kMaxPeers,
            SSD_ERR_ARG, "peer count outside [0, %d]", kMaxPeers);
    SSD_REQ(a.ar_in_n == 0 || (a.ar_in && a.ar_in_flag && a.ar_epoch && al16(a.ar_in) &&
                               a.x_add == nullptr),
            SSD_ERR_ARG, "peer all-reduce input incomplete");
    SSD_REQ(epi != EPI_PEERS || (a.ar_counter && a.ar_epoch), SSD_ERR_ARG,
            "peer all-reduce output incomplete");
    if (epi == EPI_PEERS)
        for (int p = 0; p < a.ar_out_n; p++)
            SSD_REQ(a.ar_out[p] && a.ar_out_flag[p], SSD_ERR_ARG, "null peer buffer %d", p);
    SSD_REQ(a.map == epi_map(epi), SSD_ERR_ARG, "row map %d does not match epilogue %d", a.map,
            epi);
    SSD_REQ(epi != EPI_RESID || a.base != nullptr, SSD_ERR_ARG, "null residual base");
    SSD_REQ(epi != EPI_QKV_ROPE || (a.y_k && a.y_v), SSD_ERR_ARG, "null K/V output");
    SSD_REQ(epi != EPI_QKV_ROPE || (a.head_dim > 0 && a.head_dim / 2 <= kMaxRopePairs),
            SSD_ERR_SHAPE, "head_dim %d outside (0, %d]", a.head_dim, 2 * kMaxRopePairs);
    // Kernel choice: this FMA kernel (nibbles and scales unpacked in registers, dot products
    // on the fp32 pipe) for every shape. Two tensor-core kernels cover the common shapes
    // and are selected per call by SSD_MV_IMPL (read per call so that one process can
    // compare them): "i8" the tcgen05 kernel (matvec_i8.cu: Q4_0 / Q8_0 / Q4_K / Q5_K /
    // Q8_K, cols % 256 == 0, a weight with its split-K scratch), "tc" the mma.sync kernel
    // (matvec_tc.cu). Batch 1 keeps the FMA kernel: a tcgen05.mma of M = 128 issues at
    // most once per ~93 cycles, so the tcgen05 kernel tops out near the Q4_0 HBM rate
    // (~44 weights per cycle per SM against ~41 needed) before its fixed costs.
    SSD_REQ(!a.x_ready || (a.ar_in_n == 0 && epi != EPI_PEERS), SSD_ERR_ARG,
            "an independent launch takes no peer partials");
    const char* impl = getenv("SSD_MV_IMPL");
    if (impl && strcmp(impl, "tc") == 0 &&
        (type == SSD_TYPE_Q4_0 || type == SSD_TYPE_Q8_0 ||
         (type == SSD_TYPE_Q4_K && a.cols % 256 == 0))) {
        MvArgs t = a;
        t.x_ready = 0;  // the other kernels always wait first
        const int st = launch_matvec_tc(ctx, type, epi, t, s, pdl);
        if (st != kTcNotCovered) return st;
    }
    if (impl && strcmp(impl, "i8") == 0) {
        MvArgs t = a;
        t.x_ready = 0;
        const int st = launch_matvec_i8(ctx, type, epi, t, s, pdl);
        if (st != kI8NotCovered) return st;
    }
    switch (type) {
        case SSD_TYPE_Q4_0: return launch_fmt<SSD_TYPE_Q4_0>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q8_0: return launch_fmt<SSD_TYPE_Q8_0>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q4_K:
            SSD_REQ(a.cols % 256 == 0, SSD_ERR_SHAPE, "Q4_K cols %d not a multiple of 256", a.cols);
            return launch_fmt<SSD_TYPE_Q4_K>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q5_K:
            SSD_REQ(a.cols % 256 == 0, SSD_ERR_SHAPE, "Q5_K cols %d not a multiple of 256", a.cols);
            return launch_fmt<SSD_TYPE_Q5_K>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q6_K:
            SSD_REQ(a.cols % 256 == 0, SSD_ERR_SHAPE, "Q6_K cols %d not a multiple of 256", a.cols);
            return launch_fmt<SSD_TYPE_Q6_K>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q8_K:
            SSD_REQ(a.cols % 256 == 0, SSD_ERR_SHAPE, "Q8_K cols %d not a multiple of 256", a.cols);
            return launch_fmt<SSD_TYPE_Q8_K>(ctx, epi, a, s, pdl);
        default:
            set_error("matvec: ggml type %d not supported (Q4_0=2, Q8_0=8, Q4_K=12, Q5_K=13, "
                      "Q6_K=14, Q8_K=15)",
                      type);
            return SSD_ERR_TYPE;
    }
}

}  // namespace ssd

using namespace ssd;

static int check_w(const ssd_weight* w) {
    SSD_REQ(w != nullptr, SSD_ERR_ARG, "null weight");
    SSD_REQ(w->type == SSD_TYPE_Q4_0 || w->type == SSD_TYPE_Q8_0 || w->type == SSD_TYPE_Q4_K ||
                w->type == SSD_TYPE_Q5_K || w->type == SSD_TYPE_Q6_K || w->type == SSD_TYPE_Q8_K ||
                is_dense(w->type) || is_lowbit(w->type),
            SSD_ERR_TYPE, "matvec: ggml type %d not supported", w->type);
    return SSD_OK;
}

extern "C" int ssd_matvec(ssd_ctx* ctx, const ssd_weight* w, const float* x, float* y,
                          void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_TRY(check_w(w));
    SSD_REQ(x && y, SSD_ERR_ARG, "null vector");
    MvArgs a = mv_plain(w, x, y);
    return launch_matvec(ctx, w->type, EPI_STORE, a, pick_stream(ctx, stream), ctx->pdl);
}

extern "C" int ssd_matvec_independent(ssd_ctx* ctx, const ssd_weight* w, const float* x,
                                      float* y, void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_TRY(check_w(w));
    SSD_REQ(x && y, SSD_ERR_ARG, "null vector");
    MvArgs a = mv_plain(w, x, y);
    a.x_ready = 1;
    return launch_matvec(ctx, w->type, EPI_STORE, a, pick_stream(ctx, stream), true);
}

extern "C" int ssd_matvec_residual(ssd_ctx* ctx, const ssd_weight* w, const float* x,
                                   const float* base, float* y, void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_TRY(check_w(w));
    SSD_REQ(x && y && base, SSD_ERR_ARG, "null vector");
    MvArgs a = mv_plain(w, x, y);
    a.base = base;
    return launch_matvec(ctx, w->type, EPI_RESID, a, pick_stream(ctx, stream), ctx->pdl);
}

extern "C" int ssd_fused_rmsnorm_matvec(ssd_ctx* ctx, const ssd_weight* w, const float* x,
                                        const float* norm_w, float eps, float* y, void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_TRY(check_w(w));
    SSD_REQ(x && y && norm_w, SSD_ERR_ARG, "null vector");
    MvArgs a = mv_plain(w, x, y);
    a.norm_w = norm_w;
    a.eps = eps;
    a.norm_order = 1;  // x_norm[i] = x[i] * inv_rms * w[i]  (compute.rs:568-573)
    return launch_matvec(ctx, w->type, EPI_STORE, a, pick_stream(ctx, stream), ctx->pdl);
}

extern "C" int ssd_fused_qkv_rope(ssd_ctx* ctx, const ssd_weight* wq, const ssd_weight* wk,
                                  const ssd_weight* wv, const float* x, const float* norm_w,
                                  float eps, int head_dim, int position, float theta, float* q,
                                  float* k, float* v, void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_TRY(check_w(wq));
    SSD_TRY(check_w(wk));
    SSD_TRY(check_w(wv));
    SSD_REQ(x && q && k && v, SSD_ERR_ARG, "null vector");
    SSD_REQ(wq->type == wk->type && wk->type == wv->type, SSD_ERR_TYPE, "QKV types differ");
    SSD_REQ(wq->cols == wk->cols && wk->cols == wv->cols, SSD_ERR_SHAPE, "QKV widths differ");
    SSD_REQ(wk->rows == wv->rows, SSD_ERR_SHAPE, "K and V rows differ");
    SSD_REQ(head_dim > 0 && head_dim % 4 == 0 && wq->rows % head_dim == 0 &&
                wk->rows % head_dim == 0,
            SSD_ERR_SHAPE, "head_dim %d must divide the Q/K rows and be a multiple of 4", head_dim);
    MvArgs a = {};
    a.qs[0] = wq->qs;
    a.qs[1] = wk->qs;
    a.qs[2] = wv->qs;
    a.meta[0] = wq->meta;
    a.meta[1] = wk->meta;
    a.meta[2] = wv->meta;
    a.seg_rows[0] = wq->rows;
    a.seg_rows[1] = wk->rows;
    a.seg_rows[2] = wv->rows;
    a.map = MAP_QKV;
    a.fix_counter = wq->fix_counter;
    a.fix_partial = wq->fix_partial;
    a.rows = wq->rows + wk->rows + wv->rows;
    a.cols = wq->cols;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.norm_order = 0;  // rms_norm: x *= inv_rms * w  (compute.rs:586)
    a.y = q;
    a.y_k = k;
    a.y_v = v;
    a.head_dim = head_dim;
    a.theta = theta;
    a.position = position;
    return launch_matvec(ctx, wq->type, EPI_QKV_ROPE, a, pick_stream(ctx, stream), ctx->pdl);
}

extern "C" int ssd_fused_swiglu(ssd_ctx* ctx, const ssd_weight* wg, const ssd_weight* wu,
                                const float* x, const float* norm_w, float eps, float* act,
                                void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_TRY(check_w(wg));
    SSD_TRY(check_w(wu));
    SSD_REQ(x && act, SSD_ERR_ARG, "null vector");
    SSD_REQ(wg->type == wu->type && wg->rows == wu->rows && wg->cols == wu->cols, SSD_ERR_SHAPE,
            "gate/up shapes differ");
    SSD_REQ(wg->rows % 2 == 0, SSD_ERR_SHAPE, "n_ff must be even");
    MvArgs a = {};
    a.qs[0] = wg->qs;
    a.qs[1] = wu->qs;
    a.meta[0] = wg->meta;
    a.meta[1] = wu->meta;
    a.seg_rows[0] = wg->rows;
    a.seg_rows[1] = wu->rows;
    a.map = MAP_SWIGLU;
    a.fix_counter = wg->fix_counter;
    a.fix_partial = wg->fix_partial;
    a.rows = 2 * wg->rows;
    a.cols = wg->cols;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.norm_order = 1;  // ffn input from fused_post_attn_norm: h * inv_rms * w
    a.y = act;
    return launch_matvec(ctx, wg->type, EPI_SWIGLU, a, pick_stream(ctx, stream), ctx->pdl);
}

extern "C" int ssd_matvec_peer_input(ssd_ctx* ctx, const ssd_weight* w, const float* x,
                                     const float* partials, int n_ranks,
                                     const unsigned long long* flags,
                                     const unsigned long long* epoch, int call, float* y,
                                     void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_TRY(check_w(w));
    SSD_REQ(x && y && partials && flags && epoch, SSD_ERR_ARG, "null argument");
    SSD_REQ(n_ranks >= 1 && n_ranks <= kMaxPeers, SSD_ERR_ARG, "n_ranks %d outside [1, %d]",
            n_ranks, kMaxPeers);
    SSD_REQ(!is_dense(w->type) && !is_lowbit(w->type), SSD_ERR_TYPE,
            "peer input: Q4_0 / Q8_0 / Q4_K / Q5_K / Q6_K / Q8_K weights only");
    MvArgs a = mv_plain(w, x, y);
    a.ar_in = partials;
    a.ar_in_flag = flags;
    a.ar_in_n = n_ranks;
    a.ar_epoch = epoch;
    a.ar_call = call;
    return launch_matvec(ctx, w->type, EPI_STORE, a, pick_stream(ctx, stream), ctx->pdl);
}

extern "C" int ssd_matvec_quantized_host(ssd_ctx* ctx, const uint8_t* w_raw, size_t w_bytes,
                                         const float* x, float* y, int out_dim, int in_dim,
                                         int type) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(w_raw && x && y, SSD_ERR_ARG, "null pointer");
    SSD_REQ(type == SSD_TYPE_Q4_0 || type == SSD_TYPE_Q8_0 || type == SSD_TYPE_Q4_K ||
                type == SSD_TYPE_Q5_K || type == SSD_TYPE_Q6_K || type == SSD_TYPE_Q8_K ||
                type == SSD_TYPE_F16 || type == SSD_TYPE_BF16 || is_lowbit(type),
            SSD_ERR_TYPE, "matvec_quantized: ggml type %d not supported", type);
    ssd_weight* w = nullptr;
    SSD_TRY(ssd_weight_upload(ctx, w_raw, w_bytes, type, out_dim, in_dim, &w));
    size_t xb = (size_t)in_dim * 4, yb = (size_t)out_dim * 4;
    int st = ensure_scratch(ctx, xb + yb + 512);
    if (st == SSD_OK) {
        float* xd = (float*)ctx->scratch;
        float* yd = (float*)((char*)ctx->scratch + ((xb + 255) & ~(size_t)255));
        cudaMemcpyAsync(xd, x, xb, cudaMemcpyHostToDevice, ctx->stream);
        st = ssd_matvec(ctx, w, xd, yd, (void*)ctx->stream);
        if (st == SSD_OK) {
            cudaMemcpyAsync(y, yd, yb, cudaMemcpyDeviceToHost, ctx->stream);
            if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
                set_error("matvec_quantized_host: %s", cudaGetErrorString(cudaGetLastError()));
                st = SSD_ERR_CUDA;
            }
        }
    }
    ssd_weight_free(w);
    return st;
}
