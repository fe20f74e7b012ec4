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
//  * Weight loads for the first steps are issued before griddepcontrol.wait: they do
//    not depend on the previous kernel, so under programmatic dependent launch they
//    overlap its tail. Loads are double-buffered in registers across chunk steps.
//  * The kernel is persistent: x is staged once per CTA by TMA into shared memory with
//    the 128-byte swizzle (chunk c's 16-byte unit u at unit u ^ (c & 7)), so the 8
//    float4 reads of a chunk are bank-conflict free across a quarter warp; the
//    residual add and RMSNorm are applied there.
//  * Quantized values become floats without int->float conversion instructions:
//    byte_perm places a byte under exponent byte 0x4B, giving 2^23 + b exactly, and one
//    FADD removes the offset: q - 8 for Q4_0, q for Q4_K, (q+128) - 128 for Q8_0. The
//    values are exact, so each chunk dot product carries only fp32 FMA rounding.
//  * Epilogues fuse what follows the matvec in the decode step: residual add,
//    SwiGLU, RoPE on Q/K, or argmax (LAST index on ties, sampler.rs:572-578).
#include <mutex>

#include "matvec.cuh"

namespace ssd {

constexpr float kQ80Magic = 8388736.0f;  // 2^23 + 128

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

struct RowPtr {
    const uint8_t* qs;
    const uint8_t* meta;
};

__device__ __forceinline__ void map_row(const MvArgs& a, int v, int& seg, int& lr) {
    if (a.map == MAP_PLAIN) {
        seg = 0;
        lr = v;
    } else if (a.map == MAP_QKV) {
        if (v < a.seg_rows[0]) {
            seg = 0;
            lr = v;
        } else if (v < a.seg_rows[0] + a.seg_rows[1]) {
            seg = 1;
            lr = v - a.seg_rows[0];
        } else {
            seg = 2;
            lr = v - a.seg_rows[0] - a.seg_rows[1];
        }
    } else {  // MAP_SWIGLU: virtual rows 4g..4g+3 = gate 2g, gate 2g+1, up 2g, up 2g+1
        int g = v >> 2, j = v & 3;
        seg = j >> 1;
        lr = 2 * g + (j & 1);
    }
}

template <int FMT>
__device__ __forceinline__ RowPtr row_ptr(const MvArgs& a, int v) {
    int seg, lr;
    map_row(a, v, seg, lr);
    const size_t nc = (size_t)(a.cols >> 5);
    RowPtr p;
    const uint8_t* qs = seg == 0 ? a.qs[0] : (seg == 1 ? a.qs[1] : a.qs[2]);
    const uint8_t* mt = seg == 0 ? a.meta[0] : (seg == 1 ? a.meta[1] : a.meta[2]);
    if constexpr (FMT == SSD_TYPE_Q4_0) {
        p.qs = qs + (size_t)lr * nc * 16;
        p.meta = mt + (size_t)lr * nc * 2;
    } else if constexpr (FMT == SSD_TYPE_Q8_0) {
        p.qs = qs + (size_t)lr * nc * 32;
        p.meta = mt + (size_t)lr * nc * 2;
    } else {
        p.qs = qs + (size_t)lr * nc * 16;
        p.meta = mt + (size_t)lr * (nc >> 3) * 16;
    }
    return p;
}

template <int FMT>
__device__ __forceinline__ void load_chunk(Chunk<FMT>& ch, const RowPtr& p, int c, bool valid) {
    if constexpr (FMT == SSD_TYPE_Q4_0) {
        auto& k = ch;
        if (valid) {
            k.q = ldg_stream(p.qs + (size_t)c * 16);
            k.d = ldg_u16(p.meta + (size_t)c * 2);
        } else {
            k.q = make_uint4(0, 0, 0, 0);
            k.d = 0;
        }
    } else if constexpr (FMT == SSD_TYPE_Q8_0) {
        auto& k = ch;
        if (valid) {
            k.q0 = ldg_stream(p.qs + (size_t)c * 32);
            k.q1 = ldg_stream(p.qs + (size_t)c * 32 + 16);
            k.d = ldg_u16(p.meta + (size_t)c * 2);
        } else {
            k.q0 = k.q1 = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
            k.d = 0;
        }
    } else {
        auto& k = ch;
        if (valid) {
            k.q = ldg_stream(p.qs + (size_t)c * 16);
            k.m = __ldg(reinterpret_cast<const uint4*>(p.meta) + (c >> 3));
        } else {
            k.q = make_uint4(0, 0, 0, 0);
            k.m = make_uint4(0, 0, 0, 0);
        }
    }
}

__device__ __forceinline__ uint32_t word_of(const uint4& q, int m) {
    return m == 0 ? q.x : (m == 1 ? q.y : (m == 2 ? q.z : q.w));
}

// s += sum over the chunk of (q - OFF) * x for a 16-byte nibble chunk (element 2j is
// the low nibble of byte j, 2j+1 the high nibble: src/metal/compute.rs:693-699).
// OFF = 8 for Q4_0 (q - 8, compute.rs:696-697), 0 for Q4_K (q, compute.rs:739-740).
template <int R, int OFF>
__device__ __forceinline__ void nib_dot(const float4* xc, int c, const uint4 (&q)[R],
                                        float (&s)[R]) {
    constexpr float kMagic = 8388608.0f + (float)OFF;  // 2^23 + OFF
#pragma unroll
    for (int m = 0; m < 4; m++) {
        const float4 xa = xc[(2 * m) ^ (c & 7)];
        const float4 xb = xc[(2 * m + 1) ^ (c & 7)];
#pragma unroll
        for (int r = 0; r < R; r++) {
            const uint32_t w = word_of(q[r], m);
            const uint32_t lo = w & 0x0F0F0F0Fu;
            const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;
            float t = s[r];
            t = fmaf(magic_byte(lo, 0) - kMagic, xa.x, t);
            t = fmaf(magic_byte(hi, 0) - kMagic, xa.y, t);
            t = fmaf(magic_byte(lo, 1) - kMagic, xa.z, t);
            t = fmaf(magic_byte(hi, 1) - kMagic, xa.w, t);
            t = fmaf(magic_byte(lo, 2) - kMagic, xb.x, t);
            t = fmaf(magic_byte(hi, 2) - kMagic, xb.y, t);
            t = fmaf(magic_byte(lo, 3) - kMagic, xb.z, t);
            t = fmaf(magic_byte(hi, 3) - kMagic, xb.w, t);
            s[r] = t;
        }
    }
}

template <int FMT, int R>
__device__ __forceinline__ void compute_chunk(const Chunk<FMT> (&ch)[R], const float4* xs4,
                                              const float* csum, int c, int lane,
                                              float (&acc)[R]) {
    const float4* xc = xs4 + (size_t)c * 8;
    if constexpr (FMT == SSD_TYPE_Q4_0) {
        uint4 q[R];
        float s[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            q[r] = ch[r].q;
            s[r] = 0.0f;
        }
        nib_dot<R, 8>(xc, c, q, s);
#pragma unroll
        for (int r = 0; r < R; r++) {
            const float d = f16_bits_to_f32((uint16_t)ch[r].d);
            acc[r] = fmaf(d, s[r], acc[r]);
        }
    } else if constexpr (FMT == SSD_TYPE_Q8_0) {
        float s[R];
#pragma unroll
        for (int r = 0; r < R; r++) s[r] = 0.0f;
#pragma unroll
        for (int m = 0; m < 8; m++) {
            const float4 xa = xc[m ^ (c & 7)];
#pragma unroll
            for (int r = 0; r < R; r++) {
                const auto& k = ch[r];
                const uint32_t b = word_of(m < 4 ? k.q0 : k.q1, m & 3) ^ 0x80808080u;
                float t = s[r];
                t = fmaf(magic_byte(b, 0) - kQ80Magic, xa.x, t);
                t = fmaf(magic_byte(b, 1) - kQ80Magic, xa.y, t);
                t = fmaf(magic_byte(b, 2) - kQ80Magic, xa.z, t);
                t = fmaf(magic_byte(b, 3) - kQ80Magic, xa.w, t);
                s[r] = t;
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++) {
            const float d = f16_bits_to_f32((uint16_t)ch[r].d);
            acc[r] = fmaf(d, s[r], acc[r]);
        }
    } else {  // Q4_K: this lane's sub-block index is c & 7 == lane & 7
        uint4 q[R];
        float s[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            q[r] = ch[r].q;
            s[r] = 0.0f;
        }
        nib_dot<R, 0>(xc, c, q, s);
        const float X = csum[c];  // sum of the chunk's x
        const int sb = lane & 7, sh = 8 * (sb & 3);
#pragma unroll
        for (int r = 0; r < R; r++) {
            const uint4 m = ch[r].m;
            const float d = f16_bits_to_f32((uint16_t)(m.x & 0xFFFF));
            const float dmin = f16_bits_to_f32((uint16_t)(m.x >> 16));
            const uint32_t b0 = (m.y >> sh) & 0xFF, b4 = (m.z >> sh) & 0xFF,
                           b8 = (m.w >> sh) & 0xFF;
            uint32_t s6, m6;  // src/metal/compute.rs:725-733
            if (sb < 4) {
                s6 = b0 & 0x3F;
                m6 = b4 & 0x3F;
            } else {
                s6 = (b0 >> 6) | ((b8 & 0x0F) << 2);
                m6 = (b4 >> 6) | ((b8 >> 4) << 2);
            }
            // sum((scale*q - min) x) = scale * sum(q x) - min * X
            const float scale = __fmul_rn(d, (float)s6);
            const float mn = __fmul_rn(dmin, (float)m6);
            acc[r] = fmaf(-mn, X, fmaf(scale, s[r], acc[r]));
        }
    }
}

// RoPE of one adjacent pair (src/metal/compute.rs:494-503). The angle's powf /
// sin / cos are evaluated in double and rounded once to float.
__device__ __forceinline__ void rope_pair(float& x0, float& x1, int lr, int head_dim, float theta,
                                          int pos) {
    const int i = (lr % head_dim) >> 1;
    const float e = __fdiv_rn(__fmul_rn(2.0f, (float)i), (float)head_dim);
    const float p = (float)pow((double)theta, (double)e);
    const float freq = __fdiv_rn(1.0f, p);
    const float ang = __fmul_rn((float)pos, freq);
    double sd, cd;
    sincos((double)ang, &sd, &cd);
    const float sn = (float)sd, cs = (float)cd;
    const float a0 = x0, a1 = x1;
    x0 = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(a1, sn));
    x1 = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(a1, cs));
}

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | idx;
}

// Shared-memory plan of one CTA (offsets from a 1024-byte aligned base).
struct SmemPlan {
    int nc, xrows;              // chunks, staged rows (multiple of kVecBoxRows)
    size_t xs, xa, xn, csum, red, bar, total;
};
__host__ __device__ inline SmemPlan smem_plan(int cols, bool add, bool norm, bool sums, int nw) {
    SmemPlan p;
    p.nc = cols >> 5;
    p.xrows = (p.nc + kVecBoxRows - 1) / kVecBoxRows * kVecBoxRows;
    const size_t vb = (size_t)p.xrows * 128;
    size_t o = 0;
    p.xs = o;
    o += vb;
    p.xa = add ? o : 0;
    o += add ? vb : 0;
    p.xn = norm ? o : 0;
    o += norm ? vb : 0;
    p.csum = o;
    o += sums ? ((size_t)p.nc * 4 + 15) & ~(size_t)15 : 0;
    p.red = o;
    o += 64 * 4 + (size_t)nw * 8;
    p.bar = o;
    o += 16;
    p.total = o + 1024;  // alignment slack
    return p;
}

// Persistent fused dequant-matvec. Grid = resident CTAs (or fewer for small matrices);
// warp w of the grid owns row-groups (R rows) w, w + W, w + 2W, ... (W = warps in the
// grid). Weight loads run two register stages ahead across row-group boundaries; the
// first stage is issued before griddepcontrol.wait. x (and x_add / norm_w) arrive by
// TMA into 128B-swizzled shared memory; the residual add and RMSNorm are applied there.
template <int FMT, int EPI, int R, int U, int NW>
__global__ void __launch_bounds__(NW * 32, (NW == 8 ? 2 : 4))
    k_matvec(const MvArgs a, const __grid_constant__ CUtensorMap tm_x,
             const __grid_constant__ CUtensorMap tm_add, const __grid_constant__ CUtensorMap tm_norm) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const bool has_add = a.x_add != nullptr, has_norm = a.norm_w != nullptr;
    const SmemPlan P = smem_plan(a.cols, has_add, has_norm, FMT == SSD_TYPE_Q4_K, NW);
    float4* xs4 = reinterpret_cast<float4*>(base + P.xs);
    float* csum = reinterpret_cast<float*>(base + P.csum);
    float* red = reinterpret_cast<float*>(base + P.red);
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(base + P.red + 256);
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + P.bar);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nc = P.nc;
    const int iters = (nc + 31) >> 5;               // chunk iterations per lane per row
    const int spr = (iters + U - 1) / U;            // register steps per row-group
    const int n_rg = (a.rows + R - 1) / R;
    const int W = gridDim.x * NW;
    const int wg = blockIdx.x * NW + warp;
    const int my_rg = wg < n_rg ? (n_rg - 1 - wg) / W + 1 : 0;
    const int total = my_rg * spr;

    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }

    Chunk<FMT> A[U][R], B[U][R];
    auto load_step = [&](Chunk<FMT>(&buf)[U][R], int s) {
        const int rg = wg + (s / spr) * W, st = s % spr;
        const int v0 = rg * R;
#pragma unroll
        for (int r = 0; r < R; r++) {
            const bool rv = v0 + r < a.rows;
            const RowPtr rp = rv ? row_ptr<FMT>(a, v0 + r) : RowPtr{nullptr, nullptr};
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int c = lane + 32 * (st * U + u);
                load_chunk<FMT>(buf[u][r], rp, c, rv && c < nc);
            }
        }
    };
    // Weights never depend on the previous kernel: issue the first stage before waiting.
    if (total > 0) load_step(A, 0);
    __syncthreads();  // barrier initialised
    pdl_wait();

    if (tid == 0) {
        const int nbox = P.xrows / kVecBoxRows;
        const uint32_t vbytes = (uint32_t)P.xrows * 128u;
        mbar_expect_tx(bar, vbytes * (1u + (has_add ? 1u : 0u) + (has_norm ? 1u : 0u)));
        for (int b = 0; b < nbox; b++) {
            tma_load_2d(base + P.xs + (size_t)b * kVecBoxRows * 128, &tm_x, 0, b * kVecBoxRows, bar);
            if (has_add)
                tma_load_2d(base + P.xa + (size_t)b * kVecBoxRows * 128, &tm_add, 0,
                            b * kVecBoxRows, bar);
            if (has_norm)
                tma_load_2d(base + P.xn + (size_t)b * kVecBoxRows * 128, &tm_norm, 0,
                            b * kVecBoxRows, bar);
        }
    }
    const bool ok = mbar_wait(bar, 0, a.status);
    if (__syncthreads_or(!ok)) return;  // timed out: status recorded, nothing computed

    // prologue in shared memory: x_eff = x (+ x_add); optional RMSNorm; chunk sums
    const int nunits = nc * 8;  // 16-byte units
    const unsigned gmask = 0xFFu << (lane & 24);
    if (has_add || has_norm) {
        const float4* xa4 = reinterpret_cast<const float4*>(base + P.xa);
        const float4* xn4 = reinterpret_cast<const float4*>(base + P.xn);
        const bool wb = a.x_writeback != nullptr && blockIdx.x == 0;
        float ss = 0.0f;
        for (int i = tid; i < nunits; i += NW * 32) {
            const int c = i >> 3, ph = c * 8 + ((i & 7) ^ (c & 7));
            float4 v = xs4[ph];
            if (has_add) {  // hidden[i] += attn_output[i] (src/metal/compute.rs:547-549)
                const float4 r = xa4[ph];
                v.x = __fadd_rn(v.x, r.x);
                v.y = __fadd_rn(v.y, r.y);
                v.z = __fadd_rn(v.z, r.z);
                v.w = __fadd_rn(v.w, r.w);
                xs4[ph] = v;
                if (wb) reinterpret_cast<float4*>(a.x_writeback)[i] = v;
            }
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
        if (has_norm) {
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; w++) tot += red[w];
            // inv_rms = 1 / sqrt(sum_sq / n + eps)   (src/metal/compute.rs:583-584)
            const float inv =
                __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.cols), a.eps)));
            for (int i = tid; i < nunits; i += NW * 32) {
                const int c = i >> 3, ph = c * 8 + ((i & 7) ^ (c & 7));
                float4 v = xs4[ph];
                const float4 w = xn4[ph];
                if (a.norm_order == 0) {  // x * (inv_rms * w)
                    v.x = __fmul_rn(v.x, __fmul_rn(inv, w.x));
                    v.y = __fmul_rn(v.y, __fmul_rn(inv, w.y));
                    v.z = __fmul_rn(v.z, __fmul_rn(inv, w.z));
                    v.w = __fmul_rn(v.w, __fmul_rn(inv, w.w));
                } else {  // (x * inv_rms) * w
                    v.x = __fmul_rn(__fmul_rn(v.x, inv), w.x);
                    v.y = __fmul_rn(__fmul_rn(v.y, inv), w.y);
                    v.z = __fmul_rn(__fmul_rn(v.z, inv), w.z);
                    v.w = __fmul_rn(__fmul_rn(v.w, inv), w.w);
                }
                xs4[ph] = v;
            }
        }
    }
    if constexpr (FMT == SSD_TYPE_Q4_K) {  // chunk sums of x for the min term
        for (int i = tid; i < nunits; i += NW * 32) {
            const int c = i >> 3, ph = c * 8 + ((i & 7) ^ (c & 7));
            const float4 v = xs4[ph];
            float t = (v.x + v.y) + (v.z + v.w);
            t += __shfl_xor_sync(gmask, t, 1);
            t += __shfl_xor_sync(gmask, t, 2);
            t += __shfl_xor_sync(gmask, t, 4);
            if ((i & 7) == 0) csum[c] = t;
        }
    }
    __syncthreads();
    pdl_trigger();

    float acc[R];
#pragma unroll
    for (int r = 0; r < R; r++) acc[r] = 0.0f;
    unsigned long long best = 0ull;

    auto compute_step = [&](const Chunk<FMT>(&buf)[U][R], int s) {
        const int st = s % spr;
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = lane + 32 * (st * U + u);
            if (c < nc) compute_chunk<FMT, R>(buf[u], xs4, csum, c, lane, acc);
        }
        if (st != spr - 1) return;
        // row-group finished: reduce across the warp and run the epilogue
        const int v0 = (wg + (s / spr) * W) * R;
        float res[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            res[r] = warp_sum(acc[r]);
            acc[r] = 0.0f;
        }
        if constexpr (EPI == EPI_STORE || EPI == EPI_RESID) {
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int row = v0 + r;
                if (lane == r && row < a.rows)
                    a.y[row] = (EPI == EPI_RESID) ? __fadd_rn(a.base[row], res[r]) : res[r];
            }
        } else if constexpr (EPI == EPI_SWIGLU) {  // rows (gate 2g, gate 2g+1, up 2g, up 2g+1)
            if (lane < 2 && v0 < a.rows) {
                const float g = lane == 0 ? res[0] : res[1];
                const float up = lane == 0 ? res[2] : res[3];
                // silu(v) = v / (1 + exp(-v)), then gate *= up (feed_forward.rs:31-39,
                // compute.rs:641-645)
                const float si = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
                a.y[(v0 >> 1) + lane] = __fmul_rn(si, up);
            }
        } else if constexpr (EPI == EPI_QKV_ROPE) {  // adjacent pairs (v0+2p, v0+2p+1)
            if (lane < R / 2 && v0 < a.rows) {
                const int pos = a.position_dev ? *a.position_dev : a.position;
                int seg, lr;
                map_row(a, v0 + 2 * lane, seg, lr);
                float x0 = lane == 0 ? res[0] : res[2];
                float x1 = lane == 0 ? res[1] : res[3];
                if (seg < 2) rope_pair(x0, x1, lr, a.head_dim, a.theta, pos);
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
                    const unsigned long long k = argmax_key(res[r], (uint32_t)(row + a.index_offset));
                    best = k > best ? k : best;
                }
            }
        }
    };

    for (int s = 0; s < total; s += 2) {
        if (s + 1 < total) load_step(B, s + 1);
        compute_step(A, s);
        if (s + 2 < total) load_step(A, s + 2);
        if (s + 1 < total) compute_step(B, s + 1);
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
}

// --------------------------------------------------------------- host side

struct Cfg {
    int R, U, NW;
};

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

// Resident CTAs per SM of one kernel at a given dynamic shared-memory size, cached
// per (kernel, device, size); sets the shared-memory opt-in attribute on first use.
template <typename K>
static int occupancy(ssd_ctx* ctx, K kern, int threads, size_t smem, int* out) {
    struct Entry {
        const void* fn;
        int dev;
        size_t smem;
        int blocks;
    };
    static Entry cache[256];
    static int n = 0;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    const void* fn = reinterpret_cast<const void*>(kern);
    bool attr_set = false;
    for (int i = 0; i < n; i++) {
        if (cache[i].fn != fn || cache[i].dev != ctx->device) continue;
        attr_set = true;
        if (cache[i].smem == smem) {
            *out = cache[i].blocks;
            return SSD_OK;
        }
    }
    if (!attr_set)
        SSD_CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)ctx->smem_optin));
    int nb = 0;
    SSD_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, threads, smem));
    SSD_REQ(nb > 0, SSD_ERR_SHAPE, "matvec kernel does not fit on an SM (%zu B smem)", smem);
    if (n < 256) cache[n++] = Entry{fn, ctx->device, smem, nb};
    *out = nb;
    return SSD_OK;
}

template <int FMT, int EPI, int R, int U, int NW>
static int launch_t(ssd_ctx* ctx, const MvArgs& a, cudaStream_t s, bool pdl) {
    auto kern = k_matvec<FMT, EPI, R, U, NW>;
    const SmemPlan P =
        smem_plan(a.cols, a.x_add != nullptr, a.norm_w != nullptr, FMT == SSD_TYPE_Q4_K, NW);
    SSD_REQ(P.total <= ctx->smem_optin, SSD_ERR_SHAPE,
            "cols %d too large for shared-memory staging (%zu bytes)", a.cols, P.total);
    int nb = 0;
    SSD_TRY(occupancy(ctx, kern, NW * 32, P.total, &nb));
    const int n_rg = (a.rows + R - 1) / R;
    const int need = (n_rg + NW - 1) / NW;
    const int grid = need < ctx->num_sms * nb ? need : ctx->num_sms * nb;
    CUtensorMap mx, madd, mnorm;
    SSD_TRY(encode_vec_map(&mx, a.x, a.cols));
    madd = mx;
    mnorm = mx;
    if (a.x_add) SSD_TRY(encode_vec_map(&madd, a.x_add, a.cols));
    if (a.norm_w) SSD_TRY(encode_vec_map(&mnorm, a.norm_w, a.cols));
    SSD_CK(launch_pdl(kern, dim3(grid), dim3(NW * 32), P.total, s, pdl, a, mx, madd, mnorm));
    return SSD_OK;
}

// Active warps per SM the launch would get with NW warps per CTA.
template <int FMT, int EPI, int R, int U, int NW>
static int active_warps(ssd_ctx* ctx, const MvArgs& a, int* warps) {
    const SmemPlan P =
        smem_plan(a.cols, a.x_add != nullptr, a.norm_w != nullptr, FMT == SSD_TYPE_Q4_K, NW);
    *warps = 0;
    if (P.total > ctx->smem_optin) return SSD_OK;
    int nb = 0;
    SSD_TRY(occupancy(ctx, k_matvec<FMT, EPI, R, U, NW>, NW * 32, P.total, &nb));
    const int n_rg = (a.rows + R - 1) / R;
    const int ctas = (n_rg + NW - 1) / NW;
    const int resident = ctx->num_sms * nb;
    const long long w = (long long)(ctas < resident ? ctas : resident) * NW;
    *warps = (int)(w / ctx->num_sms);
    return SSD_OK;
}

// Tiling: R = 4 rows per warp; 4 or 8 warps per CTA, whichever keeps more warps
// resident per SM for this width and prologue (ties go to 8: fewer x stagings).
// Q4_0 keeps two chunk steps per register stage (128 registers, no spill), Q8_0 / Q4_K
// one. SSD_MV_CONFIG="R,U,NW" selects another instantiation of the plain matvec.
template <int FMT, int EPI>
static int launch_fmt_epi(ssd_ctx* ctx, const MvArgs& a, cudaStream_t s, bool pdl) {
    if constexpr (EPI == EPI_STORE) {
        const Cfg c = env_cfg();
        if (c.R == 4 && c.U == 1 && c.NW == 4) return launch_t<FMT, EPI, 4, 1, 4>(ctx, a, s, pdl);
        if (c.R == 4 && c.U == 1 && c.NW == 8) return launch_t<FMT, EPI, 4, 1, 8>(ctx, a, s, pdl);
        if (c.R == 2 && c.U == 2 && c.NW == 4) return launch_t<FMT, EPI, 2, 2, 4>(ctx, a, s, pdl);
    }
    constexpr int U = FMT == SSD_TYPE_Q4_0 ? 2 : 1;
    int w4 = 0, w8 = 0;
    SSD_TRY((active_warps<FMT, EPI, 4, U, 4>(ctx, a, &w4)));
    SSD_TRY((active_warps<FMT, EPI, 4, U, 8>(ctx, a, &w8)));
    if (w8 >= w4 && w8 > 0) return launch_t<FMT, EPI, 4, U, 8>(ctx, a, s, pdl);
    return launch_t<FMT, EPI, 4, U, 4>(ctx, a, s, pdl);
}

template <int FMT>
static int launch_fmt(ssd_ctx* ctx, int epi, const MvArgs& a, cudaStream_t s, bool pdl) {
    switch (epi) {
        case EPI_STORE: return launch_fmt_epi<FMT, EPI_STORE>(ctx, a, s, pdl);
        case EPI_RESID: return launch_fmt_epi<FMT, EPI_RESID>(ctx, a, s, pdl);
        case EPI_SWIGLU: return launch_fmt_epi<FMT, EPI_SWIGLU>(ctx, a, s, pdl);
        case EPI_QKV_ROPE: return launch_fmt_epi<FMT, EPI_QKV_ROPE>(ctx, a, s, pdl);
        case EPI_ARGMAX: return launch_fmt_epi<FMT, EPI_ARGMAX>(ctx, a, s, pdl);
        default: set_error("bad epilogue %d", epi); return SSD_ERR_ARG;
    }
}

static inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

int launch_matvec(ssd_ctx* ctx, int type, int epi, const MvArgs& a0, cudaStream_t s, bool pdl) {
    MvArgs a = a0;
    if (!a.status) a.status = ctx->dev_status;
    SSD_REQ(a.cols > 0 && a.cols % 32 == 0, SSD_ERR_SHAPE, "cols %d not a multiple of 32", a.cols);
    SSD_REQ(a.rows > 0, SSD_ERR_SHAPE, "no rows");
    // x, x_add, x_writeback and norm_w are read by TMA / written as float4
    SSD_REQ(a.x && al16(a.x) && al16(a.x_add) && al16(a.x_writeback) && al16(a.norm_w),
            SSD_ERR_ARG, "vector inputs must be non-null and 16-byte aligned");
    SSD_REQ(epi == EPI_ARGMAX ? a.argmax_key != nullptr : a.y != nullptr, SSD_ERR_ARG,
            "null output");
    SSD_REQ(epi != EPI_RESID || a.base != nullptr, SSD_ERR_ARG, "null residual base");
    SSD_REQ(epi != EPI_QKV_ROPE || (a.y_k && a.y_v), SSD_ERR_ARG, "null K/V output");
    switch (type) {
        case SSD_TYPE_Q4_0: return launch_fmt<SSD_TYPE_Q4_0>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q8_0: return launch_fmt<SSD_TYPE_Q8_0>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q4_K:
            SSD_REQ(a.cols % 256 == 0, SSD_ERR_SHAPE, "Q4_K cols %d not a multiple of 256", a.cols);
            return launch_fmt<SSD_TYPE_Q4_K>(ctx, epi, a, s, pdl);
        default:
            set_error("matvec: ggml type %d not supported (Q4_0=2, Q8_0=8, Q4_K=12)", type);
            return SSD_ERR_TYPE;
    }
}

}  // namespace ssd

using namespace ssd;

static int check_w(const ssd_weight* w) {
    SSD_REQ(w != nullptr, SSD_ERR_ARG, "null weight");
    SSD_REQ(w->type == SSD_TYPE_Q4_0 || w->type == SSD_TYPE_Q8_0 || w->type == SSD_TYPE_Q4_K,
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
    a.rows = 2 * wg->rows;
    a.cols = wg->cols;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.norm_order = 1;  // ffn input from fused_post_attn_norm: h * inv_rms * w
    a.y = act;
    return launch_matvec(ctx, wg->type, EPI_SWIGLU, a, pick_stream(ctx, stream), ctx->pdl);
}

extern "C" int ssd_matvec_quantized_host(ssd_ctx* ctx, const uint8_t* w_raw, size_t w_bytes,
                                         const float* x, float* y, int out_dim, int in_dim,
                                         int type) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(w_raw && x && y, SSD_ERR_ARG, "null pointer");
    SSD_REQ(type == SSD_TYPE_Q4_0 || type == SSD_TYPE_Q8_0 || type == SSD_TYPE_Q4_K, SSD_ERR_TYPE,
            "matvec_quantized: ggml type %d not supported", type);
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
