// matvec_b.cu — batched dequant-matvec for continuous-batch decode: Y[t] = W X[t] for
// NB = 16 token vectors at once, on the tcgen05 integer tensor cores (sm_100a).
//
// The batch step of BatchScheduler::step (src/inference/batch_scheduler.rs:236-296) runs
// every decoding request through each layer in turn; the weights it streams are the same
// for all of them. Here the 16 requests' vectors share one weight stream: each 32-weight
// block (the rows of Q4_0 / Q8_0 / Q4_K, src/metal/compute.rs:680-750, :904-925) is read
// from HBM once and multiplied against all 16 vectors by one tcgen05.mma of N = 64.
//
// Arithmetic (as matvec_i8.cu, per token): A = the block's weights as signed bytes (Q4_0 /
// Q4_K nibbles unpacked to 16 (q - 8)); B = the tokens' x as exact fixed point per
// 32-element block, xf = rint(x 2^e), split into four signed byte limbs. Column 16 l + t of
// B is limb l of token t, so one MMA gives the 64 exact int32 limb sums of a block; the
// readout combines each token's four limbs, rounds once to fp32 and adds d * 2^-e * sum.
// The exponent e of a block is shared by the 16 tokens (max |x| over the tokens' 32
// elements in [2^25, 2^26)), so the scale d * 2^-e is one product per (row, block).
//
// Two kernels per matvec:
//  * k_bprep (one CTA per 256 columns): x_eff = x (+ x_add, written back), optional RMSNorm
//    per token (order 0 / 1 as the single-vector kernels), then the limbs of its 8 blocks in
//    the exact shared-memory layout of the B operand ([block][K half][64 rows][16 B]) and
//    the blocks' scales and sums, into global buffers that stay in L2;
//  * k_mv_b: one CTA per SM over units of 128 rows x 256 columns (tile-major ranges, the
//    split tiles finished by the last CTA to arrive, adding partial rows in CTA order).
//    Each unit's stage brings by TMA the packed weights, their scales and the unit's B block
//    (16 KB) with its scale table; warps 18-21 unpack nibbles, warp 17 issues the MMAs,
//    warps 0-15 read TMEM back (warp group g = warps 4g..4g+3: tokens 4g..4g+3, lanes = rows).
// Every mbarrier wait is bounded (timeout -> SSD_ERR_TIMEOUT in the status word, then no
// role of the CTA waits any longer).
#include <cstring>

#include "matvec_b.cuh"
#include "matvec_dev.cuh"
#include "umma.cuh"

namespace ssd {

constexpr int kBN = kBatchTokens;     // tokens per launch (16)
constexpr int kBCols = 4 * kBN;       // MMA N: 4 limbs per token
constexpr int kBRW = 16;              // readout warps: 4 warp groups of 4 tokens each
constexpr int kBTG = kBN / (kBRW / 4);  // tokens per readout thread
// warps 0-15 readout, 16 producer, 17 MMA, 18-21 unpack
constexpr int kBThreads = (kBRW + 6) * 32;
constexpr int kBMaxStages = 6;
constexpr int kBASlots = 2;
constexpr int kBDSlots = 2;           // TMEM slots of 4 blocks x 64 columns
constexpr uint32_t kBTmemCols = 512;
constexpr int kBBlk = 2 * kBCols * 16;  // B bytes per block: 2 K halves x 64 rows x 16 B
constexpr int kBUnitB = 8 * kBBlk;      // B bytes per unit (16 KB)
constexpr int kBCst = 1024;             // scale table bytes per unit: sx[8], X[8][16]
// kind::i8, s32 accumulator, A and B signed, K-major, M = 128, N = 64
constexpr uint32_t kBIdesc =
    (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBCols >> 3) << 17) | ((128u >> 4) << 24);

template <int FMT>
struct BFmt {
    static constexpr bool NIB = FMT == SSD_TYPE_Q4_0 || FMT == SSD_TYPE_Q4_K;
    static constexpr int QBOX = NIB ? 1 : 2;
    static constexpr int QB = QBOX * 16384;
    static constexpr int MB = 16 * 128;
    static constexpr int STAGE = QB + MB + kBUnitB + kBCst;  // multiple of 1024
    static constexpr bool SUMX = FMT == SSD_TYPE_Q4_K;
};

struct BPlan {
    size_t ring, a, rope, red, bars, total;
};
__host__ __device__ inline BPlan b_plan(int stage_bytes, bool nib, int stages, bool rope, bool swiglu) {
    BPlan p;
    size_t o = 0;
    p.ring = o;
    o += (size_t)stages * stage_bytes;
    p.a = o;
    o += nib ? (size_t)kBASlots * 16384 : 0;
    p.rope = o;  // (cos, sin) per token and pair, head_dim <= 128
    o += rope ? (size_t)kBN * 64 * 8 : 0;
    p.red = o;  // SwiGLU exchange [16][128] floats, else flags
    o += swiglu ? (size_t)kBN * 128 * 4 : 64;
    p.bars = o;
    o += 48 * 8;
    p.total = o + 1024;
    return p;
}

__device__ __forceinline__ uint64_t b_desc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;
    return d;
}
// D += A B: every TMEM slot holds the preset kBMagic before its MMAs (see the readout)
__device__ __forceinline__ void b_umma(uint32_t tmem_d, uint64_t da, uint64_t db) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %3, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %4, p;\n}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(1u), "r"(kBIdesc)
        : "memory");
}
// 0x4B400000 = 1.5 * 2^23 as fp32 bits. An int32 accumulator preset to it and added an
// exact limb sum c (|c| < 2^19, well inside 2^22) holds the bits of the fp32 value
// 1.5 * 2^23 + c, so the readout recovers c with one exact subtraction (no conversion).
constexpr uint32_t kBMagic = 0x4B400000u;
constexpr float kBMagicF = 12582912.0f;
__device__ __forceinline__ void b_tmem_st_magic4(uint32_t taddr) {
    const uint32_t m = kBMagic;
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %1, %1, %1};" ::"r"(taddr), "r"(m)
                 : "memory");
}
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
// (a0, a1) += d * (F - M) for the preset-carrying pair F, exact subtraction then one fma
__device__ __forceinline__ uint64_t b_acc2(uint64_t acc, uint64_t F, uint64_t nM, uint64_t d) {
    uint64_t g;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(g) : "l"(F), "l"(nM));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(g), "l"(d));
    return acc;
}
// kBTG consecutive 32-bit TMEM columns of this thread's lane (no wait).
__device__ __forceinline__ void b_tmem_ld4(uint32_t taddr, uint32_t (&v)[kBTG]) {
    static_assert(kBTG == 4, "x4 loads");
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr));
}
__device__ __forceinline__ void b_bar(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void b_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                       int* status) {
    if (*abort) return;
    const uint32_t addr = smem_u32(bar);
    for (uint32_t it = 0; it < (1u << 21); it++) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return;
        if ((it & 63) == 63 && *abort) return;
    }
    atomicExch(status, SSD_ERR_TIMEOUT);
    *abort = 1;
}
// 1-D bulk copy global -> shared completing on an mbarrier (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void b_bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void b_scale_min(const uint4& m, int sb, uint32_t& s6, uint32_t& m6) {
    auto byte = [&](int i) {
        const uint32_t w = (i >> 2) == 0 ? m.y : ((i >> 2) == 1 ? m.z : m.w);
        return (w >> (8 * (i & 3))) & 0xFFu;
    };
    if (sb < 4) {
        s6 = byte(sb) & 63u;
        m6 = byte(sb + 4) & 63u;
    } else {
        s6 = (byte(sb - 4) >> 6) | ((byte(sb + 4) & 15u) << 2);
        m6 = (byte(sb) >> 6) | ((byte(sb + 4) >> 4) << 2);
    }
}

// ----------------------------------------------------------------------- norm stats
// inv_rms of every token's x_eff (x + x_add): one CTA of 1024 threads per token, all of its
// row's float4 loads in flight at once, sum of squares fp32 (rmsnorm_f32_fast_scalar,
// src/metal/compute.rs:580-588: inv_rms = 1 / sqrt(sum_sq / n + eps)).
__global__ void __launch_bounds__(1024) k_bstats(const BPrepArgs p) {
    __shared__ float red[32];
    const int t = blockIdx.x, tid = threadIdx.x;
    pdl_wait();
    // the dependent's part before its own wait only reads weights: let it launch now
    pdl_trigger();
    const float4* x4 = reinterpret_cast<const float4*>(p.x + (size_t)t * p.ldx);
    const float4* a4 = p.x_add ? reinterpret_cast<const float4*>(p.x_add + (size_t)t * p.ldx) : nullptr;
    const int n4 = p.cols / 4;
    constexpr int kIn = 8;  // float4 per thread per round (rows up to 32768 in one round)
    float ss = 0.0f;
    for (int i0 = tid; i0 < n4; i0 += kIn * 1024) {
        float4 v[kIn];
#pragma unroll
        for (int j = 0; j < kIn; j++) {
            const int i = i0 + j * 1024;
            v[j] = i < n4 ? __ldcg(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            if (a4 && i < n4) {
                const float4 w = __ldcg(a4 + i);
                v[j].x = __fadd_rn(v[j].x, w.x);
                v[j].y = __fadd_rn(v[j].y, w.y);
                v[j].z = __fadd_rn(v[j].z, w.z);
                v[j].w = __fadd_rn(v[j].w, w.w);
            }
        }
#pragma unroll
        for (int j = 0; j < kIn; j++) {
            ss = fmaf(v[j].x, v[j].x, ss);
            ss = fmaf(v[j].y, v[j].y, ss);
            ss = fmaf(v[j].z, v[j].z, ss);
            ss = fmaf(v[j].w, v[j].w, ss);
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid < 32) {
        float v = red[tid];
        v = warp_sum(v);
        if (tid == 0)
            p.inv[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, (float)p.cols), p.eps)));
    }
}

// ----------------------------------------------------------------------- B prep
// One CTA (256 threads) per k-group of 256 columns. Warp w = block w of the group, lane =
// element; the 16 tokens are looped. NIB: nibble formats (block K order: 16 even elements,
// then 16 odd ones).
template <bool NIB, bool SUMX>
__global__ void __launch_bounds__(256) k_bprep(const BPrepArgs p) {
    __shared__ __align__(16) uint8_t tile[kBUnitB];
    __shared__ float inv_s[kBN];
    __shared__ float xsum[8][kBN];
    __shared__ float sxs[8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kg = blockIdx.x;
    const int c = warp;  // block within the k-group
    const int k = kg * 256 + c * 32 + lane;
    // the norm weight is a weight (never written by the previous kernel): load it first
    const float w = p.norm_w ? __ldg(p.norm_w + k) : 0.0f;
    pdl_wait();
    // k_mv_b, the dependent, streams its first weight stages before its wait: launching it
    // now overlaps that with this kernel
    pdl_trigger();
    // x_eff of token t, element k
    auto xe = [&](int t, int k) {
        float v = __ldcg(p.x + (size_t)t * p.ldx + k);
        if (p.x_add) v = __fadd_rn(v, __ldcg(p.x_add + (size_t)t * p.ldx + k));
        return v;
    };
    float v[kBN];
#pragma unroll
    for (int t = 0; t < kBN; t++) v[t] = xe(t, k);
    if (p.norm_w) {  // the tokens' inverse RMS, loaded while the x loads are in flight
        if (tid < kBN) inv_s[tid] = __ldcg(p.inv + tid);
        __syncthreads();
    }
    if (p.x_writeback) {
#pragma unroll
        for (int t = 0; t < kBN; t++) p.x_writeback[(size_t)t * p.ldx + k] = v[t];
    }
    if (p.norm_w) {
#pragma unroll
        for (int t = 0; t < kBN; t++)
            v[t] = p.norm_order == 0 ? __fmul_rn(v[t], __fmul_rn(inv_s[t], w))
                                     : __fmul_rn(__fmul_rn(v[t], inv_s[t]), w);
    }
    uint32_t mx = 0;
#pragma unroll
    for (int t = 0; t < kBN; t++) mx = max(mx, __float_as_uint(v[t]) & 0x7FFFFFFFu);
    mx = __reduce_max_sync(0xffffffffu, mx);
    const int ex = (int)(mx >> 23);
    int e = mx == 0 ? 0 : 152 - ex;
    e = e < -100 ? -100 : (e > 126 ? 126 : e);
    const float sc = __uint_as_float((uint32_t)(e + 127) << 23);
    // K position of this element in the block; limb l of token t (B row 16 l + t) at
    // [(2 c + h) * 64 + 16 l + t] * 16 + idx
    const int pp = NIB ? ((lane & 1) * 16 + (lane >> 1)) : lane;
    const int h = pp >> 4, idx = pp & 15;
    uint8_t* tb = tile + (size_t)(2 * c + h) * kBCols * 16 + idx;
#pragma unroll
    for (int t = 0; t < kBN; t++) {
        int xf = __float2int_rn(__fmul_rn(v[t], sc));
        const int l0 = (int)(int8_t)(xf & 0xFF);
        xf = (xf - l0) >> 8;
        const int l1 = (int)(int8_t)(xf & 0xFF);
        xf = (xf - l1) >> 8;
        const int l2 = (int)(int8_t)(xf & 0xFF);
        const int l3 = (xf - l2) >> 8;
        tb[(0 * kBN + t) * 16] = (uint8_t)l0;
        tb[(1 * kBN + t) * 16] = (uint8_t)l1;
        tb[(2 * kBN + t) * 16] = (uint8_t)l2;
        tb[(3 * kBN + t) * 16] = (uint8_t)l3;
        if constexpr (SUMX) {
            const float X = warp_sum(v[t]);
            if (lane == 0) xsum[c][t] = X;
        }
    }
    if (lane == 0) {
        // 2^-e (2^-(e+4) for the nibble formats, whose A carries 16 (q - 8)); a non-finite
        // block makes the rows NaN, as the reference's sums would be
        const int es = NIB ? e + 4 : e;
        float sx = es <= 126 ? __uint_as_float((uint32_t)(127 - es) << 23)
                             : __uint_as_float(1u << (149 - es));
        if (ex == 0xFF) sx = __int_as_float(0x7FC00000);
        sxs[c] = sx;
    }
    __syncthreads();
    uint4* dst = reinterpret_cast<uint4*>(p.b + (size_t)kg * kBUnitB);
    const uint4* src = reinterpret_cast<const uint4*>(tile);
    for (int i = tid; i < kBUnitB / 16; i += 256) dst[i] = src[i];
    float* cst = p.cst + (size_t)kg * (kBCst / 4);
    if (tid < 8) cst[tid] = sxs[tid];
    if constexpr (SUMX) {
        if (tid < 8 * kBN) cst[8 + tid] = xsum[tid / kBN][tid % kBN];
    }
}

// ----------------------------------------------------------------------- matvec
template <int FMT, int EPI>
__global__ void __launch_bounds__(kBThreads, 1)
    k_mv_b(const MvArgs a, const BWork wk, const __grid_constant__ I8MapsB maps) {
    using F = BFmt<FMT>;
    constexpr int kMap = epi_map(EPI);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const BPlan P = b_plan(F::STAGE, F::NIB, wk.stages, EPI == EPI_QKV_ROPE, EPI == EPI_SWIGLU);
    const int S = wk.stages;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + P.bars);
    uint64_t* p_full = bars;
    uint64_t* p_empty = bars + kBMaxStages;
    uint64_t* a_full = bars + 2 * kBMaxStages;
    uint64_t* a_empty = a_full + kBASlots;
    uint64_t* d_full = a_empty + kBASlots;
    uint64_t* d_empty = d_full + kBDSlots;
    uint64_t* mma_done = d_empty + kBDSlots;
    uint64_t* tmem_ready = mma_done + 8;  // every TMEM slot preset (readout warps)
    uint32_t* tslot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(mma_done + 2);
    int* flag = reinterpret_cast<int*>(mma_done + 3);
    float* red = reinterpret_cast<float*>(base + P.red);
    float2* rope_tab = reinterpret_cast<float2*>(base + P.rope);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int U = wk.n_units, nk = wk.nk;
    const int u0 = (int)((long long)U * b / G), u1 = (int)((long long)U * (b + 1) / G);
    const int n = u1 - u0;
    const int t0 = u0 / nk, kg0 = u0 % nk;

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(p_full + s, 1);
            // readout warps, MMA commit, and (nibble formats) unpack warps
            mbar_init(p_empty + s, F::NIB ? kBRW + 5 : kBRW + 1);
        }
        for (int s = 0; s < kBASlots; s++) {
            mbar_init(a_full + s, 4);
            mbar_init(a_empty + s, 1);
        }
        for (int s = 0; s < kBDSlots; s++) {
            mbar_init(d_full + s, 1);
            mbar_init(d_empty + s, kBRW);
        }
        mbar_init(mma_done, 1);
        mbar_init(tmem_ready, kBRW);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tslot, kBTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_trigger();

    if (warp == kBRW) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            // weights of one unit into stage ps (the B block follows separately)
            auto issue_w = [&](int i, int t, int kg, int ps) {
                int seg, r0;
                if constexpr (kMap == MAP_SWIGLU) {
                    seg = 0;
                    r0 = 64 * t;
                } else {
                    map_row<kMap>(a, 128, 128 * t, seg, r0);
                }
                uint8_t* st = base + P.ring + (size_t)ps * F::STAGE;
                mbar_expect_tx(p_full + ps, (uint32_t)F::STAGE);
                if constexpr (kMap == MAP_SWIGLU) {
#pragma unroll
                    for (int h = 0; h < 2; h++) {
#pragma unroll
                        for (int qb = 0; qb < F::QBOX; qb++)
                            tma_load_2d(st + qb * 16384 + h * 8192, &maps.q[h],
                                        (kg * F::QBOX + qb) * 128, r0, p_full + ps);
                        tma_load_2d(st + F::QB + h * 1024, &maps.m[h], kg * 16, r0, p_full + ps);
                    }
                } else {
#pragma unroll
                    for (int qb = 0; qb < F::QBOX; qb++)
                        tma_load_2d(st + qb * 16384, &maps.q[seg], (kg * F::QBOX + qb) * 128, r0,
                                    p_full + ps);
                    tma_load_2d(st + F::QB, &maps.m[seg], kg * 16, r0, p_full + ps);
                }
            };
            // the unit's B block and scale table, produced by k_bprep (the previous kernel)
            auto issue_b = [&](int kg, int ps) {
                uint8_t* st = base + P.ring + (size_t)ps * F::STAGE;
                b_bulk(st + F::QB + F::MB, wk.b + (size_t)kg * kBUnitB, kBUnitB, p_full + ps);
                b_bulk(st + F::QB + F::MB + kBUnitB, wk.cst + (size_t)kg * (kBCst / 4), kBCst,
                       p_full + ps);
            };
            // weights of the first stages before the PDL wait, their B blocks after it
            const int pre = n < S ? n : S;
            int t = t0, kg = kg0;
            for (int i = 0; i < pre; i++) {
                issue_w(i, t, kg, i);
                if (++kg == nk) {
                    kg = 0;
                    t++;
                }
            }
            pdl_wait();
            int kb = kg0;
            for (int i = 0; i < pre; i++) {
                issue_b(kb, i);
                if (++kb == nk) kb = 0;
            }
            int ps = pre % S, rnd = pre / S;
            for (int i = pre; i < n; i++) {
                b_wait(p_empty + ps, (rnd - 1) & 1, abort, a.status);
                issue_w(i, t, kg, ps);
                issue_b(kg, ps);
                if (++kg == nk) {
                    kg = 0;
                    t++;
                }
                if (++ps == S) {
                    ps = 0;
                    rnd++;
                }
            }
            ps = n % S;
            rnd = n / S;
            for (int k = 0; k < (n < S ? n : S); k++) {
                if (--ps < 0) {
                    ps = S - 1;
                    rnd--;
                }
                b_wait(p_full + ps, rnd & 1, abort, a.status);
            }
        }
    } else if (warp == kBRW + 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            b_wait(tmem_ready, 0, abort, a.status);
            int ps = 0, rnd = 0, as = 0, aph = 0, ds = 0, dph = 0;
            for (int h = 0; h < 2 * n; h++) {
                const int hh = h & 1;
                if (hh == 0) b_wait(p_full + ps, rnd & 1, abort, a.status);
                if constexpr (F::NIB) b_wait(a_full + as, aph, abort, a.status);
                if (h >= kBDSlots) b_wait(d_empty + ds, dph ^ 1, abort, a.status);
                tc_fence_after();
                uint8_t* st = base + P.ring + (size_t)ps * F::STAGE;
                const uint32_t abase =
                    F::NIB ? smem_u32(base + P.a + (size_t)as * 16384) : smem_u32(st + hh * 16384);
                const uint64_t da = umma_desc_sw128(abase);
                // B of block 4 hh + j: K halves 1 KB apart (LBO), 8-row groups 128 B (SBO)
                const uint64_t db = b_desc_plain(smem_u32(st + F::QB + F::MB + hh * 4 * kBBlk),
                                                 kBCols * 16, 128);
                const uint32_t td = tmem + (uint32_t)(ds * 4 * kBCols);
#pragma unroll
                for (int j = 0; j < 4; j++)
                    b_umma(td + (uint32_t)(j * kBCols), da + (uint64_t)(2 * j),
                           db + (uint64_t)((j * kBBlk) >> 4));
                umma_commit(d_full + ds);
                if constexpr (F::NIB) umma_commit(a_empty + as);
                if (hh) umma_commit(p_empty + ps);
                if constexpr (F::NIB) {
                    if (++as == kBASlots) {
                        as = 0;
                        aph ^= 1;
                    }
                }
                if (++ds == kBDSlots) {
                    ds = 0;
                    dph ^= 1;
                }
                if (hh && ++ps == S) {
                    ps = 0;
                    rnd++;
                }
            }
            umma_commit(mma_done);
            if (n > 0) b_wait(mma_done, 0, abort, a.status);
        }
    } else if (warp >= kBRW + 2) {
        // ------------------------------------------------------------ nibble unpack
        if constexpr (F::NIB) {
            const int r = tid - (kBRW + 2) * 32;
            int ps = 0, rnd = 0, as = 0, aph = 0;
            for (int h = 0; h < 2 * n; h++) {
                const int hh = h & 1;
                if (hh == 0) b_wait(p_full + ps, rnd & 1, abort, a.status);
                if (h >= kBASlots) b_wait(a_empty + as, aph ^ 1, abort, a.status);
                const uint8_t* qrow = base + P.ring + (size_t)ps * F::STAGE + r * 128;
                uint8_t* arow = base + P.a + (size_t)as * 16384 + r * 128;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int c = 4 * hh + j;
                    const uint4 w = *reinterpret_cast<const uint4*>(qrow + ((c ^ (r & 7)) << 4));
                    uint4 lo, hi;
                    lo.x = ((w.x << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
                    lo.y = ((w.y << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
                    lo.z = ((w.z << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
                    lo.w = ((w.w << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
                    hi.x = (w.x & 0xF0F0F0F0u) ^ 0x80808080u;
                    hi.y = (w.y & 0xF0F0F0F0u) ^ 0x80808080u;
                    hi.z = (w.z & 0xF0F0F0F0u) ^ 0x80808080u;
                    hi.w = (w.w & 0xF0F0F0F0u) ^ 0x80808080u;
                    *reinterpret_cast<uint4*>(arow + (((2 * j) ^ (r & 7)) << 4)) = lo;
                    *reinterpret_cast<uint4*>(arow + (((2 * j + 1) ^ (r & 7)) << 4)) = hi;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(a_full + as);
                    if (hh) mbar_arrive(p_empty + ps);
                }
                if (++as == kBASlots) {
                    as = 0;
                    aph ^= 1;
                }
                if (hh && ++ps == S) {
                    ps = 0;
                    rnd++;
                }
            }
        }
    } else {
        // ------------------------------------------------------------ readout warps 0-15
        const int r = tid & 127;       // tile row = TMEM lane
        const int tg = tid >> 7;       // tokens kBTG tg .. kBTG tg + kBTG - 1
        pdl_wait();
        if constexpr (EPI == EPI_QKV_ROPE) {
            for (int i = tid; i < kBN * (a.head_dim >> 1); i += kBRW * 32) {
                const int t = i / (a.head_dim >> 1), pr = i % (a.head_dim >> 1);
                rope_tab[t * 64 + pr] = rope_pair(a, pr, wk.pos[t]);
            }
            b_bar(1, kBRW * 32);
        }
        // accumulators of tokens (8 tg + 2 p, 8 tg + 2 p + 1) as fp32 pairs
        uint64_t acc2[kBTG / 2];
#pragma unroll
        for (int q = 0; q < kBTG / 2; q++) acc2[q] = 0ull;
        int seg_first = kg0;
        int t = t0, kg = kg0, ps = 0, rnd = 0, ds = 0, dph = 0;
        uint4 meta = make_uint4(0, 0, 0, 0);
        const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(kBTG * tg);
        // preset every slot's columns of this warp group before the first MMA
#pragma unroll
        for (int q = 0; q < kBDSlots * 4; q++)
#pragma unroll
            for (int l = 0; l < 4; l++) b_tmem_st_magic4(tl + (uint32_t)(q * kBCols + l * kBN));
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tmem_ready);
        const uint64_t nM = f2pack(-kBMagicF, -kBMagicF);
        for (int h = 0; h < 2 * n; h++) {
            const int i = h >> 1, hh = h & 1;
            const uint8_t* st = base + P.ring + (size_t)ps * F::STAGE;
            const float* cst = reinterpret_cast<const float*>(st + F::QB + F::MB + kBUnitB);
            if (hh == 0) {
                b_wait(p_full + ps, rnd & 1, abort, a.status);
                meta = *reinterpret_cast<const uint4*>(st + F::QB + r * 16);
            }
            b_wait(d_full + ds, dph, abort, a.status);
            tc_fence_after();
#pragma unroll
            for (int j = 0; j < 4; j++) {
                // limb l of this group's tokens: columns 16 l + kBTG tg .. (tl adds kBTG tg)
                const uint32_t ta = tl + (uint32_t)(ds * 4 * kBCols + j * kBCols);
                uint32_t cv[4][kBTG];
#pragma unroll
                for (int l = 0; l < 4; l++) b_tmem_ld4(ta + (uint32_t)(l * kBN), cv[l]);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int l = 0; l < 4; l++) b_tmem_st_magic4(ta + (uint32_t)(l * kBN));  // next preset
                const int c = 4 * hh + j;
                const float sx = cst[c];
                float dd, bias_s = 0.0f;
                if constexpr (FMT == SSD_TYPE_Q4_K) {
                    const float d = f16_bits_to_f32((uint16_t)(meta.x & 0xFFFF));
                    const float dmin = f16_bits_to_f32((uint16_t)(meta.x >> 16));
                    uint32_t s6, m6;
                    b_scale_min(meta, c, s6, m6);
                    const float scale = __fmul_rn(d, (float)s6);
                    const float mn = __fmul_rn(dmin, (float)m6);
                    dd = __fmul_rn(scale, sx);
                    bias_s = __fsub_rn(__fmul_rn(8.0f, scale), mn);
                } else {
                    const uint32_t mw = c < 2 ? meta.x : (c < 4 ? meta.y : (c < 6 ? meta.z : meta.w));
                    const float d = f16_bits_to_f32((uint16_t)((c & 1) ? (mw >> 16) : (mw & 0xFFFF)));
                    dd = __fmul_rn(d, sx);
                }
                // limb l weighs 256^l: d * 2^-e * 256^l is exact (a power-of-two scaling)
                const uint64_t dl[4] = {f2pack(dd, dd), f2pack(dd * 256.0f, dd * 256.0f),
                                        f2pack(dd * 65536.0f, dd * 65536.0f),
                                        f2pack(dd * 16777216.0f, dd * 16777216.0f)};
#pragma unroll
                for (int q = 0; q < kBTG / 2; q++) {
#pragma unroll
                    for (int l = 3; l >= 0; l--)
                        acc2[q] = b_acc2(acc2[q], f2pack(__uint_as_float(cv[l][2 * q]),
                                                         __uint_as_float(cv[l][2 * q + 1])),
                                         nM, dl[l]);
                    if constexpr (FMT == SSD_TYPE_Q4_K) {
                        const float* X = cst + 8 + c * kBN + kBTG * tg + 2 * q;
                        asm("fma.rn.f32x2 %0, %1, %2, %0;"
                            : "+l"(acc2[q])
                            : "l"(f2pack(bias_s, bias_s)), "l"(f2pack(X[0], X[1])));
                    }
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(d_empty + ds);
                if (hh) mbar_arrive(p_empty + ps);
            }
            if (++ds == kBDSlots) {
                ds = 0;
                dph ^= 1;
            }
            if (hh == 0) continue;
            if (++ps == S) {
                ps = 0;
                rnd++;
            }
            const int tcur = t, kcur = kg;
            if (++kg == nk) {
                kg = 0;
                t++;
            }
            if (i != n - 1 && kcur != nk - 1) continue;
            const bool whole = seg_first == 0 && kcur == nk - 1;
            seg_first = 0;
            float res[kBTG];
#pragma unroll
            for (int q = 0; q < kBTG / 2; q++) {
                f2unpack(acc2[q], res[2 * q], res[2 * q + 1]);
                acc2[q] = 0ull;
            }
            bool do_epi = whole;
            if (!whole) {
                // partial rows [slot][token][128] of this CTA; the last CTA of the tile to
                // arrive adds every CTA's partial in CTA order
                const int slot = tcur == t0 ? 0 : 1;
                float* pp = wk.partial + ((size_t)b * 2 + slot) * kBN * 128;
#pragma unroll
                for (int q = 0; q < kBTG; q++) pp[(kBTG * tg + q) * 128 + r] = res[q];
                b_bar(1, kBRW * 32);
                const long long U64 = U;
                const int bf = (int)((((long long)tcur * nk + 1) * G + U64 - 1) / U64) - 1;
                const int bl = (int)((((long long)tcur * nk + nk) * G + U64 - 1) / U64) - 1;
                if (tid == 0) {
                    unsigned prev;
                    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                                 : "=r"(prev)
                                 : "l"(wk.counter + tcur)
                                 : "memory");
                    const bool last = prev == (unsigned)(bl - bf);
                    if (last) wk.counter[tcur] = 0u;
                    flag[0] = last;
                }
                b_bar(1, kBRW * 32);
                do_epi = flag[0] != 0;
                if (do_epi) {
#pragma unroll
                    for (int q = 0; q < kBTG; q++) res[q] = 0.0f;
                    for (int bc = bf; bc <= bl; bc++) {
                        const int tf = (int)(((long long)U * bc / G) / nk);
                        const float* pc = wk.partial + ((size_t)bc * 2 + (tcur == tf ? 0 : 1)) * kBN * 128;
#pragma unroll
                        for (int q = 0; q < kBTG; q++) res[q] += __ldcg(pc + (kBTG * tg + q) * 128 + r);
                    }
                }
                b_bar(1, kBRW * 32);
            }
            if (!do_epi) continue;
            // ---- epilogue of tile tcur, row r, tokens 8 tg + q
            if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll
                for (int q = 0; q < kBTG; q++) red[(kBTG * tg + q) * 128 + r] = res[q];
                b_bar(1, kBRW * 32);
                const int row = 64 * tcur + r;
                if (r < 64 && row < a.seg_rows[0]) {
#pragma unroll
                    for (int q = 0; q < kBTG; q++) {
                        const int tt = kBTG * tg + q;
                        a.y[(size_t)tt * wk.ldy + row] =
                            swiglu(red[tt * 128 + r], red[tt * 128 + r + 64]);
                    }
                }
                b_bar(1, kBRW * 32);
            } else if constexpr (EPI == EPI_QKV_ROPE) {
                int seg, lr;
                map_row<kMap>(a, 128, 128 * tcur + r, seg, lr);
                const bool valid = 128 * tcur + r < a.rows;
                float* dst = seg == 0 ? a.y : (seg == 1 ? a.y_k : a.y_v);
                const int ld = seg == 0 ? wk.ldy : wk.ldk;
#pragma unroll
                for (int q = 0; q < kBTG; q++) {
                    const int tt = kBTG * tg + q;
                    const float other = __shfl_xor_sync(0xffffffffu, res[q], 1);
                    float x0 = (r & 1) ? other : res[q], x1 = (r & 1) ? res[q] : other;
                    if (seg < 2) rope_apply(x0, x1, rope_tab[tt * 64 + ((lr % a.head_dim) >> 1)]);
                    if (valid) dst[(size_t)tt * ld + lr] = (r & 1) ? x1 : x0;
                }
            } else {
                const int row = 128 * tcur + r;
                const bool valid = row < a.rows;
                if constexpr (EPI == EPI_STORE || EPI == EPI_RESID) {
                    if (valid) {
#pragma unroll
                        for (int q = 0; q < kBTG; q++) {
                            const int tt = kBTG * tg + q;
                            float v = res[q];
                            if (EPI == EPI_RESID) v = __fadd_rn(a.base[(size_t)tt * wk.ldy + row], v);
                            a.y[(size_t)tt * wk.ldy + row] = v;
                        }
                    }
                } else {  // EPI_ARGMAX: one key per token
#pragma unroll
                    for (int q = 0; q < kBTG; q++) {
                        const int tt = kBTG * tg + q;
                        unsigned long long key = 0ull;
                        if (valid) {
                            if (a.y) a.y[(size_t)tt * wk.ldy + row] = res[q];
                            key = argmax_key(res[q], (uint32_t)(row + a.index_offset));
                        }
#pragma unroll
                        for (int o = 16; o; o >>= 1) {
                            const unsigned long long kk = __shfl_xor_sync(0xffffffffu, key, o);
                            key = kk > key ? kk : key;
                        }
                        if (lane == 0 && key) atomicMax(wk.keys + tt, key);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kBTmemCols);
    }
}

// --------------------------------------------------------------- host side

int launch_bprep(ssd_ctx* ctx, int type, const BPrepArgs& p, cudaStream_t s, bool pdl) {
    (void)ctx;
    SSD_REQ(p.cols > 0 && p.cols % 256 == 0, SSD_ERR_SHAPE, "batch prep: cols %d %% 256", p.cols);
    SSD_REQ(p.x && p.b && p.cst, SSD_ERR_ARG, "batch prep: null buffer");
    const bool nib = type == SSD_TYPE_Q4_0 || type == SSD_TYPE_Q4_K;
    const int nk = p.cols / 256;
    if (p.norm_w) {
        SSD_REQ(p.inv != nullptr && p.cols % 4 == 0, SSD_ERR_ARG, "batch prep: norm needs inv");
        SSD_CK(launch_pdl(k_bstats, dim3(kBN), dim3(1024), 0, s, pdl, p));
    }
    if (type == SSD_TYPE_Q4_K)
        SSD_CK(launch_pdl(k_bprep<true, true>, dim3(nk), dim3(256), 0, s, pdl, p));
    else if (nib)
        SSD_CK(launch_pdl(k_bprep<true, false>, dim3(nk), dim3(256), 0, s, pdl, p));
    else
        SSD_CK(launch_pdl(k_bprep<false, false>, dim3(nk), dim3(256), 0, s, pdl, p));
    return SSD_OK;
}

template <int FMT, int EPI>
static int launch_b_t(ssd_ctx* ctx, const MvArgs& a, BWork wk, cudaStream_t s, bool pdl) {
    using F = BFmt<FMT>;
    constexpr int kMap = epi_map(EPI);
    const int nk = a.cols / 256;
    const int n_tiles = kMap == MAP_SWIGLU ? a.seg_rows[0] / 64 : (a.rows + 127) / 128;
    const long long U = (long long)n_tiles * nk;
    int G = ctx->num_sms < kI8MaxGrid ? ctx->num_sms : kI8MaxGrid;
    if (U < G) G = (int)U;
    const int per = (int)((U + G - 1) / G);
    int stages = per < kBMaxStages ? per : kBMaxStages;
    if (stages < 2) stages = 2;
    constexpr bool kRope = EPI == EPI_QKV_ROPE, kSw = EPI == EPI_SWIGLU;
    while (stages > 2 && b_plan(F::STAGE, F::NIB, stages, kRope, kSw).total > ctx->smem_optin) stages--;
    const BPlan P = b_plan(F::STAGE, F::NIB, stages, kRope, kSw);
    SSD_REQ(P.total <= ctx->smem_optin, SSD_ERR_SHAPE, "batch matvec: %zu bytes of shared memory",
            P.total);
    wk.n_tiles = n_tiles;
    wk.nk = nk;
    wk.n_units = (int)U;
    wk.stages = stages;
    I8MapsB maps;
    memset(&maps, 0, sizeof(maps));
    const int nseg = kMap == MAP_QKV ? 3 : (kMap == MAP_SWIGLU ? 2 : 1);
    const uint32_t BR = kMap == MAP_SWIGLU ? 64 : 128;
    const uint64_t qrow = (uint64_t)(a.cols / 32) * (F::NIB ? 16 : 32);
    const uint64_t mrow = (uint64_t)(a.cols / 32) * 2;
    for (int g = 0; g < nseg; g++) {
        const uint64_t rows = (uint64_t)(kMap == MAP_PLAIN ? a.rows : a.seg_rows[g]);
        SSD_TRY(encode_bytes_map(&maps.q[g], a.qs[g], qrow, rows, 128, BR, true));
        SSD_TRY(encode_bytes_map(&maps.m[g], a.meta[g], mrow, rows, 16, BR, false));
    }
    auto kern = k_mv_b<FMT, EPI>;
    static bool attr = false;
    if (!attr) {
        SSD_CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)ctx->smem_optin));
        attr = true;
    }
    SSD_CK(launch_pdl(kern, dim3(G), dim3(kBThreads), P.total, s, pdl, a, wk, maps));
    return SSD_OK;
}

template <int FMT>
static int launch_b_fmt(ssd_ctx* ctx, int epi, const MvArgs& a, const BWork& wk, cudaStream_t s,
                        bool pdl) {
    switch (epi) {
        case EPI_STORE: return launch_b_t<FMT, EPI_STORE>(ctx, a, wk, s, pdl);
        case EPI_RESID: return launch_b_t<FMT, EPI_RESID>(ctx, a, wk, s, pdl);
        case EPI_SWIGLU: return launch_b_t<FMT, EPI_SWIGLU>(ctx, a, wk, s, pdl);
        case EPI_QKV_ROPE: return launch_b_t<FMT, EPI_QKV_ROPE>(ctx, a, wk, s, pdl);
        case EPI_ARGMAX: return launch_b_t<FMT, EPI_ARGMAX>(ctx, a, wk, s, pdl);
        default: set_error("batch matvec: epilogue %d", epi); return SSD_ERR_ARG;
    }
}

int launch_matvec_batch(ssd_ctx* ctx, int type, int epi, const MvArgs& a, const BWork& wk,
                        cudaStream_t s, bool pdl) {
    if (!a.status) {
        MvArgs b = a;
        b.status = ctx->dev_status;
        return launch_matvec_batch(ctx, type, epi, b, wk, s, pdl);
    }
    SSD_REQ(a.cols > 0 && a.cols % 256 == 0, SSD_ERR_SHAPE, "batch matvec: cols %d %% 256", a.cols);
    SSD_REQ(wk.b && wk.cst && wk.counter && wk.partial, SSD_ERR_ARG, "batch matvec: null scratch");
    const int map = epi_map(epi);
    SSD_REQ(a.map == map, SSD_ERR_ARG, "row map %d does not match epilogue %d", a.map, epi);
    if (map == MAP_QKV)
        SSD_REQ(a.seg_rows[0] % 128 == 0 && a.seg_rows[1] % 128 == 0 && a.seg_rows[2] % 128 == 0 &&
                    a.head_dim > 0 && a.head_dim <= 128 && a.head_dim % 2 == 0 && wk.pos,
                SSD_ERR_SHAPE, "batch QKV: segments of 128 rows, head_dim <= 128, positions");
    if (map == MAP_SWIGLU) SSD_REQ(a.seg_rows[0] % 64 == 0, SSD_ERR_SHAPE, "batch SwiGLU rows %% 64");
    SSD_REQ(epi != EPI_ARGMAX || wk.keys, SSD_ERR_ARG, "batch argmax: null keys");
    switch (type) {
        case SSD_TYPE_Q4_0: return launch_b_fmt<SSD_TYPE_Q4_0>(ctx, epi, a, wk, s, pdl);
        case SSD_TYPE_Q8_0: return launch_b_fmt<SSD_TYPE_Q8_0>(ctx, epi, a, wk, s, pdl);
        case SSD_TYPE_Q4_K: return launch_b_fmt<SSD_TYPE_Q4_K>(ctx, epi, a, wk, s, pdl);
        default:
            set_error("batch matvec: ggml type %d not supported (Q4_0, Q8_0, Q4_K)", type);
            return SSD_ERR_TYPE;
    }
}

}  // namespace ssd
