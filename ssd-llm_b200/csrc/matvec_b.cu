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
// 32-element block, xf = rint(x 2^e), split into four signed byte limbs. Column 4 t + l of
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
//    (16 KB) with its scale table; warps 10-13 unpack nibbles, warp 9 issues the MMAs,
//    warps 0-7 read TMEM back (warps 0-3 tokens 0-7, warps 4-7 tokens 8-15, lanes = rows).
// Every mbarrier wait is bounded (timeout -> SSD_ERR_TIMEOUT in the status word, then no
// role of the CTA waits any longer).
#include <cstring>

#include "matvec_b.cuh"
#include "matvec_dev.cuh"
#include "umma.cuh"

namespace ssd {

constexpr int kBN = kBatchTokens;     // tokens per launch (16)
constexpr int kBCols = 4 * kBN;       // MMA N: 4 limbs per token
constexpr int kBThreads = 448;        // warps 0-7 readout, 8 producer, 9 MMA, 10-13 unpack
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
__device__ __forceinline__ void b_umma(uint32_t tmem_d, uint64_t da, uint64_t db) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %3, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %4, p;\n}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(0u), "r"(kBIdesc)
        : "memory");
}
// 32 consecutive 32-bit TMEM columns of this thread's lane (no wait).
__device__ __forceinline__ void b_tmem_ld32(uint32_t taddr, int (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
          "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
          "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
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
    pdl_wait();
    // x_eff of token t, element k
    auto xe = [&](int t, int k) {
        float v = __ldcg(p.x + (size_t)t * p.ldx + k);
        if (p.x_add) v = __fadd_rn(v, __ldcg(p.x_add + (size_t)t * p.ldx + k));
        return v;
    };
    if (p.norm_w) {  // per-token inv_rms over the whole row: warp w takes tokens 2w, 2w + 1
        for (int q = 0; q < 2; q++) {
            const int t = 2 * warp + q;
            float ss = 0.0f;
            for (int k0 = lane; k0 < p.cols; k0 += 8 * 32) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; j++) v[j] = k0 + 32 * j < p.cols ? xe(t, k0 + 32 * j) : 0.0f;
#pragma unroll
                for (int j = 0; j < 8; j++) ss = fmaf(v[j], v[j], ss);
            }
            ss = warp_sum(ss);
            // inv_rms = 1 / sqrt(sum_sq / n + eps)   (src/metal/compute.rs:583-584)
            if (lane == 0)
                inv_s[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)p.cols), p.eps)));
        }
        __syncthreads();
    }
    const int c = warp;  // block within the k-group
    const int k = kg * 256 + c * 32 + lane;
    float v[kBN];
#pragma unroll
    for (int t = 0; t < kBN; t++) v[t] = xe(t, k);
    if (p.x_writeback) {
#pragma unroll
        for (int t = 0; t < kBN; t++) p.x_writeback[(size_t)t * p.ldx + k] = v[t];
    }
    if (p.norm_w) {
        const float w = __ldg(p.norm_w + k);
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
    // K position of this element in the block; limb l of token t at
    // [(2 c + h) * 64 + 4 t + l] * 16 + idx
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
        tb[(4 * t + 0) * 16] = (uint8_t)l0;
        tb[(4 * t + 1) * 16] = (uint8_t)l1;
        tb[(4 * t + 2) * 16] = (uint8_t)l2;
        tb[(4 * t + 3) * 16] = (uint8_t)l3;
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
    pdl_trigger();
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
            mbar_init(p_empty + s, F::NIB ? 13 : 9);
        }
        for (int s = 0; s < kBASlots; s++) {
            mbar_init(a_full + s, 4);
            mbar_init(a_empty + s, 1);
        }
        for (int s = 0; s < kBDSlots; s++) {
            mbar_init(d_full + s, 1);
            mbar_init(d_empty + s, 8);
        }
        mbar_init(mma_done, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tslot, kBTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_trigger();

    if (warp == 8) {
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
    } else if (warp == 9) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
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
    } else if (warp >= 10) {
        // ------------------------------------------------------------ nibble unpack
        if constexpr (F::NIB) {
            const int r = tid - 320;
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
        // ------------------------------------------------------------ readout warps 0-7
        const int r = tid & 127;       // tile row = TMEM lane
        const int tg = tid >> 7;       // tokens 8 tg .. 8 tg + 7
        pdl_wait();
        if constexpr (EPI == EPI_QKV_ROPE) {
            for (int i = tid; i < kBN * (a.head_dim >> 1); i += 256) {
                const int t = i / (a.head_dim >> 1), pr = i % (a.head_dim >> 1);
                rope_tab[t * 64 + pr] = rope_cs(pr, a.head_dim, a.theta, wk.pos[t]);
            }
            b_bar(1, 256);
        }
        float acc[8];
#pragma unroll
        for (int q = 0; q < 8; q++) acc[q] = 0.0f;
        int seg_first = kg0;
        int t = t0, kg = kg0, ps = 0, rnd = 0, ds = 0, dph = 0;
        uint4 meta = make_uint4(0, 0, 0, 0);
        const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(32 * tg);
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
                int cv[32];
                b_tmem_ld32(tl + (uint32_t)(ds * 4 * kBCols + j * kBCols), cv);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
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
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const int lo = cv[4 * q] + cv[4 * q + 1] * 256;
                    const int hi = cv[4 * q + 2] + cv[4 * q + 3] * 256;
                    const float tot = fmaf((float)hi, 65536.0f, (float)lo);
                    if constexpr (FMT == SSD_TYPE_Q4_K)
                        acc[q] = fmaf(dd, tot, fmaf(bias_s, cst[8 + c * kBN + 8 * tg + q], acc[q]));
                    else
                        acc[q] = fmaf(dd, tot, acc[q]);
                }
            }
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
            float res[8];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                res[q] = acc[q];
                acc[q] = 0.0f;
            }
            bool do_epi = whole;
            if (!whole) {
                // partial rows [slot][token][128] of this CTA; the last CTA of the tile to
                // arrive adds every CTA's partial in CTA order
                const int slot = tcur == t0 ? 0 : 1;
                float* pp = wk.partial + ((size_t)b * 2 + slot) * kBN * 128;
#pragma unroll
                for (int q = 0; q < 8; q++) pp[(8 * tg + q) * 128 + r] = res[q];
                b_bar(1, 256);
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
                b_bar(1, 256);
                do_epi = flag[0] != 0;
                if (do_epi) {
#pragma unroll
                    for (int q = 0; q < 8; q++) res[q] = 0.0f;
                    for (int bc = bf; bc <= bl; bc++) {
                        const int tf = (int)(((long long)U * bc / G) / nk);
                        const float* pc = wk.partial + ((size_t)bc * 2 + (tcur == tf ? 0 : 1)) * kBN * 128;
#pragma unroll
                        for (int q = 0; q < 8; q++) res[q] += __ldcg(pc + (8 * tg + q) * 128 + r);
                    }
                }
                b_bar(1, 256);
            }
            if (!do_epi) continue;
            // ---- epilogue of tile tcur, row r, tokens 8 tg + q
            if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll
                for (int q = 0; q < 8; q++) red[(8 * tg + q) * 128 + r] = res[q];
                b_bar(1, 256);
                const int row = 64 * tcur + r;
                if (r < 64 && row < a.seg_rows[0]) {
#pragma unroll
                    for (int q = 0; q < 8; q++) {
                        const int tt = 8 * tg + q;
                        a.y[(size_t)tt * wk.ldy + row] =
                            swiglu(red[tt * 128 + r], red[tt * 128 + r + 64]);
                    }
                }
                b_bar(1, 256);
            } else if constexpr (EPI == EPI_QKV_ROPE) {
                int seg, lr;
                map_row<kMap>(a, 128, 128 * tcur + r, seg, lr);
                const bool valid = 128 * tcur + r < a.rows;
                float* dst = seg == 0 ? a.y : (seg == 1 ? a.y_k : a.y_v);
                const int ld = seg == 0 ? wk.ldy : wk.ldk;
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const int tt = 8 * tg + q;
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
                        for (int q = 0; q < 8; q++) {
                            const int tt = 8 * tg + q;
                            float v = res[q];
                            if (EPI == EPI_RESID) v = __fadd_rn(a.base[(size_t)tt * wk.ldy + row], v);
                            a.y[(size_t)tt * wk.ldy + row] = v;
                        }
                    }
                } else {  // EPI_ARGMAX: one key per token
#pragma unroll
                    for (int q = 0; q < 8; q++) {
                        const int tt = 8 * tg + q;
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
