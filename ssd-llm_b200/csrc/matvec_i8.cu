// matvec_i8.cu — fused GGUF dequant-matvec on the tcgen05 integer tensor cores (sm_100a).
//
// Same operator as matvec.cu (matvec_quantized, src/metal/compute.rs:157-191; the
// per-format loops :680-750, :845-925, :971-993), same prologue (residual add, RMSNorm,
// tensor-parallel partials) and epilogues (store, residual, SwiGLU, QKV + RoPE, argmax,
// peer all-reduce). What differs is where the multiply-adds run. The FMA kernel spends
// ~3 instructions per weight (decode, FMA, x reads) and is issue-bound near two thirds
// of HBM bandwidth; here the products run on tcgen05.mma.kind::i8 and the CUDA cores
// only unpack nibbles (~0.4 instructions per weight) and apply one scale per block.
//
// Arithmetic (exact until one fp32 rounding per 32-weight block):
//  * A (M = 128 weight rows x K = 32 per MMA) is the block's integers as signed bytes:
//    Q8_0 / Q8_K bytes as they are, Q5_K bytes (q ^ 0x80 = q - 128) as they are, Q4_0 /
//    Q4_K nibbles unpacked per 32-bit word w into 16 (q - 8):
//      even elements: ((w << 4) & 0xF0F0F0F0) ^ 0x80808080, odd: (w & 0xF0F0F0F0) ^ 0x80808080
//    (element 2j is the low nibble of byte j, src/metal/compute.rs:693-699), so a block's
//    K order is [16 even elements][16 odd elements].
//  * B (K x N = 16) carries x as exact fixed point per 32-element block: xf = rint(x 2^e)
//    with max|x| 2^e in [2^25, 2^26), split into four signed bytes ("limbs",
//    xf = sum_l 256^l b_l). Rows 0-3 of B are the limbs; rows 4-15 read whatever follows
//    in shared memory and only feed TMEM columns that are never read.
//  * Each block's MMA writes its own 16 TMEM columns (no accumulation across blocks:
//    the scale changes every 32 weights); the readout warps combine the four exact int32
//    limb sums, c0 + 256 c1 + 2^16 (c2 + 256 c3), round once to fp32 and add
//    d * 2^-e * sum into the row's fp32 accumulator (Q4_K / Q5_K: scale and min as the
//    FMA kernel, min * X with X the block's sum of x).
//
// Work split ("stream-K"): a unit is 128 rows x 256 columns (8 blocks). The units of all
// row tiles, tile-major, are cut into one contiguous range per CTA (one CTA per SM), so
// every SM gets the same number of units whatever the shape. A tile whose units are
// spread over several CTAs is finished by the last of them to arrive (a counter per
// tile in the weight's scratch): it adds the CTAs' partial rows in CTA order, so the
// result does not depend on timing.
//
// Pipeline per CTA (320 threads):
//  * warp 4 (one thread): TMA producer, a ring of packed stages (payload 128 B boxes with
//    the 128-byte swizzle + the unit's scales); the first stages are issued before the
//    PDL wait, so a small matrix is in shared memory before the previous kernel ends;
//  * warps 6-9 (nibble formats): unpack a stage's nibbles into int8 A tiles (two slots);
//  * warp 5 (one thread): issues the MMAs once the x limbs exist, commits to mbarriers;
//  * warps 0-3: after griddepcontrol.wait build the x limbs (and RMSNorm), then read the
//    TMEM results of each 4-block half-unit (warp w owns TMEM lanes 32w..32w+31 = rows),
//    apply the scales, and run the epilogue of every finished tile.
// Every mbarrier wait is bounded: a timeout records SSD_ERR_TIMEOUT and sets an abort
// flag after which no role waits any longer, so the kernel ends with the status set.
#include <cstring>

#include "matvec_dev.cuh"
#include "umma.cuh"

namespace ssd {

constexpr int kI8Rows = 128;     // rows per tile = TMEM lanes
constexpr int kI8Threads = 320;  // warps 0-3 readout, 4 producer, 5 MMA, 6-9 unpack
constexpr int kI8MaxStages = 8;
constexpr int kI8ASlots = 2;           // unpacked A tiles of 4 blocks (16 KB each)
constexpr int kI8DSlots = 4;           // TMEM slots of 4 blocks x 16 columns
constexpr uint32_t kI8TmemCols = 64 * kI8DSlots;
// kind::i8, s32 accumulator, A and B signed, both K-major, M = 128, N = 16
constexpr uint32_t kI8Idesc =
    (2u << 4) | (1u << 7) | (1u << 10) | ((16u >> 3) << 17) | ((128u >> 4) << 24);

template <int FMT>
struct I8Fmt {
    static constexpr bool NIB = FMT == SSD_TYPE_Q4_0 || FMT == SSD_TYPE_Q4_K;
    static constexpr int QBOX = NIB ? 1 : 2;  // 128-byte payload boxes per (row, unit)
    static constexpr int MROW = FMT == SSD_TYPE_Q8_K ? 32 : 16;  // scale bytes per (row, unit)
    static constexpr int QB = QBOX * 128 * kI8Rows;
    static constexpr int MB = MROW * kI8Rows;
    static constexpr int STAGE = QB + MB;  // a multiple of 1024
    static constexpr bool SUMX = FMT == SSD_TYPE_Q4_K || FMT == SSD_TYPE_Q5_K;  // needs X
};

struct I8Work {
    int n_tiles, nk, n_units, stages, nb;
};

struct I8Maps {
    CUtensorMap q[3];  // payload rows of each segment (box 128 B x BR rows, 128-byte swizzle)
    CUtensorMap m[3];  // scale rows of each segment (box MROW x BR rows)
};

struct I8Plan {
    size_t ring, a, b, cs, bars, rope, red, total;
};
__host__ __device__ inline I8Plan i8_plan(int stage_bytes, bool nib, int stages, int nb, bool rope) {
    I8Plan p;
    size_t o = 0;
    p.ring = o;
    o += (size_t)stages * stage_bytes;
    p.a = o;
    o += nib ? (size_t)kI8ASlots * 16384 : 0;
    p.b = o;  // x limbs: 8 blocks x 128 B per B slot, + the bytes the last block's
    o += (size_t)nb * 1024 + 256;  // descriptor reads past it (unused columns)
    p.cs = o;  // (2^-e scale, X) per block
    o += (size_t)nb * 8 * 8;
    p.bars = o;
    o += 40 * 8;
    p.rope = o;
    o += rope ? (size_t)kMaxRopePairs * 8 : 0;
    p.red = o;  // 128 floats + 32 flags/keys
    o += 128 * 4 + 32 * 8;
    p.total = o + 1024;  // alignment slack
    return p;
}

// Shared-memory descriptor of a K-major operand without swizzle: core matrices of 8 rows x
// 16 bytes, lbo / sbo the byte distances to the next core matrix along K / along rows.
__device__ __forceinline__ uint64_t umma_desc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;
    return d;
}
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t da, uint64_t db) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %3, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %4, p;\n}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(0u), "r"(kI8Idesc)
        : "memory");
}
// 4 consecutive 32-bit TMEM columns of this thread's lane (no wait).
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, int (&v)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void bar_named(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Bounded mbarrier wait that gives up at once after any role of the CTA has timed out.
__device__ __forceinline__ void i8_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
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

__device__ __forceinline__ int owner_of(long long u, int G, long long U) {
    return (int)(((u + 1) * G + U - 1) / U) - 1;
}

// x value k of the prologue: x (+ x_add, or the ranks' partials in rank order), then the
// optional RMSNorm (order 0: v * (inv * w), order 1: (v * inv) * w).
__device__ __forceinline__ float x_eff(const MvArgs& a, int k) {
    float v = __ldcg(a.x + k);
    if (a.ar_in_n > 0) {
        float r = __ldcg(a.ar_in + k);
        for (int p = 1; p < a.ar_in_n; p++) r = __fadd_rn(r, __ldcg(a.ar_in + (size_t)p * a.cols + k));
        v = __fadd_rn(v, r);
    } else if (a.x_add) {
        v = __fadd_rn(v, __ldcg(a.x_add + k));
    }
    return v;
}
__device__ __forceinline__ float x_norm(const MvArgs& a, float v, int k, float inv) {
    if (!a.norm_w) return v;
    const float w = __ldg(a.norm_w + k);
    return a.norm_order == 0 ? __fmul_rn(v, __fmul_rn(inv, w)) : __fmul_rn(__fmul_rn(v, inv), w);
}

// Q4_K / Q5_K 6-bit (scale, min) of sub-block sb from the 12 packed bytes (header bytes
// 4-15, src/metal/compute.rs:725-733), sb a compile-time constant after unrolling.
__device__ __forceinline__ void k_scale_min(const uint4& m, int sb, uint32_t& s6, uint32_t& m6) {
    // byte i of the 12: word (i >> 2) of (m.y, m.z, m.w), selected without local memory
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

template <int FMT, int EPI>
__global__ void __launch_bounds__(kI8Threads, 1)
    k_mv_i8(const MvArgs a, const I8Work wk, const __grid_constant__ I8Maps maps) {
    using F = I8Fmt<FMT>;
    constexpr int kMap = epi_map(EPI);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const I8Plan P = i8_plan(F::STAGE, F::NIB, wk.stages, wk.nb, EPI == EPI_QKV_ROPE);
    const int S = wk.stages;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + P.bars);
    uint64_t* p_full = bars;                      // [S] packed stage landed
    uint64_t* p_empty = bars + kI8MaxStages;      // [S] packed stage consumed
    uint64_t* a_full = bars + 2 * kI8MaxStages;   // [kI8ASlots] A tile unpacked
    uint64_t* a_empty = a_full + kI8ASlots;       // [kI8ASlots] A tile read by the MMAs
    uint64_t* d_full = a_empty + kI8ASlots;       // [kI8DSlots] MMAs of a half-unit done
    uint64_t* d_empty = d_full + kI8DSlots;       // [kI8DSlots] TMEM slot read out
    uint64_t* b_ready = d_empty + kI8DSlots;      // x limbs written
    uint64_t* mma_done = b_ready + 1;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(mma_done + 2);
    float* red = reinterpret_cast<float*>(base + P.red);
    int* flag = reinterpret_cast<int*>(base + P.red + 128 * 4);
    float2* cstab = reinterpret_cast<float2*>(base + P.cs);
    float2* rope_tab = reinterpret_cast<float2*>(base + P.rope);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int U = wk.n_units, nk = wk.nk;
    const int u0 = (int)((long long)U * b / G), u1 = (int)((long long)U * (b + 1) / G);
    const int n = u1 - u0;
    const int t0 = u0 / nk, kg0 = u0 % nk;  // tile and k-group of the first unit
    const bool all_k = n >= nk;  // B slot = k-group when the range covers every k-group,
                                 // else = unit index (k-groups kg0, kg0 + 1, ... mod nk)

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(p_full + s, 1);
            mbar_init(p_empty + s, F::NIB ? 8 : 5);  // unpack or MMA, and readout warps
        }
        for (int s = 0; s < kI8ASlots; s++) {
            mbar_init(a_full + s, 4);
            mbar_init(a_empty + s, 1);
        }
        for (int s = 0; s < kI8DSlots; s++) {
            mbar_init(d_full + s, 1);
            mbar_init(d_empty + s, 4);
        }
        mbar_init(b_ready, 1);
        mbar_init(mma_done, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tslot, kI8TmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    // Dependents may launch now: every CTA of this grid is resident and holds its TMEM.
    pdl_trigger();

    if (warp == 4) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int t = t0, kg = kg0, ps = 0, rnd = 0;
            for (int i = 0; i < n; i++) {
                if (i >= S) i8_wait(p_empty + ps, (rnd - 1) & 1, abort, a.status);
                int seg, r0;
                if constexpr (kMap == MAP_SWIGLU) {
                    seg = 0;
                    r0 = 64 * t;
                } else {
                    map_row<kMap>(a, 128, 128 * t, seg, r0);
                }
                uint8_t* st = base + P.ring + (size_t)ps * F::STAGE;
                mbar_expect_tx(p_full + ps, (uint32_t)F::STAGE);
                if constexpr (kMap == MAP_SWIGLU) {  // gate rows -> tile rows 0-63, up -> 64-127
#pragma unroll
                    for (int h = 0; h < 2; h++) {
#pragma unroll
                        for (int qb = 0; qb < F::QBOX; qb++)
                            tma_load_2d(st + qb * 16384 + h * 8192, &maps.q[h],
                                        (kg * F::QBOX + qb) * 128, r0, p_full + ps);
                        tma_load_2d(st + F::QB + h * 64 * F::MROW, &maps.m[h], kg * F::MROW, r0,
                                    p_full + ps);
                    }
                } else {
#pragma unroll
                    for (int qb = 0; qb < F::QBOX; qb++)
                        tma_load_2d(st + qb * 16384, &maps.q[seg], (kg * F::QBOX + qb) * 128, r0,
                                    p_full + ps);
                    tma_load_2d(st + F::QB, &maps.m[seg], kg * F::MROW, r0, p_full + ps);
                }
                if (++kg == nk) {
                    kg = 0;
                    t++;
                }
                if (++ps == S) {
                    ps = 0;
                    rnd++;
                }
            }
            // every issued stage lands before the CTA may end (its shared memory is reused)
            ps = n % S;
            rnd = n / S;
            for (int k = 0; k < (n < S ? n : S); k++) {
                if (--ps < 0) {
                    ps = S - 1;
                    rnd--;
                }
                i8_wait(p_full + ps, rnd & 1, abort, a.status);
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            i8_wait(b_ready, 0, abort, a.status);
            const uint32_t bbase = smem_u32(base + P.b);
            // descriptor of B block 0 of B slot 0; +8 per 128-byte block (address >> 4)
            const uint64_t db0 = umma_desc_plain(bbase, 64, 64);
            int kg = kg0, ps = 0, rnd = 0, as = 0, aph = 0, ds = 0, dph = 0;
            for (int h = 0; h < 2 * n; h++) {
                const int i = h >> 1, hh = h & 1;
                if constexpr (F::NIB) {
                    i8_wait(a_full + as, aph, abort, a.status);
                } else {
                    if (hh == 0) i8_wait(p_full + ps, rnd & 1, abort, a.status);
                }
                if (h >= kI8DSlots) i8_wait(d_empty + ds, dph ^ 1, abort, a.status);
                tc_fence_after();
                const int bslot = all_k ? kg : i;
                const uint32_t abase =
                    F::NIB ? smem_u32(base + P.a + (size_t)as * 16384)
                           : smem_u32(base + P.ring + (size_t)ps * F::STAGE + hh * 16384);
                const uint64_t da = umma_desc_sw128(abase);
                const uint64_t db = db0 + (uint64_t)((bslot * 1024 + hh * 512) >> 4);
                const uint32_t td = tmem + (uint32_t)(ds * 64);
#pragma unroll
                for (int j = 0; j < 4; j++)  // A: +32 bytes per block; B: +128 bytes
                    umma_i8(td + (uint32_t)(j * 16), da + (uint64_t)(2 * j), db + (uint64_t)(8 * j));
                umma_commit(d_full + ds);
                if constexpr (F::NIB)
                    umma_commit(a_empty + as);
                else if (hh)
                    umma_commit(p_empty + ps);
                if constexpr (F::NIB) {
                    if (++as == kI8ASlots) {
                        as = 0;
                        aph ^= 1;
                    }
                }
                if (++ds == kI8DSlots) {
                    ds = 0;
                    dph ^= 1;
                }
                if (hh) {
                    if (++kg == nk) kg = 0;
                    if (++ps == S) {
                        ps = 0;
                        rnd++;
                    }
                }
            }
            // every MMA has finished with TMEM and shared memory before the CTA ends
            umma_commit(mma_done);
            if (n > 0) i8_wait(mma_done, 0, abort, a.status);
        }
    } else if (warp >= 6) {
        // ------------------------------------------------------------ nibble unpack
        if constexpr (F::NIB) {
            const int r = tid - 192;
            int ps = 0, rnd = 0, as = 0, aph = 0;
            for (int h = 0; h < 2 * n; h++) {
                const int hh = h & 1;
                if (hh == 0) i8_wait(p_full + ps, rnd & 1, abort, a.status);
                if (h >= kI8ASlots) i8_wait(a_empty + as, aph ^ 1, abort, a.status);
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
                if (++as == kI8ASlots) {
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
        // ------------------------------------------------------------ readout warps 0-3
        const int r = tid;  // tile row = TMEM lane
        pdl_wait();
        if constexpr (EPI == EPI_QKV_ROPE) {
            const int pos = a.position_dev ? *a.position_dev : a.position;
            for (int i = r; i < (a.head_dim >> 1); i += 128)
                rope_tab[i] = rope_pair(a, i, pos);
        }
        if (a.ar_in_n > 0) {  // wait for every rank's partial of this call (bounded)
            if (warp == 0 && lane < a.ar_in_n && *(volatile int*)a.status == SSD_OK) {
                const unsigned long long ep = *a.ar_epoch + (unsigned long long)a.ar_call + 1ull;
                bool done = false;
                for (uint32_t it = 0; it < (1u << 21) && !done; it++) {
                    unsigned long long f;
                    asm volatile("ld.acquire.sys.global.u64 %0, [%1];"
                                 : "=l"(f)
                                 : "l"(a.ar_in_flag + lane)
                                 : "memory");
                    done = f >= ep;
                    if (!done) __nanosleep(100);
                }
                if (!done) atomicExch(a.status, SSD_ERR_TIMEOUT);
            }
            bar_named(1, 128);
        }
        // pass 1: sum of squares of x_eff (RMSNorm) and its write-back by CTA 0; eight
        // loads per thread in flight per round
        float inv = 1.0f;
        const bool wb = a.x_writeback != nullptr && b == 0;
        if (a.norm_w || wb) {
            float ss = 0.0f;
            const int nv = a.cols;
            for (int k0 = r; k0 < nv; k0 += 8 * 128) {
                float v[8];
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const int k = k0 + q * 128;
                    v[q] = k < nv ? x_eff(a, k) : 0.0f;
                }
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const int k = k0 + q * 128;
                    if (wb && k < nv) a.x_writeback[k] = v[q];
                    ss = fmaf(v[q], v[q], ss);
                }
            }
            if (a.norm_w) {
                ss = warp_sum(ss);
                if (lane == 0) red[warp] = ss;
                bar_named(1, 128);
                const float tot = (red[0] + red[1]) + (red[2] + red[3]);
                // inv_rms = 1 / sqrt(sum_sq / n + eps)   (src/metal/compute.rs:583-584)
                inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.cols), a.eps)));
            }
        }
        // pass 2: the limbs of the k-groups this CTA multiplies. Warp w takes blocks w and
        // w + 4 of each k-group, lane = element; the x values of four k-groups are loaded
        // before any is used.
        {
            uint8_t* bb = base + P.b;
            const int nbs = all_k ? nk : n;
            const int kgb = all_k ? 0 : kg0;  // k-group of B slot 0
            // K position of element `lane` in a block: nibble formats lane / 2 (+16 when
            // odd), byte formats lane; limb l at byte (p / 16) * 64 + l * 16 + p % 16
            const int kh = F::NIB ? (lane & 1) : (lane >> 4);
            const int kp = F::NIB ? (lane >> 1) : (lane & 15);
            for (int sl0 = 0; sl0 < nbs; sl0 += 4) {
                float xv[8];
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const int sl = sl0 + (q >> 1), c = warp + 4 * (q & 1);
                    int kgq = kgb + sl;
                    if (kgq >= nk) kgq -= nk;
                    const int k = kgq * 256 + c * 32 + lane;
                    xv[q] = sl < nbs ? x_norm(a, x_eff(a, k), k, inv) : 0.0f;
                }
                uint32_t mx[8];
#pragma unroll
                for (int q = 0; q < 8; q++)
                    mx[q] = __reduce_max_sync(0xffffffffu, __float_as_uint(xv[q]) & 0x7FFFFFFFu);
                float X[8];
#pragma unroll
                for (int q = 0; q < 8; q++) X[q] = 0.0f;
                if constexpr (F::SUMX) {
#pragma unroll
                    for (int q = 0; q < 8; q++) X[q] = xv[q];
#pragma unroll
                    for (int o = 16; o; o >>= 1)
#pragma unroll
                        for (int q = 0; q < 8; q++) X[q] += __shfl_xor_sync(0xffffffffu, X[q], o);
                }
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const int sl = sl0 + (q >> 1), c = warp + 4 * (q & 1);
                    if (sl < nbs) {
                        // e: max|v| 2^e in [2^25, 2^26); all-zero blocks get e = 0
                        const int ex = (int)(mx[q] >> 23);
                        int e = mx[q] == 0 ? 0 : 152 - ex;
                        e = e < -100 ? -100 : (e > 126 ? 126 : e);
                        const float sc = __uint_as_float((uint32_t)(e + 127) << 23);
                        int xf = __float2int_rn(__fmul_rn(xv[q], sc));
                        const int l0 = (int)(int8_t)(xf & 0xFF);
                        xf = (xf - l0) >> 8;
                        const int l1 = (int)(int8_t)(xf & 0xFF);
                        xf = (xf - l1) >> 8;
                        const int l2 = (int)(int8_t)(xf & 0xFF);
                        const int l3 = (xf - l2) >> 8;
                        uint8_t* blk = bb + sl * 1024 + c * 128 + kh * 64 + kp;
                        blk[0] = (uint8_t)l0;
                        blk[16] = (uint8_t)l1;
                        blk[32] = (uint8_t)l2;
                        blk[48] = (uint8_t)l3;
                        if (lane == 0) {
                            // 2^-e (2^-(e+4) for the nibble formats, whose A carries
                            // 16 (q - 8)); a non-finite block makes the row NaN, as the
                            // reference's sum would be
                            const int es = F::NIB ? e + 4 : e;
                            float sx = es <= 126 ? __uint_as_float((uint32_t)(127 - es) << 23)
                                                 : __uint_as_float(1u << (149 - es));
                            if (ex == 0xFF) sx = __int_as_float(0x7FC00000);
                            cstab[sl * 8 + c] = make_float2(sx, X[q]);
                        }
                    }
                }
            }
            fence_proxy_async_smem();
            bar_named(1, 128);
            if (r == 0) mbar_arrive(b_ready);
        }

        // readout: one 4-block half-unit per TMEM slot
        float acc = 0.0f;
        int seg_first = kg0;  // k-group of the current tile segment's first unit
        int t = t0, kg = kg0, ps = 0, rnd = 0, ds = 0, dph = 0;
        uint4 meta0 = make_uint4(0, 0, 0, 0), meta1 = make_uint4(0, 0, 0, 0);
        const uint32_t tl = tmem + ((uint32_t)(32 * warp) << 16);
        for (int h = 0; h < 2 * n; h++) {
            const int i = h >> 1, hh = h & 1;
            if (hh == 0) {
                i8_wait(p_full + ps, rnd & 1, abort, a.status);
                const uint8_t* mrow = base + P.ring + (size_t)ps * F::STAGE + F::QB + r * F::MROW;
                meta0 = *reinterpret_cast<const uint4*>(mrow);
                if constexpr (F::MROW == 32) meta1 = *reinterpret_cast<const uint4*>(mrow + 16);
                __syncwarp();
                if (lane == 0) mbar_arrive(p_empty + ps);
            }
            i8_wait(d_full + ds, dph, abort, a.status);
            tc_fence_after();
            int cv[4][4];
#pragma unroll
            for (int j = 0; j < 4; j++) tmem_ld4(tl + (uint32_t)(ds * 64 + j * 16), cv[j]);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(d_empty + ds);
            if (++ds == kI8DSlots) {
                ds = 0;
                dph ^= 1;
            }
            const float2* cs = cstab + (all_k ? kg : i) * 8 + 4 * hh;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int lo = cv[j][0] + cv[j][1] * 256;
                const int hi = cv[j][2] + cv[j][3] * 256;
                const float tot = fmaf((float)hi, 65536.0f, (float)lo);
                const float2 c2 = cs[j];
                if constexpr (FMT == SSD_TYPE_Q4_0 || FMT == SSD_TYPE_Q8_0) {
                    // f16 d of block 4 hh + j: word (2 hh + j / 2) of meta0, half j & 1
                    const uint32_t mw = hh ? (j < 2 ? meta0.z : meta0.w) : (j < 2 ? meta0.x : meta0.y);
                    const float d = f16_bits_to_f32((uint16_t)((j & 1) ? (mw >> 16) : (mw & 0xFFFF)));
                    acc = fmaf(__fmul_rn(d, c2.x), tot, acc);
                } else if constexpr (FMT == SSD_TYPE_Q8_K) {
                    const uint4 mq = hh ? meta1 : meta0;
                    const uint32_t dw = j == 0 ? mq.x : (j == 1 ? mq.y : (j == 2 ? mq.z : mq.w));
                    acc = fmaf(__fmul_rn(__uint_as_float(dw), c2.x), tot, acc);
                } else {  // Q4_K (A = 16 (q - 8)) / Q5_K (A = q - 128): scale q - min
                    const float d = f16_bits_to_f32((uint16_t)(meta0.x & 0xFFFF));
                    const float dmin = f16_bits_to_f32((uint16_t)(meta0.x >> 16));
                    uint32_t s6, m6;
                    k_scale_min(meta0, 4 * hh + j, s6, m6);
                    const float scale = __fmul_rn(d, (float)s6);
                    const float mn = __fmul_rn(dmin, (float)m6);
                    // sum (scale q - min) x = scale sum (q - o) x + (o scale - min) X
                    const float off = FMT == SSD_TYPE_Q4_K ? 8.0f : 128.0f;
                    acc = fmaf(__fmul_rn(scale, c2.x), tot,
                               fmaf(__fsub_rn(__fmul_rn(off, scale), mn), c2.y, acc));
                }
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
            // end of a tile segment: the CTA's last unit or the tile's last k-group
            if (i != n - 1 && kcur != nk - 1) continue;
            const bool whole = seg_first == 0 && kcur == nk - 1;
            seg_first = 0;
            float res = acc;
            acc = 0.0f;
            bool do_epi = whole;
            if (!whole) {
                // partial rows: slot 0 for the CTA's first tile, 1 for its last. The stores
                // are published by the barrier and one release-acquire atomic per CTA; the
                // last CTA to arrive adds every CTA's partial in CTA order.
                const int slot = tcur == t0 ? 0 : 1;
                a.fix_partial[((size_t)b * 2 + slot) * 128 + r] = res;
                bar_named(1, 128);
                const int bf = owner_of((long long)tcur * nk, G, U);
                const int bl = owner_of((long long)tcur * nk + nk - 1, G, U);
                if (r == 0) {
                    unsigned prev;
                    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                                 : "=r"(prev)
                                 : "l"(a.fix_counter + tcur)
                                 : "memory");
                    const bool last = prev == (unsigned)(bl - bf);
                    if (last) a.fix_counter[tcur] = 0u;  // for the next launch (stream-ordered)
                    flag[0] = last;
                }
                bar_named(1, 128);
                do_epi = flag[0] != 0;
                if (do_epi) {
                    res = 0.0f;
                    for (int bc = bf; bc <= bl; bc++) {
                        const int tf = (int)(((long long)U * bc / G) / nk);
                        res += __ldcg(a.fix_partial + ((size_t)bc * 2 + (tcur == tf ? 0 : 1)) * 128 + r);
                    }
                }
                bar_named(1, 128);  // flag[] is reused by the next segment
            }
            if (!do_epi) continue;
            // ---- epilogue of tile tcur, row r
            if constexpr (EPI == EPI_SWIGLU) {
                red[r] = res;
                bar_named(1, 128);
                const int row = 64 * tcur + r;
                if (r < 64 && row < a.seg_rows[0]) a.y[row] = swiglu(res, red[r + 64]);
                bar_named(1, 128);
            } else if constexpr (EPI == EPI_QKV_ROPE) {
                int seg, lr;
                map_row<kMap>(a, 128, 128 * tcur + r, seg, lr);
                const float other = __shfl_xor_sync(0xffffffffu, res, 1);
                float x0 = (r & 1) ? other : res, x1 = (r & 1) ? res : other;
                if (seg < 2) rope_apply(x0, x1, rope_tab[(lr % a.head_dim) >> 1]);
                float* dst = seg == 0 ? a.y : (seg == 1 ? a.y_k : a.y_v);
                if (128 * tcur + r < a.rows) dst[lr] = (r & 1) ? x1 : x0;
            } else {
                const int row = 128 * tcur + r;
                const bool valid = row < a.rows;
                if constexpr (EPI == EPI_STORE) {
                    if (valid) a.y[row] = res;
                } else if constexpr (EPI == EPI_RESID) {
                    if (valid) a.y[row] = __fadd_rn(a.base[row], res);
                } else if constexpr (EPI == EPI_PEERS) {
                    if (valid)
                        for (int p = 0; p < a.ar_out_n; p++) a.ar_out[p][row] = res;
                } else {  // EPI_ARGMAX
                    unsigned long long key = 0ull;
                    if (valid) {
                        if (a.y) a.y[row] = res;
                        key = argmax_key(res, (uint32_t)(row + a.index_offset));
                    }
#pragma unroll
                    for (int o = 16; o; o >>= 1) {
                        const unsigned long long kk = __shfl_xor_sync(0xffffffffu, key, o);
                        key = kk > key ? kk : key;
                    }
                    if (lane == 0 && key) atomicMax(a.argmax_key, key);
                }
            }
        }
    }

    if constexpr (EPI == EPI_PEERS) {
        peers_publish(a);  // then the last CTA raises the flags on every rank
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kI8TmemCols);
    }
}

// --------------------------------------------------------------- host side

template <int FMT>
static int i8_row_bytes(int cols, uint64_t* qrow, uint64_t* mrow) {
    const int nc = cols / 32;
    *qrow = (uint64_t)nc * (I8Fmt<FMT>::NIB ? 16 : 32);
    *mrow = (uint64_t)nc * (FMT == SSD_TYPE_Q8_K ? 4 : 2);
    return SSD_OK;
}

template <int FMT, int EPI>
static int launch_i8_t(ssd_ctx* ctx, const MvArgs& a, cudaStream_t s, bool pdl) {
    using F = I8Fmt<FMT>;
    constexpr int kMap = epi_map(EPI);
    const int nk = a.cols / 256;
    int n_tiles;
    if (kMap == MAP_SWIGLU)
        n_tiles = a.seg_rows[0] / 64;
    else
        n_tiles = (a.rows + 127) / 128;
    const long long U = (long long)n_tiles * nk;
    int G = ctx->num_sms < kI8MaxGrid ? ctx->num_sms : kI8MaxGrid;
    if (U < G) G = (int)U;
    const int per = (int)((U + G - 1) / G);
    const int nb = per < nk ? per : nk;  // distinct k-groups of one CTA's range
    constexpr bool kRope = EPI == EPI_QKV_ROPE;
    // stages: the whole share when it is small (prefetched before the PDL wait), else a
    // ring deep enough to keep ~100 KB in flight, within the shared-memory opt-in
    int stages = per < kI8MaxStages ? per : kI8MaxStages;
    if (stages < 2) stages = 2;
    while (stages > 2 && i8_plan(F::STAGE, F::NIB, stages, nb, kRope).total > ctx->smem_optin)
        stages--;
    const I8Plan P = i8_plan(F::STAGE, F::NIB, stages, nb, kRope);
    SSD_REQ(P.total <= ctx->smem_optin, SSD_ERR_SHAPE,
            "tensor-core matvec: %zu bytes of shared memory for cols %d", P.total, a.cols);
    I8Work wk{n_tiles, nk, (int)U, stages, nb};
    I8Maps maps;
    memset(&maps, 0, sizeof(maps));
    const int nseg = kMap == MAP_QKV ? 3 : (kMap == MAP_SWIGLU ? 2 : 1);
    const uint32_t BR = kMap == MAP_SWIGLU ? 64 : 128;
    uint64_t qrow, mrow;
    i8_row_bytes<FMT>(a.cols, &qrow, &mrow);
    for (int g = 0; g < nseg; g++) {
        const uint64_t rows = (uint64_t)(kMap == MAP_PLAIN ? a.rows : a.seg_rows[g]);
        SSD_TRY(encode_bytes_map(&maps.q[g], a.qs[g], qrow, rows, 128, BR, true));
        SSD_TRY(encode_bytes_map(&maps.m[g], a.meta[g], mrow, rows, F::MROW, BR, false));
    }
    auto kern = k_mv_i8<FMT, EPI>;
    static bool attr = false;  // per instantiation; the opt-in size is the same on every B200
    if (!attr) {
        SSD_CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)ctx->smem_optin));
        attr = true;
    }
    SSD_CK(launch_pdl(kern, dim3(G), dim3(kI8Threads), P.total, s, pdl, a, wk, maps));
    return SSD_OK;
}

template <int FMT>
static int launch_i8_fmt(ssd_ctx* ctx, int epi, const MvArgs& a, cudaStream_t s, bool pdl) {
    switch (epi) {
        case EPI_STORE: return launch_i8_t<FMT, EPI_STORE>(ctx, a, s, pdl);
        case EPI_RESID: return launch_i8_t<FMT, EPI_RESID>(ctx, a, s, pdl);
        case EPI_SWIGLU: return launch_i8_t<FMT, EPI_SWIGLU>(ctx, a, s, pdl);
        case EPI_QKV_ROPE: return launch_i8_t<FMT, EPI_QKV_ROPE>(ctx, a, s, pdl);
        case EPI_ARGMAX: return launch_i8_t<FMT, EPI_ARGMAX>(ctx, a, s, pdl);
        case EPI_PEERS: return launch_i8_t<FMT, EPI_PEERS>(ctx, a, s, pdl);
        default: return kI8NotCovered;
    }
}

int launch_matvec_i8(ssd_ctx* ctx, int type, int epi, const MvArgs& a, cudaStream_t s, bool pdl) {
    if (!a.fix_counter || !a.fix_partial || a.cols % 256 != 0) return kI8NotCovered;
    if (!(type == SSD_TYPE_Q4_0 || type == SSD_TYPE_Q8_0 || type == SSD_TYPE_Q4_K ||
          type == SSD_TYPE_Q5_K || type == SSD_TYPE_Q8_K))
        return kI8NotCovered;
    const int map = epi_map(epi);
    if (map == MAP_QKV &&
        (a.seg_rows[0] % 128 != 0 || a.seg_rows[1] % 128 != 0 || a.seg_rows[2] % 128 != 0))
        return kI8NotCovered;
    if (map == MAP_SWIGLU && a.seg_rows[0] % 64 != 0) return kI8NotCovered;
    if (epi == EPI_QKV_ROPE && a.head_dim % 2 != 0) return kI8NotCovered;
    switch (type) {
        case SSD_TYPE_Q4_0: return launch_i8_fmt<SSD_TYPE_Q4_0>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q8_0: return launch_i8_fmt<SSD_TYPE_Q8_0>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q4_K: return launch_i8_fmt<SSD_TYPE_Q4_K>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q5_K: return launch_i8_fmt<SSD_TYPE_Q5_K>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q8_K: return launch_i8_fmt<SSD_TYPE_Q8_K>(ctx, epi, a, s, pdl);
        default: return kI8NotCovered;
    }
}

}  // namespace ssd
