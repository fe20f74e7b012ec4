// matvec_tc.cu — fused dequant-matvec (Q4_0 / Q8_0 / Q4_K) on the integer tensor cores,
// fed by a TMA + mbarrier pipeline.
//
// Same operator as matvec.cu (matvec_quantized, src/metal/compute.rs:157-191, :680-750,
// :904-925) with the same prologue and epilogues; it differs in how the weights are
// streamed and how the dot products are formed. The FMA kernel spends ~3 instructions
// per weight (decode + FMA + x reads) and is issue-bound at two thirds of HBM
// bandwidth; here the products run on mma.sync.m16n8k32 (8-bit integer inputs, exact
// 32-bit integer sums), about one instruction per weight.
//
// Arithmetic:
//  * Weights are the exact integers of the block format: a Q4_0 / Q4_K word gives its
//    8 nibbles as two A fragments with one AND each (w & 0x0F0F0F0F: 4 low nibbles;
//    w & 0xF0F0F0F0: 4 high nibbles times 16), a Q8_0 word is an A fragment as it is.
//  * x is made exact fixed point per 32-element chunk: xf = rint(x * 2^e), e chosen so
//    that max |x| * 2^e lies in [2^25, 2^26) (every x within 8x of the chunk maximum
//    converts exactly, smaller ones keep 26 bits below the maximum), and xf is split into
//    four signed bytes ("limbs", xf = sum_j 256^j l_j). Low-nibble positions carry the
//    limbs of 16 * xf so that both nibble halves share the scale 16.
//  * One MMA multiplies a 16-row tile by a block-diagonal B: lane quad t (lanes with
//    lane % 4 == t) owns chunk t of a group of 4 chunks, and columns 2t, 2t+1 of B hold
//    two limbs of that chunk's x, so the accumulator of lane (g, t) collects
//    sum_k q * limb for rows g and g+8 of its own chunk. Two MMAs (limb pairs 0,1 and
//    2,3) per 8 elements; the four limb sums recombine exactly in 32-bit integers
//    (lo = C0 + 256 C1, hi = C2 + 256 C3) and once in fp32 (hi * 65536 + lo).
//  * Offsets are integers too: Q4_0's (q - 8) is folded in by starting the
//    accumulators at -128 * sum(xf) (split into 16-bit halves); Q4_K subtracts
//    min * X per sub-block as the FMA kernel does.
//  * Each chunk's sum is scaled once per (row, chunk): y += (d * 2^-e) * D.
//
// Streaming: virtual rows form units of 8; CTA b (one per SM) takes a contiguous,
// balanced range of units and walks it as 16-row tiles. A tile's K is streamed in
// stages of 64 chunks per row (1 KB of Q4_0 per row, contiguous in HBM): a producer
// warp issues, per 8-row half, one TMA box of the slab (a 3-D view of the rows as
// 128-byte blocks, landing as [block][row][128 B] with the 128-byte swizzle) plus one box
// of the chunk scales (Q4_K: super-block headers) into a ring of
// kStages stages, completing on the stage's "full" mbarrier; the first stages are issued
// before griddepcontrol.wait, so they overlap the previous kernel. The 16 consumer warps
// all work on the same stage, warp w on chunks 4w..4w+3, and release it through the
// stage's "empty" mbarrier. At a tile's end the warps' partial rows meet in shared
// memory (one named barrier) and one warp adds them in warp order (deterministic) and
// runs the epilogue while the others go on with the next tile.
#include <cstring>

#include "matvec_dev.cuh"

namespace ssd {

constexpr int kTcNW = 16;                      // consumer warps
constexpr int kTcThreads = (kTcNW + 1) * 32;   // + one producer warp
constexpr int kTcMaxStages = 12;

// Stage geometry for a slab of SLAB chunks per row: NBOX payload blocks and MBOX scale
// blocks of 128 bytes per row; stage = [half h][NBOX payload, MBOX scale blocks][8 rows]
// [128 B]; each consumer warp takes U = SLAB / 64 groups of 4 chunks.
template <int FMT, int SLAB>
struct TcFmt {
    static constexpr int QB = FMT == SSD_TYPE_Q8_0 ? 32 : 16;  // payload bytes per (row, chunk)
    static constexpr int NBOX = SLAB * QB / 128;
    static constexpr int MBOX = SLAB * 2 / 128;  // f16 d per chunk, or 16 B per 8 chunks
    static constexpr int HB = (NBOX + MBOX) * 1024;  // bytes of one half
    static constexpr int SB = 2 * HB;
    static constexpr int U = SLAB / 64;
};

struct TcPlan {
    int nc, xrows;
    size_t xs, cst, red, keys, bars, abort, rope, parts, ring, total;
};
__host__ __device__ inline TcPlan tc_plan(int cols, int stages, int stage_bytes) {
    TcPlan p;
    p.nc = cols >> 5;
    p.xrows = (p.nc + kVecBoxRows - 1) / kVecBoxRows * kVecBoxRows;
    size_t o = 0;
    p.xs = o;
    o += (size_t)p.xrows * 128;
    p.cst = o;
    o += (size_t)p.nc * 16;
    p.red = o;
    o += 32 * 4;
    p.keys = o;
    o += 32 * 8;
    p.bars = o;  // full[stages], empty[stages], the x barrier
    o += (size_t)(2 * kTcMaxStages + 2) * 8;
    p.abort = o;
    o += 16;
    p.rope = o;
    o += (size_t)kMaxRopePairs * 8;
    p.parts = o;  // [2 buffers][kTcNW warps][16 rows]
    o += 2 * kTcNW * 16 * 4;
    o = (o + 1023) & ~(size_t)1023;
    p.ring = o;
    o += (size_t)stages * stage_bytes;
    p.total = o + 1024;  // alignment slack
    return p;
}

struct TcMaps {
    CUtensorMap q[3];  // payload rows of each segment
    CUtensorMap m[3];  // f16 scales (Q4_K: super-block headers) of each segment
};

// C (4 x s32) += A (16x32, 8-bit, row) * B (32x8, s8, col)
template <bool ASIGNED>
__device__ __forceinline__ void imma(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                     uint32_t b0, uint32_t b1) {
    if constexpr (ASIGNED)
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};"
            : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else
        asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};"
            : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t wsel(const uint4& q, int m) {
    return m == 0 ? q.x : (m == 1 ? q.y : (m == 2 ? q.z : q.w));
}

// Named barrier of the consumer warps only (the producer warp keeps streaming).
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kTcNW * 32) : "memory");
}

template <int FMT, int EPI, int SLAB>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_matvec_tc(const MvArgs a, const __grid_constant__ CUtensorMap tm_x,
                const __grid_constant__ TcMaps maps, int n_units, int stages) {
    constexpr int NW = kTcNW;
    using F = TcFmt<FMT, SLAB>;
    constexpr int QB = F::QB, NBOX = F::NBOX, MBOX = F::MBOX, HB = F::HB, SB = F::SB, U = F::U;
    constexpr bool kQ8 = FMT == SSD_TYPE_Q8_0;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const TcPlan P = tc_plan(a.cols, stages, SB);
    uint8_t* xs = base + P.xs;
    int4* cst = reinterpret_cast<int4*>(base + P.cst);
    float* red = reinterpret_cast<float*>(base + P.red);
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(base + P.keys);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + P.bars);
    uint64_t* empty = full + kTcMaxStages;
    uint64_t* xbar = full + 2 * kTcMaxStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(base + P.abort);
    float2* rope_tab = reinterpret_cast<float2*>(base + P.rope);
    float* parts = reinterpret_cast<float*>(base + P.parts);
    uint8_t* ring = base + P.ring;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int nc = P.nc, spr = (nc + SLAB - 1) / SLAB;
    // this CTA's units [ub, ue) (SWIGLU: whole 16-row gate/up groups)
    int ub, ue;
    if (a.map == MAP_SWIGLU) {
        const int np = n_units >> 1;
        ub = 2 * (int)((long long)blockIdx.x * np / gridDim.x);
        ue = 2 * (int)((long long)(blockIdx.x + 1) * np / gridDim.x);
    } else {
        ub = (int)((long long)blockIdx.x * n_units / gridDim.x);
        ue = (int)((long long)(blockIdx.x + 1) * n_units / gridDim.x);
    }
    const int n_t = (ue - ub + 1) >> 1;
    const int vend = min(8 * ue, a.rows);  // end of this CTA's virtual rows
    const int T = n_t * spr;               // stages of this CTA

    if (tid == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        mbar_init(xbar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // ---- producer warp: stage k = (tile k / spr, K slab k % spr) into slot k % stages.
    // Lane 0 arms the stage's full barrier, then every lane issues one box (payload boxes
    // of both halves, then the two scale boxes), so a stage's boxes go out together.
    const bool producer = warp == NW;
    int pk = 0, pslot = 0, pphase = 0;  // next stage to issue, its slot and round parity
    auto issue_stage = [&]() {
        const int j = pk / spr, sl = pk - j * spr;
        const int vb = 8 * (ub + 2 * j);
        const int nh = vb + 8 < vend ? 2 : 1;
        uint8_t* st = ring + (size_t)pslot * SB;
        // per half: one box of NBOX 128-byte blocks x 8 rows (the slab; blocks past the
        // row end read as zero) and MBOX 128-byte x 8-row boxes of scales
        if (lane == 0) mbar_expect_tx(&full[pslot], (uint32_t)(nh * HB));
        __syncwarp();
        if (lane < nh * (1 + MBOX)) {
            const int h = lane / (1 + MBOX), b = lane - h * (1 + MBOX);
            int seg, lr;
            map_row(a, 16, vb + 8 * h, seg, lr);
            uint8_t* hb = st + (size_t)h * HB;
            if (b == 0)
                tma_load_3d(hb, &maps.q[seg], 0, lr, sl * NBOX, &full[pslot]);
            else
                tma_load_2d(hb + (NBOX + b - 1) * 1024, &maps.m[seg], sl * SLAB * 2 + (b - 1) * 128,
                            lr, &full[pslot]);
        }
        pk++;
        if (++pslot == stages) {
            pslot = 0;
            pphase ^= 1;
        }
    };
    // Weights never depend on the previous kernel: fill the ring before waiting.
    if (producer)
        while (pk < T && pk < stages) issue_stage();

    // ---- prologue: x -> per-chunk fixed point, split into limbs, in place.
    // Unit u of chunk c (elements 4u..4u+3) belongs to word wi = u >> 1, half h = u & 1.
    // Chunk c's 128 bytes become [slot wi ^ (c & 3)][parity e][p0.b0 p0.b1 p1.b0 p1.b1]:
    // the B registers of lane (g, t) with g & 1 == e for word wi of chunk c (limbs e and
    // 2 + e; b0 = the low-nibble (Q8_0: first four) elements, b1 = the others).
    auto finish = [&](int i, int c, int ph, float4 v, unsigned gmask) {
        (void)ph;
        const int u = i & 7, wi = u >> 1, h = u & 1;
        // chunk maximum of |x| as bits (NaN / Inf sort above every finite value)
        const uint32_t ubits = __reduce_max_sync(
            gmask, max(max(__float_as_uint(v.x) & 0x7FFFFFFFu, __float_as_uint(v.y) & 0x7FFFFFFFu),
                       max(__float_as_uint(v.z) & 0x7FFFFFFFu, __float_as_uint(v.w) & 0x7FFFFFFFu)));
        const bool finite = ubits < 0x7F800000u;
        int e = 0;
        if (finite && ubits != 0u) e = 25 - max((int)(ubits >> 23) - 127, -100);  // e in [-102, 125]
        const float two_e = __uint_as_float((uint32_t)(127 + e) << 23);
        int xf[4] = {0, 0, 0, 0};  // |xf| <= 2^26 - 4, so a chunk's sum fits in 32 bits
        if (finite) {
            xf[0] = __float2int_rn(__fmul_rn(v.x, two_e));
            xf[1] = __float2int_rn(__fmul_rn(v.y, two_e));
            xf[2] = __float2int_rn(__fmul_rn(v.z, two_e));
            xf[3] = __float2int_rn(__fmul_rn(v.w, two_e));
        }
        const int xsum = __reduce_add_sync(gmask, xf[0] + xf[1] + xf[2] + xf[3]);
        // limbs of each value packed as bytes [l0 l1 l2 l3]: with w = v + 0x808080, the
        // low three bytes of w minus 128 (= byte ^ 0x80) and the top byte of w
        uint32_t p[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int val = (!kQ8 && (k & 1) == 0) ? xf[k] * 16 : xf[k];  // low nibbles: 16 x
            p[k] = (uint32_t)(val + 0x808080) ^ 0x00808080u;
        }
        // transpose to one word per limb j: nibble formats [b0 half | b1 half] =
        // [p0.j p2.j p1.j p3.j]; Q8_0 [p0.j p1.j p2.j p3.j] (the 4 bytes of b_h)
        const uint32_t pa = kQ8 ? p[1] : p[2], pb = kQ8 ? p[2] : p[1];
        const uint32_t t0l = __byte_perm(p[0], pa, 0x5140), t0h = __byte_perm(p[0], pa, 0x7362);
        const uint32_t t1l = __byte_perm(pb, p[3], 0x5140), t1h = __byte_perm(pb, p[3], 0x7362);
        uint32_t own[4];
        own[0] = __byte_perm(t0l, t1l, 0x5410);
        own[1] = __byte_perm(t0l, t1l, 0x7632);
        own[2] = __byte_perm(t0h, t1h, 0x5410);
        own[3] = __byte_perm(t0h, t1h, 0x7632);
        // partner (the other half of the word) gets the limbs of its parity 1 - h
        const uint32_t s0 = h ? own[0] : own[1], s1 = h ? own[2] : own[3];
        const uint32_t r0 = __shfl_xor_sync(gmask, s0, 1), r1 = __shfl_xor_sync(gmask, s1, 1);
        const uint32_t m0 = h ? own[1] : own[0], m1 = h ? own[3] : own[2];  // my parity's limbs
        uint4 o;
        if constexpr (kQ8) {  // b_h is mine, b_{1-h} the partner's
            o.x = h ? r0 : m0;
            o.y = h ? m0 : r0;
            o.z = h ? r1 : m1;
            o.w = h ? m1 : r1;
        } else {  // each b register: half 0 from h = 0, half 1 from h = 1
            const uint32_t lo0 = h ? r0 : m0, hi0 = h ? m0 : r0;
            const uint32_t lo1 = h ? r1 : m1, hi1 = h ? m1 : r1;
            o.x = __byte_perm(lo0, hi0, 0x5410);  // b0 of limb e: lo halves
            o.y = __byte_perm(lo0, hi0, 0x7632);  // b1 of limb e: hi halves
            o.z = __byte_perm(lo1, hi1, 0x5410);
            o.w = __byte_perm(lo1, hi1, 0x7632);
        }
        __syncwarp(gmask);  // every unit of the chunk has been read
        *reinterpret_cast<uint4*>(xs + (size_t)c * 128 + 32 * (wi ^ (c & 3)) + 16 * h) = o;
        if (u == 0) {
            const float s = finite ? ldexpf(1.0f, -e - (kQ8 ? 0 : 4)) : __uint_as_float(0x7FC00000u);
            int4 k;
            k.x = __float_as_int(s);
            k.y = 0;
            k.z = 0;
            k.w = 0;
            if constexpr (FMT == SSD_TYPE_Q4_0) {  // accumulators start at -128 sum(xf)
                const long long A = 128ll * xsum;
                const long long Ah = (A + 32768) >> 16;
                k.y = -(int)(A - (Ah << 16));
                k.z = -(int)Ah;
            } else if constexpr (FMT == SSD_TYPE_Q4_K) {  // X = sum of the chunk's x
                k.w = __float_as_int(finite ? __fmul_rn((float)xsum, ldexpf(1.0f, -e))
                                            : __uint_as_float(0x7FC00000u));
            }
            cst[c] = k;
        }
    };
    if (!mv_prologue<kTcThreads, EPI>(a, &tm_x, xs, nc, P.xrows, red, xbar, rope_tab, finish))
        *abort_flag = 1;

    unsigned long long best = 0ull;
    if (warp < NW) {
        // ---- consumers: warp w takes chunks 64u + 4w .. 64u + 4w + 3 of every stage
        constexpr int QP = QB / 16;
        const bool bact = (g >> 1) == t;
        const int cl = 4 * warp + t;  // this lane quad's chunk within a group of 64
        // lane-constant shared-memory offsets; group u of a stage adds compile-time deltas
        int poff[QP];  // payload: 16-byte part p of chunk cl, row g (swizzled by g)
#pragma unroll
        for (int p = 0; p < QP; p++) {
            const int ob = cl * QB + 16 * p;
            poff[p] = (ob >> 7) * 1024 + g * 128 + ((((ob >> 4) & 7) ^ g) << 4);
        }
        // scales: byte 2c of the slab's scale row (Q4_K: header 16 (c / 8)), c = 64u + cl
        const int moff = NBOX * 1024 + g * 128 + ((((cl >> 3) & 7) ^ g) << 4) +
                         (FMT == SSD_TYPE_Q4_K ? 0 : ((2 * cl) & 15));
        const uint8_t* xsl = xs + (size_t)cl * 128 + 16 * (g & 1);
        int bx[4];  // word i of the chunk's limbs: slot i ^ t
#pragma unroll
        for (int i = 0; i < 4; i++) bx[i] = 32 * (i ^ t);
        uint4 bz[2];  // B fragments, double-buffered over the 4 words; inactive lanes keep 0
        bz[0] = make_uint4(0u, 0u, 0u, 0u);
        bz[1] = bz[0];
        float acc0 = 0.0f, acc8 = 0.0f;
        int slot = 0, phase = 0, j = 0, sl = 0;
        for (int k = 0; k < T; k++) {
            if (!*abort_flag && !mbar_wait(&full[slot], phase, a.status)) *abort_flag = 1;
            const int nch = min(SLAB, nc - sl * SLAB);
            const uint8_t* st = ring + (size_t)slot * SB;
            const int4* kcp = cst + sl * SLAB + cl;
            const uint8_t* xsp = xsl + (size_t)sl * SLAB * 128;
#pragma unroll
            for (int u = 0; u < U; u++) {
                if (64 * u + 4 * warp >= nch) continue;  // past the row end
                const int4 kc = kcp[64 * u];
                const uint8_t* sq = st + u * (64 * QB / 128) * 1024;
                uint4 w0[QP], w8[QP];
#pragma unroll
                for (int p = 0; p < QP; p++) {
                    w0[p] = *reinterpret_cast<const uint4*>(sq + poff[p]);
                    w8[p] = *reinterpret_cast<const uint4*>(sq + HB + poff[p]);
                }
                const uint8_t* sm = st + moff + u * 1024;
                uint4 hm0, hm8;  // Q4_K: super-block headers of rows g, g + 8
                float d0 = 0.0f, d8 = 0.0f;
                if constexpr (FMT == SSD_TYPE_Q4_K) {
                    hm0 = *reinterpret_cast<const uint4*>(sm);
                    hm8 = *reinterpret_cast<const uint4*>(sm + HB);
                } else {
                    d0 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sm));
                    d8 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sm + HB));
                }
                int C0[4] = {kc.y, 0, kc.y, 0}, C1[4] = {kc.z, 0, kc.z, 0};
                const uint8_t* xb = xsp + u * 64 * 128;
                if (bact) bz[0] = *reinterpret_cast<const uint4*>(xb + bx[0]);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    if (i < 3 && bact) bz[(i + 1) & 1] = *reinterpret_cast<const uint4*>(xb + bx[i + 1]);
                    uint32_t a0, a1, a2, a3;
                    if constexpr (kQ8) {  // words 2i, 2i+1 of the row's 32 bytes
                        a0 = wsel(w0[i >> 1], (2 * i) & 3);
                        a2 = wsel(w0[i >> 1], (2 * i + 1) & 3);
                        a1 = wsel(w8[i >> 1], (2 * i) & 3);
                        a3 = wsel(w8[i >> 1], (2 * i + 1) & 3);
                    } else {
                        const uint32_t x0 = wsel(w0[0], i), x8 = wsel(w8[0], i);
                        a0 = x0 & 0x0F0F0F0Fu;
                        a1 = x8 & 0x0F0F0F0Fu;
                        a2 = x0 & 0xF0F0F0F0u;
                        a3 = x8 & 0xF0F0F0F0u;
                    }
                    const uint4 b = bz[i & 1];
                    imma<kQ8>(C0, a0, a1, a2, a3, b.x, b.y);
                    imma<kQ8>(C1, a0, a1, a2, a3, b.z, b.w);
                }
                const float D0 = fmaf((float)(C1[1] * 256 + C1[0]), 65536.0f, (float)(C0[1] * 256 + C0[0]));
                const float D8 = fmaf((float)(C1[3] * 256 + C1[2]), 65536.0f, (float)(C0[3] * 256 + C0[2]));
                const float s = __int_as_float(kc.x);
                if constexpr (FMT == SSD_TYPE_Q4_K) {
                    // sub-block (64u + 4w + t) & 7 = 4 (w & 1) + t of its super-block
                    const float X = __int_as_float(kc.w);
                    const bool lo_sb = (warp & 1) == 0;
                    auto sub = [&](const uint4& m, float D, float& acc) {
                        const float d = f16_bits_to_f32((uint16_t)(m.x & 0xFFFF));
                        const float dmin = f16_bits_to_f32((uint16_t)(m.x >> 16));
                        const int sh = 8 * t;
                        const uint32_t b0 = (m.y >> sh) & 0xFF, b4 = (m.z >> sh) & 0xFF,
                                       b8 = (m.w >> sh) & 0xFF;
                        uint32_t s6, m6;  // src/metal/compute.rs:725-733
                        if (lo_sb) {
                            s6 = b0 & 0x3F;
                            m6 = b4 & 0x3F;
                        } else {
                            s6 = (b0 >> 6) | ((b8 & 0x0F) << 2);
                            m6 = (b4 >> 6) | ((b8 >> 4) << 2);
                        }
                        // sum((scale*q - min) x) = scale * sum(q x) - min * X
                        const float scale = __fmul_rn(d, (float)s6);
                        const float mn = __fmul_rn(dmin, (float)m6);
                        acc = fmaf(-mn, X, fmaf(__fmul_rn(scale, s), D, acc));
                    };
                    sub(hm0, D0, acc0);
                    sub(hm8, D8, acc8);
                } else {
                    acc0 = fmaf(__fmul_rn(d0, s), D0, acc0);
                    acc8 = fmaf(__fmul_rn(d8, s), D8, acc8);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);  // this warp is done with the stage
            if (++slot == stages) {
                slot = 0;
                phase ^= 1;
            }
            if (++sl != spr) continue;
            // ---- tile j done: park this warp's rows, meet, one warp finishes the tile
            sl = 0;
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
            acc8 += __shfl_xor_sync(0xffffffffu, acc8, 1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
            acc8 += __shfl_xor_sync(0xffffffffu, acc8, 2);
            float* pb = parts + (j & 1) * NW * 16;
            if (t == 0) pb[warp * 16 + g] = acc0;
            if (t == 1) pb[warp * 16 + 8 + g] = acc8;
            acc0 = 0.0f;
            acc8 = 0.0f;
            consumer_sync();
            if (warp == j % NW) {
                // rows g, g + 8 summed over the 16 warps: lane t adds warps 4t..4t+3, then a
                // fixed tree over t
                float r0 = 0.0f, r8 = 0.0f;
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    r0 += pb[(4 * t + w) * 16 + g];
                    r8 += pb[(4 * t + w) * 16 + 8 + g];
                }
                r0 += __shfl_xor_sync(0xffffffffu, r0, 1);
                r8 += __shfl_xor_sync(0xffffffffu, r8, 1);
                r0 += __shfl_xor_sync(0xffffffffu, r0, 2);
                r8 += __shfl_xor_sync(0xffffffffu, r8, 2);
                const int vb = 8 * (ub + 2 * j);
                const int va = vb + g, v8r = vb + 8 + g;
                const bool ok0 = va < vend, ok8 = v8r < vend;
                if constexpr (EPI == EPI_STORE || EPI == EPI_RESID) {
                    if (t == 0 && ok0) a.y[va] = (EPI == EPI_RESID) ? __fadd_rn(a.base[va], r0) : r0;
                    if (t == 1 && ok8) a.y[v8r] = (EPI == EPI_RESID) ? __fadd_rn(a.base[v8r], r8) : r8;
                } else if constexpr (EPI == EPI_PEERS) {  // partial rows -> every rank's buffer
                    for (int p = t; p < a.ar_out_n; p += 4) {
                        if (ok0) a.ar_out[p][va] = r0;
                        if (ok8) a.ar_out[p][v8r] = r8;
                    }
                } else if constexpr (EPI == EPI_SWIGLU) {  // row g: gate, row g+8: the matching up
                    if (t == 0 && ok0) a.y[(vb >> 4) * 8 + g] = swiglu(r0, r8);
                } else if constexpr (EPI == EPI_QKV_ROPE) {  // pairs (2p, 2p+1) = lanes g, g^1
                    const float p0 = __shfl_xor_sync(0xffffffffu, r0, 4);
                    const float p8 = __shfl_xor_sync(0xffffffffu, r8, 4);
                    if ((t == 0 && ok0) || (t == 1 && ok8)) {
                        const int v = t == 0 ? va : v8r;
                        const float mine = t == 0 ? r0 : r8, other = t == 0 ? p0 : p8;
                        int seg, lr;
                        map_row(a, 16, v, seg, lr);
                        const bool even = (g & 1) == 0;
                        float x0 = even ? mine : other, x1 = even ? other : mine;
                        if (seg < 2) rope_apply(x0, x1, rope_tab[(lr % a.head_dim) >> 1]);
                        float* dst = seg == 0 ? a.y : (seg == 1 ? a.y_k : a.y_v);
                        dst[lr] = even ? x0 : x1;
                    }
                } else {  // EPI_ARGMAX
                    if ((t == 0 && ok0) || (t == 1 && ok8)) {
                        const int v = t == 0 ? va : v8r;
                        const float val = t == 0 ? r0 : r8;
                        if (a.y) a.y[v] = val;
                        const unsigned long long kk = argmax_key(val, (uint32_t)(v + a.index_offset));
                        best = kk > best ? kk : best;
                    }
                }
            }
            j++;
        }
    } else if (producer) {
        // ---- the rest of the stages, each once its slot's previous stage is released
        while (pk < T) {
            int ok = 1;
            if (lane == 0) ok = !*abort_flag && mbar_wait(&empty[pslot], pphase ^ 1, a.status);
            if (!__shfl_sync(0xffffffffu, ok, 0)) {
                if (lane == 0) *abort_flag = 1;
                break;
            }
            issue_stage();
        }
        // nothing may land in shared memory after the CTA exits: wait (bounded) for the
        // copies of the last `stages` issued stages if a wait gave up on the way
        if (lane == 0 && *abort_flag) {
            int s = pslot, ph = pphase;
            for (int n = 0; n < min(pk, stages); n++) {
                if (--s < 0) {
                    s = stages - 1;
                    ph ^= 1;
                }
                mbar_wait(&full[s], ph, nullptr);
            }
        }
    }

    if constexpr (EPI == EPI_PEERS) {
        peers_publish(a);  // then the last CTA raises the flags on every rank
    }
    if constexpr (EPI == EPI_ARGMAX) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0) keys[warp] = best;
        __syncthreads();
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int w = 0; w <= NW; w++) b = keys[w] > b ? keys[w] : b;
            if (b) atomicMax(a.argmax_key, b);
        }
    }
}

// --------------------------------------------------------------- host side

template <int FMT, int EPI, int SLAB>
static int launch_tc_slab(ssd_ctx* ctx, const MvArgs& a, cudaStream_t s, bool pdl) {
    using F = TcFmt<FMT, SLAB>;
    const int n_units = (a.rows + 7) / 8;
    int G = ctx->num_sms;
    if (a.map == MAP_SWIGLU)
        G = min(G, n_units / 2);
    else
        G = min(G, n_units);
    const size_t fixed = tc_plan(a.cols, 0, F::SB).total;
    if (fixed >= ctx->smem_optin) return kTcNotCovered;
    const size_t fit = (ctx->smem_optin - fixed) / F::SB;
    if (fit < 3) return kTcNotCovered;
    const int stages = fit < (size_t)kTcMaxStages ? (int)fit : kTcMaxStages;
    const TcPlan P = tc_plan(a.cols, stages, F::SB);
    const int nseg = a.map == MAP_PLAIN ? 1 : (a.map == MAP_SWIGLU ? 2 : 3);
    const uint64_t nc = (uint64_t)(a.cols >> 5);
    TcMaps maps;
    memset(&maps, 0, sizeof maps);
    for (int i = 0; i < nseg; i++) {  // payload rows of nc * QB bytes, scale rows of nc * 2
        SSD_TRY(encode_blocks_map(&maps.q[i], a.qs[i], nc * F::QB, (uint64_t)a.seg_rows[i], 8,
                                  F::NBOX));
        SSD_TRY(encode_rows_map(&maps.m[i], a.meta[i], nc * 2, (uint64_t)a.seg_rows[i], 8));
    }
    auto kern = k_matvec_tc<FMT, EPI, SLAB>;
    int nb = 0;
    SSD_TRY(occupancy(ctx, kern, kTcThreads, P.total, &nb));
    CUtensorMap mx;
    SSD_TRY(encode_vec_map(&mx, a.x, a.cols));
    SSD_CK(launch_pdl(kern, dim3(G), dim3(kTcThreads), P.total, s, pdl, a, mx, maps, n_units, stages));
    return SSD_OK;
}

// Slab of 128 chunks (2 KB of Q4_0 per row per stage) when three such stages fit beside
// x in shared memory, else 64; Q8_0 (32-byte chunks) always 64.
template <int FMT, int EPI>
static int launch_tc_fe(ssd_ctx* ctx, const MvArgs& a, cudaStream_t s, bool pdl) {
    if constexpr (FMT != SSD_TYPE_Q8_0) {
        const int st = launch_tc_slab<FMT, EPI, 128>(ctx, a, s, pdl);
        if (st != kTcNotCovered) return st;
    }
    return launch_tc_slab<FMT, EPI, 64>(ctx, a, s, pdl);
}

template <int FMT>
static int launch_tc_f(ssd_ctx* ctx, int epi, const MvArgs& a, cudaStream_t s, bool pdl) {
    switch (epi) {
        case EPI_STORE: return launch_tc_fe<FMT, EPI_STORE>(ctx, a, s, pdl);
        case EPI_RESID: return launch_tc_fe<FMT, EPI_RESID>(ctx, a, s, pdl);
        case EPI_SWIGLU: return launch_tc_fe<FMT, EPI_SWIGLU>(ctx, a, s, pdl);
        case EPI_QKV_ROPE: return launch_tc_fe<FMT, EPI_QKV_ROPE>(ctx, a, s, pdl);
        case EPI_ARGMAX: return launch_tc_fe<FMT, EPI_ARGMAX>(ctx, a, s, pdl);
        case EPI_PEERS: return launch_tc_fe<FMT, EPI_PEERS>(ctx, a, s, pdl);
        default: return kTcNotCovered;
    }
}

// Shapes covered: cols a multiple of 256 and at least 2048 (the scale rows of one stage
// are one 128-byte TMA box; Q4_K needs 256 anyway), every segment at least 8 rows with
// 8-row aligned boundaries (a TMA box never straddles two tensors), SwiGLU gate rows a
// multiple of 8. Everything else, and any shape whose x staging leaves room for fewer
// than 3 stages, stays on the FMA kernel.
int launch_matvec_tc(ssd_ctx* ctx, int type, int epi, const MvArgs& a, cudaStream_t s, bool pdl) {
    if (a.cols % 256 != 0 || a.cols < 2048) return kTcNotCovered;
    const int nseg = a.map == MAP_PLAIN ? 1 : (a.map == MAP_SWIGLU ? 2 : 3);
    for (int i = 0; i < nseg; i++)
        if (a.seg_rows[i] < 8 || (i < nseg - 1 && a.seg_rows[i] % 8 != 0)) return kTcNotCovered;
    if (a.map == MAP_SWIGLU && a.seg_rows[0] % 8 != 0) return kTcNotCovered;
    if (a.map == MAP_PLAIN && a.seg_rows[0] != a.rows) return kTcNotCovered;
    for (int i = 0; i < nseg; i++)
        if (((uintptr_t)a.qs[i] | (uintptr_t)a.meta[i]) & 15u) return kTcNotCovered;
    switch (type) {
        case SSD_TYPE_Q4_0: return launch_tc_f<SSD_TYPE_Q4_0>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q8_0: return launch_tc_f<SSD_TYPE_Q8_0>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q4_K: return launch_tc_f<SSD_TYPE_Q4_K>(ctx, epi, a, s, pdl);
        default: return kTcNotCovered;
    }
}

}  // namespace ssd
