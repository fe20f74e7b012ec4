// attn_tc.cu — causal attention of a prompt batch on the tcgen05 tensor cores.
//
// Replaces the per-token attention of batch_prefill_lora (src/inference/transformer.rs:
// 120-250, each prompt token through multi_head_attention_fused_rope, attention.rs:172-240,
// flash_attention.rs:40-143 over the INT8 cache, quantized_kv_cache.rs:118-130): query i of
// the batch (absolute position pos0 + i) attends to positions 0 .. pos0 + i with the scores
// (q . k) * k_scale / sqrt(d) and the online softmax, exactly the reference's math, as a
// dense contraction.
//
// One CTA of 8 warps per (tile of 128 queries, query head); thread r < 128 owns query row r
// of the tile (TMEM lane r: softmax, output columns 0-63), thread 128 + r the same row's
// output columns 64-127. Per key block of 128 positions:
//  * the block's INT8 K rows and V rows are dequantized exactly (|q| <= 127 is exact in
//    fp16) into shared memory as K-major 128-byte-swizzled tiles: K [key][dim], V
//    transposed [dim][key] (8 x 8 micro-tiles transposed in registers);
//  * one thread issues S = Q_hi K^T + Q_lo K^T (tcgen05.mma kind::f16, M = N = 128, fp32
//    in TMEM): Q is split into fp16 hi + lo parts (~22 bits), K is exact, so the scores are
//    fp32-accurate; the K scale and 1/sqrt(d) are applied per column afterwards;
//  * each thread reads its row of S back (tcgen05.ld), masks keys past its own position,
//    and runs the online softmax in registers (lazy rescaling: the running maximum moves
//    only when a score exceeds it by more than 8, which keeps every weight <= e^8); the
//    weights times the V scale are split into fp16 hi + lo rows of P;
//  * one thread issues O_blk = P_hi V + P_lo V into TMEM; every thread adds its row of
//    O_blk into 64 fp32 registers (no long accumulation inside the tensor core).
// The output is O / l. Every mbarrier wait is bounded (status SSD_ERR_TIMEOUT); the CTA
// frees its TMEM before it returns.
#include "common.cuh"
#include "ops.cuh"
#include "umma.cuh"

namespace ssd {

constexpr int kAtTq = 128;                 // queries per CTA
constexpr int kAtHD = 128;                 // head_dim
constexpr int kAtSub = 128 * 128;          // one 128-row x 64-element fp16 sub-tile (16 KB)
constexpr int kAtTile = 2 * kAtSub;        // 128 x 128 fp16 as two K sub-tiles
// shared memory (from a 1024-byte aligned base): Q hi, Q lo, K, V^T, P hi, P lo tiles, then
// the block's K / V scales, two mbarriers and the TMEM address slot
constexpr int kAtQH = 0, kAtQL = kAtTile, kAtK = 2 * kAtTile, kAtV = 3 * kAtTile,
              kAtPH = 4 * kAtTile, kAtPL = 5 * kAtTile, kAtSc = 6 * kAtTile;
constexpr int kAtBar = kAtSc + 2 * 128 * 4;
constexpr int kAtSmem = kAtBar + 64 + 1024;

// Byte offset of element (row, col) of a 128 x 128 fp16 tile stored as two K-major
// 128-byte-swizzled sub-tiles (cols 0-63, 64-127): 16-byte unit u of row r at u ^ (r & 7).
__device__ __forceinline__ int at_off(int row, int col) {
    const int sub = col >> 6, c = col & 63;
    return sub * kAtSub + row * 128 + ((((c >> 3) ^ row) & 7) << 4) + ((c & 7) << 1);
}

// Eight floats -> eight fp16 (hi) and their remainders (lo), as two 16-byte units.
__device__ __forceinline__ void split8(const float (&v)[8], uint4& hi, uint4& lo) {
    __half h[8], l[8];
#pragma unroll
    for (int t = 0; t < 8; t++) {
        h[t] = __float2half_rn(v[t]);
        l[t] = __float2half_rn(v[t] - __half2float(h[t]));
    }
    hi = *reinterpret_cast<const uint4*>(h);
    lo = *reinterpret_cast<const uint4*>(l);
}

__global__ void __launch_bounds__(256, 1) k_attn_prefill_tc(const AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    float* ksc = reinterpret_cast<float*>(base + kAtSc);
    float* vsc = ksc + 128;
    __shared__ float pmax_s[8];
    __shared__ float corr_s[128];  // per row: rescale of the running output this block
    __shared__ float linv_s[128];  // per row: 1 / l at the end
    uint64_t* s_bar = reinterpret_cast<uint64_t*>(base + kAtBar);
    uint64_t* o_bar = s_bar + 1;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(s_bar + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // threads 0-127 own query row r (softmax, output columns 0-63); threads 128-255 the same
    // rows' output columns 64-127 (a warp reaches TMEM lanes 32 (warp % 4) ..)
    const int r = tid & 127, half = tid >> 7;
    const int qt = blockIdx.x, h = blockIdx.y;
    const int g_kv = a.kv_head0 + h / a.group;

    if (tid == 0) {
        mbar_init(s_bar, 1);
        mbar_init(o_bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tslot, 256);  // S: columns 0-127, O_blk: 128-255
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);  // this warp's TMEM lanes
    pdl_wait();

    // ---- Q row r, dims 64 half .. (a power-of-two pre-scale per row keeps every lo part a
    // normal fp16; both halves of the row agree on it through the row maximum)
    const int qi = qt * kAtTq + r, qpos = a.seq0 + qi;
    const float* qrow = a.q + (size_t)qi * a.q_stride + (size_t)h * kAtHD;
    float qmax = 0.0f;
    for (int d = 0; d < kAtHD; d += 4) {
        const float4 v = *reinterpret_cast<const float4*>(qrow + d);
        qmax = fmaxf(qmax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    int qe = 0;
    frexpf(qmax, &qe);
    const int qsh = qmax > 0.0f ? min(max(14 - qe, -100), 100) : 0;
    const float qs = ldexpf(1.0f, qsh);
    for (int d = 64 * half; d < 64 * half + 64; d += 8) {
        float v[8];
#pragma unroll
        for (int t = 0; t < 8; t++) v[t] = qrow[d + t] * qs;  // exact: power of two
        uint4 hi, lo;
        split8(v, hi, lo);
        *reinterpret_cast<uint4*>(base + kAtQH + at_off(r, d)) = hi;
        *reinterpret_cast<uint4*>(base + kAtQL + at_off(r, d)) = lo;
    }
    // score = (q . k) * k_scale * (1 / sqrt(d)); the pre-scale is undone here
    const float cfac = __fmul_rn(__fdiv_rn(1.0f, __fsqrt_rn((float)kAtHD)), ldexpf(1.0f, -qsh));

    float o[64];  // output columns 64 half .. 64 half + 63 of row r
#pragma unroll
    for (int d = 0; d < 64; d++) o[d] = 0.0f;
    float l = 0.0f, mu = -INFINITY;  // (row threads) running weight sum, maximum in use
    const int kend = a.seq0 + qt * kAtTq + kAtTq;  // keys of this tile: [0, kend)
    const int nkb = (kend + 127) / 128;
    constexpr uint32_t idesc = umma_idesc_f16(128, 128);
    bool ok = true;
    for (int kb = 0; kb < nkb && ok; kb++) {
        const int key0 = kb * 128;
        // ---- K row key0 + r, dims 64 half .., exact fp16; scales
        {
            const int key = min(key0 + r, kend - 1);  // rows past kend are masked below
            const int8_t* kr = a.k + (size_t)key * a.kv_dim + (size_t)g_kv * kAtHD;
#pragma unroll
            for (int d = 64 * half; d < 64 * half + 64; d += 16) {
                const uint4 w = *reinterpret_cast<const uint4*>(kr + d);
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int hl = 0; hl < 2; hl++) {
                    __half e[8];
#pragma unroll
                    for (int t = 0; t < 8; t++)
                        e[t] = __int2half_rn((int)(int8_t)(ws[2 * hl + t / 4] >> (8 * (t & 3))));
                    *reinterpret_cast<uint4*>(base + kAtK + at_off(r, d + 8 * hl)) =
                        *reinterpret_cast<const uint4*>(e);
                }
            }
            if (half == 0) {
                ksc[r] = a.ks[key];
                vsc[r] = a.vs[key];
            }
            // the block's largest V scale sets a power of two that keeps the P rows
            // (weights up to e^8 times the V scale) in fp16's normal range
            const float vm = warp_max(fabsf(a.vs[key]));
            if (lane == 0) pmax_s[warp] = vm;
        }
        // ---- V^T: one 8 x 8 micro-tile (keys 8kg.., dims 8dg..) per thread
        {
            const int kg = tid & 15, dg = tid >> 4;
            uint2 row8[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int key = min(key0 + 8 * kg + i, kend - 1);
                row8[i] = *reinterpret_cast<const uint2*>(a.v + (size_t)key * a.kv_dim +
                                                          (size_t)g_kv * kAtHD + 8 * dg);
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {  // dim 8dg + j: the 8 keys' values
                __half e[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const uint32_t w = j < 4 ? row8[i].x : row8[i].y;
                    e[i] = __int2half_rn((int)(int8_t)(w >> (8 * (j & 3))));
                }
                *reinterpret_cast<uint4*>(base + kAtV + at_off(8 * dg + j, 8 * kg)) =
                    *reinterpret_cast<const uint4*>(e);
            }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        int pe = 0;
        frexpf(fmaxf(fmaxf(fmaxf(pmax_s[0], pmax_s[1]), fmaxf(pmax_s[2], pmax_s[3])),
                     fmaxf(fmaxf(pmax_s[4], pmax_s[5]), fmaxf(pmax_s[6], pmax_s[7]))),
               &pe);
        const int psh = min(max(-pe, -100), 100);
        const float pscale = ldexpf(1.0f, psh), pinv = ldexpf(1.0f, -psh);
        // ---- S = Q_hi K^T + Q_lo K^T
        if (tid == 0) {
            const uint32_t qh = smem_u32(base + kAtQH), ql = smem_u32(base + kAtQL);
            const uint32_t kk = smem_u32(base + kAtK);
#pragma unroll
            for (int pass = 0; pass < 2; pass++)
#pragma unroll
                for (int sub = 0; sub < 2; sub++)
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        umma_f16(tmem, umma_desc_sw128((pass ? ql : qh) + sub * kAtSub + 32 * k),
                                 umma_desc_sw128(kk + sub * kAtSub + 32 * k), idesc,
                                 (pass | sub | k) ? 1u : 0u);
            umma_commit(s_bar);
        }
        ok = mbar_wait(s_bar, kb & 1, a.status);
        if (!__syncthreads_and(ok)) break;
        tc_fence_after();
        if (half == 0) {
            // ---- scores of row r: block maximum, then the weights (lazy rescaling)
            float mb = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                uint32_t v[32];
                tmem_ld32(tl + 32 * c, v);
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    const float sc = __fmul_rn(__fmul_rn(__uint_as_float(v[j]), ksc[32 * c + j]), cfac);
                    if (key0 + 32 * c + j <= qpos) mb = fmaxf(mb, sc);
                }
            }
            float corr = 1.0f;
            if (mb > mu + 8.0f || mu == -INFINITY) {  // move the maximum in use
                corr = mu == -INFINITY ? 0.0f : expf(__fsub_rn(mu, mb));
                l = __fmul_rn(l, corr);
                mu = mb;
            }
            corr_s[r] = corr;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                uint32_t v[32];
                tmem_ld32(tl + 32 * c, v);
#pragma unroll
                for (int j8 = 0; j8 < 32; j8 += 8) {
                    float p8[8];
#pragma unroll
                    for (int t = 0; t < 8; t++) {
                        const int kc = 32 * c + j8 + t;
                        const float sc = __fmul_rn(__fmul_rn(__uint_as_float(v[j8 + t]), ksc[kc]), cfac);
                        const float p = key0 + kc <= qpos ? expf(__fsub_rn(sc, mu)) : 0.0f;
                        l = __fadd_rn(l, p);
                        p8[t] = __fmul_rn(__fmul_rn(p, vsc[kc]), pscale);  // V scale on the weight
                    }
                    uint4 hi, lo;
                    split8(p8, hi, lo);
                    *reinterpret_cast<uint4*>(base + kAtPH + at_off(r, 32 * c + j8)) = hi;
                    *reinterpret_cast<uint4*>(base + kAtPL + at_off(r, 32 * c + j8)) = lo;
                }
            }
            fence_proxy_async_smem();
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- O_blk = P_hi V + P_lo V  (A = P [query][key], B = V^T [dim][key])
        if (tid == 0) {
            const uint32_t ph = smem_u32(base + kAtPH), pl = smem_u32(base + kAtPL);
            const uint32_t vv = smem_u32(base + kAtV);
#pragma unroll
            for (int pass = 0; pass < 2; pass++)
#pragma unroll
                for (int sub = 0; sub < 2; sub++)
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        umma_f16(tmem + 128, umma_desc_sw128((pass ? pl : ph) + sub * kAtSub + 32 * k),
                                 umma_desc_sw128(vv + sub * kAtSub + 32 * k), idesc,
                                 (pass | sub | k) ? 1u : 0u);
            umma_commit(o_bar);
        }
        const float corr = corr_s[r];
#pragma unroll
        for (int d = 0; d < 64; d++) o[d] = __fmul_rn(o[d], corr);
        ok = mbar_wait(o_bar, kb & 1, a.status);
        if (!__syncthreads_and(ok)) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; c++) {
            uint32_t v[32];
            tmem_ld32(tl + 128 + 64 * half + 32 * c, v);
#pragma unroll
            for (int j = 0; j < 32; j++)
                o[32 * c + j] = fmaf(__uint_as_float(v[j]), pinv, o[32 * c + j]);  // exact scale
        }
        tc_fence_before();
        __syncthreads();  // S, O_blk and the tiles are free for the next block
        tc_fence_after();
    }
    if (ok) {
        // output_acc / running_sum (flash_attention.rs:126-133); l > 0: the query's own
        // position is always attended
        if (half == 0) linv_s[r] = __fdiv_rn(1.0f, l);
        __syncthreads();
        const float inv = linv_s[r];
        const size_t o0 = (size_t)qi * a.out_stride + (size_t)h * kAtHD + 64 * half;
        if (a.out_hi) {  // the output projection's A operand, split as k_asplit splits it
#pragma unroll
            for (int d = 0; d < 64; d += 4) {
                __align__(8) __half hh[4], ll[4];
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const float v = __fmul_rn(o[d + t], inv);
                    hh[t] = __float2half_rn(v);
                    ll[t] = __float2half_rn(v - __half2float(hh[t]));
                }
                *reinterpret_cast<uint2*>(a.out_hi + o0 + d) = *reinterpret_cast<const uint2*>(hh);
                *reinterpret_cast<uint2*>(a.out_lo + o0 + d) = *reinterpret_cast<const uint2*>(ll);
            }
        } else {
            float* orow = a.out + o0;
#pragma unroll
            for (int d = 0; d < 64; d += 4)
                *reinterpret_cast<float4*>(orow + d) =
                    make_float4(__fmul_rn(o[d], inv), __fmul_rn(o[d + 1], inv),
                                __fmul_rn(o[d + 2], inv), __fmul_rn(o[d + 3], inv));
        }
    }
    pdl_trigger();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

int launch_attention_prefill_tc(ssd_ctx* ctx, const AttnArgs& a, cudaStream_t s, bool pdl) {
    SSD_REQ(a.head_dim == kAtHD && a.n_q > 0 && a.n_q % kAtTq == 0 && a.k_new == nullptr,
            SSD_ERR_SHAPE, "tensor-core prefill attention: head_dim 128, queries a multiple of 128");
    SSD_REQ(a.q_stride % 4 == 0 && a.out_stride % 4 == 0 && a.kv_dim % 16 == 0, SSD_ERR_SHAPE,
            "tensor-core prefill attention: 16-byte aligned rows");
    AttnArgs b = a;
    if (!b.status) b.status = ctx->dev_status;
    static bool attr = false;
    if (!attr) {
        SSD_CK(cudaFuncSetAttribute(k_attn_prefill_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kAtSmem));
        attr = true;
    }
    SSD_CK(launch_pdl(k_attn_prefill_tc, dim3(a.n_q / kAtTq, a.n_kv_local * a.group), dim3(256),
                      kAtSmem, s, pdl, b));
    return SSD_OK;
}

}  // namespace ssd
