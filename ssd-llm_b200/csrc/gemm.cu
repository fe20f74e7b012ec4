// gemm.cu — tensor-core GEMMs for layer-major batch prefill (sm_100a, tcgen05 + TMEM).
//
// Replaces the per-token matvecs of batch_prefill_lora (src/inference/transformer.rs:120-250:
// for each layer, for each of the n prompt tokens, the same matvec_quantized calls as
// forward_pass) by one GEMM per weight: C[m][n] = sum_k A[m][k] W[n][k] over the M prompt
// tokens.
//
// Precision. The reference computes these products in fp32; the parity bar (1e-3 relative
// with a floor of 1e-3 of the vector's max) needs about 20 correct bits, more than one
// fp16 or bf16 pass gives. Each operand is split into fp16 hi + lo parts (x = hi + lo,
// lo = fp16(x - hi), ~22 bits together) and the GEMM runs three passes into one fp32 TMEM
// accumulator: A_hi W_hi + A_hi W_lo + A_lo W_hi (the dropped A_lo W_lo term is ~2^-22 of a
// product). Weight rows are pre-scaled by a power of two so that every lo part is a normal
// fp16; the epilogue multiplies by the inverse.
//
// Kernel (one CTA of 6 warps per 128 x 128 output tile, one CTA per SM):
//  * warp 4, one thread: TMA producer — per 64-wide K step, four tiles (A hi/lo, W hi/lo, 128 x 64
//    fp16, 128-byte swizzle) into a stage of the shared-memory ring;
//  * warp 5, one thread: MMA issuer — waits for the stage, issues 3 passes x 4 tcgen05.mma
//    (kind::f16, M = N = 128, K = 16) into one of two TMEM accumulators, and
//    tcgen05.commit releases the stage back to the producer;
//  * warps 0-3: every 128 K, tcgen05.ld the finished window (warp w owns TMEM lanes
//    32w..32w+31 = tile rows) and add it into fp32 registers (the tensor core's own fp32
//    accumulation truncates at each MMA; windows keep that drift ~2^-21), then scale,
//    residual / SwiGLU, store.
// Every mbarrier wait is bounded; a timeout is recorded in the status word, the kernel
// drains what it issued, frees its TMEM and returns.
#include "common.cuh"
#include "gemm.cuh"
#include "umma.cuh"

namespace ssd {

// Tile 128 x 128; 3 ring stages of 64-wide K steps (A hi/lo + W hi/lo, 64 KB each).
// Two-level accumulation: the tensor core's fp32 accumulation truncates at every MMA, so
// each window of kWin K steps (128 K) accumulates into one of two TMEM buffers and the
// epilogue warps add the finished window into fp32 registers (round to nearest) while
// the MMA thread fills the other buffer.
constexpr int kGemmBN = 128;
struct GemmSmem {
    static constexpr int kStages = 3;
    static constexpr int kWin = 2;       // K steps (of 64) per accumulation window
    static constexpr int kA = 128 * 128;  // one 128 x 64 fp16 tile
    static constexpr int kStage = 4 * kA;
    static constexpr int kBar = kStages * kStage;
    static constexpr int kTotal = kBar + 256 + 1024;
    static constexpr int kTmemCols = 2 * kGemmBN;
};

constexpr int kGemmThreads = 192;  // warps 0-3 epilogue (TMEM lanes), 4 TMA, 5 MMA

template <int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm_f16x3(const GemmArgs g, const __grid_constant__ CUtensorMap tm_ah,
                 const __grid_constant__ CUtensorMap tm_al, const __grid_constant__ CUtensorMap tm_bh,
                 const __grid_constant__ CUtensorMap tm_bl) {
    using SM = GemmSmem;
    constexpr int S = SM::kStages, BN = kGemmBN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + SM::kBar);
    uint64_t* empty = full + S;
    uint64_t* acc_full = empty + S;  // [2]: window accumulated in TMEM buffer b
    uint64_t* acc_free = acc_full + 2;  // [2]: buffer b drained by the 4 epilogue warps
    uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_free + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // blockIdx.x = M tile (fastest): the M / 128 CTAs that read one weight tile are launched
    // together, so the weights stream from HBM once and the other reads hit L2
    const int m0 = blockIdx.x * 128, n0 = blockIdx.y * BN;
    const int KB = g.K / 64, NW = KB / SM::kWin;

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_free + b, 4);
        }
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tslot, SM::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_wait();

    bool ok = true;
    if (tid == 128) {  // ---- TMA producer (warp 4)
        for (int kb = 0; kb < KB && ok; kb++) {
            const int s = kb % S;
            if (kb >= S) ok = mbar_wait(empty + s, ((kb / S) - 1) & 1, g.status);
            if (!ok) break;
            uint8_t* st = base + (size_t)s * SM::kStage;
            mbar_expect_tx(full + s, (uint32_t)SM::kStage);
            tma_load_2d(st, &tm_ah, kb * 64, m0, full + s);
            tma_load_2d(st + SM::kA, &tm_al, kb * 64, m0, full + s);
            tma_load_2d(st + 2 * SM::kA, &tm_bh, kb * 64, n0, full + s);
            tma_load_2d(st + 3 * SM::kA, &tm_bl, kb * 64, n0, full + s);
        }
    } else if (tid == 160) {  // ---- MMA issuer (warp 5)
        constexpr uint32_t idesc = umma_idesc_f16(128, BN);
        for (int kb = 0; kb < KB && ok; kb++) {
            const int w = kb / SM::kWin, b = w & 1, first = (kb % SM::kWin) == 0;
            if (first && w >= 2) ok = mbar_wait(acc_free + b, ((w >> 1) - 1) & 1, g.status);
            const int s = kb % S;
            if (ok) ok = mbar_wait(full + s, (kb / S) & 1, g.status);
            if (!ok) break;
            tc_fence_after();
            const uint32_t st = smem_u32(base + (size_t)s * SM::kStage);
            const uint32_t ah = st, al = st + SM::kA, bh = st + 2 * SM::kA, bl = st + 3 * SM::kA;
            const uint32_t acc = tmem + (uint32_t)(b * BN);
#pragma unroll
            for (int pass = 0; pass < 3; pass++) {  // hi*hi, hi*lo, lo*hi
                const uint32_t a = pass == 2 ? al : ah, bb = pass == 1 ? bl : bh;
#pragma unroll
                for (int k = 0; k < 4; k++)  // K = 16 per MMA: 32 bytes along the row
                    umma_f16(acc, umma_desc_sw128(a + 32 * k), umma_desc_sw128(bb + 32 * k), idesc,
                             (first && pass == 0 && k == 0) ? 0u : 1u);
            }
            umma_commit(empty + s);  // stage free once these MMAs have read it
            if ((kb % SM::kWin) == SM::kWin - 1) umma_commit(acc_full + b);
        }
    }
    __syncwarp();
    // ---- epilogue warps 0-3: drain each window into fp32 registers (warp w: tile rows
    // 32w .. 32w+31, its TMEM lanes)
    float sum[BN];
#pragma unroll
    for (int j = 0; j < BN; j++) sum[j] = 0.0f;
    const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    bool acc_ok = true;
    for (int w = 0; w < NW && acc_ok && warp < 4; w++) {
        const int b = w & 1;
        acc_ok = mbar_wait(acc_full + b, (w >> 1) & 1, g.status);
        if (!acc_ok) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < BN / 32; c++) {
            uint32_t v[32];
            tmem_ld32(tl + (uint32_t)(b * BN) + 32 * c, v);
#pragma unroll
            for (int j = 0; j < 32; j++) sum[32 * c + j] = __fadd_rn(sum[32 * c + j], __uint_as_float(v[j]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_free + b);
    }
    if (__syncthreads_and(ok && acc_ok) && warp < 4) {
        const int row = m0 + 32 * warp + lane;
        if constexpr (EPI == GEMM_SWIGLU) {  // tile columns [0, 64) gate, [64, 128) up
            constexpr int H = BN / 2;
            const size_t o0 = (size_t)row * g.ldc + (n0 / 2);
#pragma unroll
            for (int j = 0; j < H; j += 4) {
                float4 o;
                float* op = &o.x;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const float gt = __fmul_rn(sum[j + t], g.rscale[n0 + j + t]);
                    const float up = __fmul_rn(sum[H + j + t], g.rscale[n0 + H + j + t]);
                    // silu(v) = v / (1 + exp(-v)), then gate *= up (feed_forward.rs:31-39)
                    op[t] = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up);
                }
                if (g.c_hi) {  // the down GEMM's A operand, split as k_asplit splits it
                    __align__(8) __half h[4], l[4];
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        h[t] = __float2half_rn(op[t]);
                        l[t] = __float2half_rn(op[t] - __half2float(h[t]));
                    }
                    *reinterpret_cast<uint2*>(g.c_hi + o0 + j) = *reinterpret_cast<const uint2*>(h);
                    *reinterpret_cast<uint2*>(g.c_lo + o0 + j) = *reinterpret_cast<const uint2*>(l);
                } else {
                    *reinterpret_cast<float4*>(g.C + o0 + j) = o;
                }
            }
        } else {
            float* out = g.C + (size_t)row * g.ldc + n0;
            const float* bs = EPI == GEMM_RESID ? g.base + (size_t)row * g.ldb + n0 : nullptr;
#pragma unroll
            for (int j = 0; j < BN; j += 4) {
                float4 o;
                float* op = &o.x;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    float y = __fmul_rn(sum[j + t], g.rscale[n0 + j + t]);
                    if constexpr (EPI == GEMM_RESID) y = __fadd_rn(bs[j + t], y);
                    op[t] = y;
                }
                *reinterpret_cast<float4*>(out + j) = o;
            }
        }
    }
    pdl_trigger();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, SM::kTmemCols);
    }
}

// ------------------------------------------------------- operand preparation
// Weight row -> fp16 hi / lo rows, scaled by a power of two s_n chosen from the row's
// largest magnitude so that hi*2^-11 (the lo part) stays a normal fp16; rscale[dst] = 1/s_n.
// dst row = row_map(src row): plain, or the SwiGLU tiling (gate rows and up rows of the same
// output columns side by side in one BN-wide tile).
__global__ void __launch_bounds__(256) k_wsplit(const ssd_weight w, int map_mode, int half_tile,
                                                int seg, int dst0, __half* hi, __half* lo,
                                                float* rscale) {
    __shared__ float red[8];
    const int r = blockIdx.x, K = w.cols;
    int dst = dst0 + r;
    if (map_mode == 1) dst = (r / half_tile) * 2 * half_tile + seg * half_tile + (r % half_tile);
    float mx = 0.0f;
    for (int e = threadIdx.x * 8; e < K; e += 256 * 8) {
        float v[8];
        dequant8(w, (int64_t)r * K + e, v);
        for (int t = 0; t < 8; t++) mx = fmaxf(mx, fabsf(v[t]));
    }
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = 0.0f;
    for (int i = 0; i < 8; i++) mx = fmaxf(mx, red[i]);
    // s = 2^(14 - e) with mx in [2^e, 2^(e+1)): scaled magnitudes below 2^15 (fp16 max 65504)
    int e = 0;
    frexpf(mx, &e);  // mx = f * 2^e, f in [0.5, 1)
    const int sh = mx > 0.0f ? min(max(15 - e, -100), 100) : 0;
    const float s = ldexpf(1.0f, sh);
    for (int e0 = threadIdx.x * 8; e0 < K; e0 += 256 * 8) {
        float v[8];
        dequant8(w, (int64_t)r * K + e0, v);
        __half h[8], l[8];
        for (int t = 0; t < 8; t++) {
            const float x = v[t] * s;  // exact: power of two
            h[t] = __float2half_rn(x);
            l[t] = __float2half_rn(x - __half2float(h[t]));
        }
        *reinterpret_cast<uint4*>(hi + (size_t)dst * K + e0) = *reinterpret_cast<const uint4*>(h);
        *reinterpret_cast<uint4*>(lo + (size_t)dst * K + e0) = *reinterpret_cast<const uint4*>(l);
    }
    if (threadIdx.x == 0) rscale[dst] = ldexpf(1.0f, -sh);
}

// Activation rows (f32 [M][K]) -> fp16 hi / lo, optionally RMSNorm'd first (per row:
// order 0 x * (inv_rms * w), order 1 (x * inv_rms) * w, src/metal/compute.rs:580-588).
__global__ void __launch_bounds__(256) k_asplit(const float* x, int K, const float* norm_w,
                                                float eps, int norm_order, __half* hi, __half* lo) {
    __shared__ float red[8];
    const int r = blockIdx.x;
    const float* xr = x + (size_t)r * K;
    pdl_wait();
    float inv = 1.0f;
    if (norm_w) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < K; i += 256) ss = fmaf(xr[i], xr[i], ss);
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        float tot = 0.0f;
        for (int i = 0; i < 8; i++) tot += red[i];
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), eps)));
    }
    for (int i = threadIdx.x; i < K; i += 256) {
        float v = xr[i];
        if (norm_w)
            v = norm_order == 0 ? __fmul_rn(v, __fmul_rn(inv, norm_w[i]))
                                : __fmul_rn(__fmul_rn(v, inv), norm_w[i]);
        const __half h = __float2half_rn(v);
        hi[(size_t)r * K + i] = h;
        lo[(size_t)r * K + i] = __float2half_rn(v - __half2float(h));
    }
}

// fp16 [rows][K] tensor map: box 64 x box_rows, 128-byte swizzle (the UMMA K-major layout).
static int encode_f16_map(CUtensorMap* map, const __half* ptr, int rows, int K, int box_rows) {
    using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeFn fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        SSD_CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q));
        SSD_REQ(f != nullptr && q == cudaDriverEntryPointSuccess, SSD_ERR_CUDA,
                "cuTensorMapEncodeTiled unavailable");
        fn = (EncodeFn)f;
    }
    SSD_REQ(((uintptr_t)ptr & 15u) == 0 && K % 64 == 0, SSD_ERR_ARG, "f16 map alignment");
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)ptr, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    SSD_REQ(r == CUDA_SUCCESS, SSD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SSD_OK;
}

int prepare_weight_split(ssd_ctx* ctx, const ssd_weight* w, int map_mode, int half_tile, int seg,
                         int dst0, __half* hi, __half* lo, float* rscale, cudaStream_t s) {
    SSD_REQ(w->cols % 64 == 0, SSD_ERR_SHAPE, "prefill GEMM needs K %% 64 == 0 (K = %d)", w->cols);
    k_wsplit<<<w->rows, 256, 0, s>>>(*w, map_mode, half_tile, seg, dst0, hi, lo, rscale);
    SSD_CK_LAUNCH();
    (void)ctx;
    return SSD_OK;
}

int prepare_act_split(const float* x, int M, int K, const float* norm_w, float eps, int norm_order,
                      __half* hi, __half* lo, cudaStream_t s, bool pdl) {
    SSD_CK(launch_pdl(k_asplit, dim3(M), dim3(256), 0, s, pdl, x, K, norm_w, eps, norm_order, hi,
                      lo));
    return SSD_OK;
}

template <int EPI>
static int launch_gemm_t(ssd_ctx* ctx, const GemmOperands& op, const GemmArgs& g, cudaStream_t s,
                         bool pdl) {
    using SM = GemmSmem;
    auto kern = k_gemm_f16x3<EPI>;
    static bool attr = false;  // per instantiation; the opt-in size is the same on every B200
    SSD_REQ((size_t)SM::kTotal <= ctx->smem_optin, SSD_ERR_SHAPE, "GEMM stage ring too large");
    if (!attr) {
        SSD_CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::kTotal));
        attr = true;
    }
    CUtensorMap mah, mal, mbh, mbl;
    SSD_TRY(encode_f16_map(&mah, op.a_hi, g.M, g.K, 128));
    SSD_TRY(encode_f16_map(&mal, op.a_lo, g.M, g.K, 128));
    SSD_TRY(encode_f16_map(&mbh, op.w_hi, g.N, g.K, kGemmBN));
    SSD_TRY(encode_f16_map(&mbl, op.w_lo, g.N, g.K, kGemmBN));
    SSD_CK(launch_pdl(kern, dim3(g.M / 128, g.N / kGemmBN), dim3(kGemmThreads), SM::kTotal, s, pdl,
                      g, mah, mal, mbh, mbl));
    return SSD_OK;
}

int launch_gemm(ssd_ctx* ctx, const GemmOperands& op, GemmArgs g, cudaStream_t s, bool pdl) {
    if (!g.status) g.status = ctx->dev_status;
    SSD_REQ(g.M > 0 && g.M % 128 == 0, SSD_ERR_SHAPE, "GEMM M %d not a multiple of 128", g.M);
    SSD_REQ(g.K > 0 && g.K % (64 * GemmSmem::kWin) == 0, SSD_ERR_SHAPE,
            "GEMM K %d not a multiple of %d", g.K, 64 * GemmSmem::kWin);
    SSD_REQ(g.N > 0 && g.N % kGemmBN == 0, SSD_ERR_SHAPE, "GEMM N %d not a multiple of %d", g.N,
            kGemmBN);
    SSD_REQ((g.C || (g.epi == GEMM_SWIGLU && g.c_hi && g.c_lo)) && g.rscale && op.a_hi && op.a_lo &&
                op.w_hi && op.w_lo,
            SSD_ERR_ARG, "null GEMM operand");
    SSD_REQ(!g.c_hi || (g.epi == GEMM_SWIGLU && g.c_lo && g.ldc % 4 == 0), SSD_ERR_ARG,
            "fp16 split output needs the SwiGLU epilogue and ldc a multiple of 4");
    SSD_REQ(g.epi != GEMM_RESID || g.base, SSD_ERR_ARG, "null residual base");
    if (g.epi == GEMM_STORE) return launch_gemm_t<GEMM_STORE>(ctx, op, g, s, pdl);
    if (g.epi == GEMM_RESID) return launch_gemm_t<GEMM_RESID>(ctx, op, g, s, pdl);
    if (g.epi == GEMM_SWIGLU) return launch_gemm_t<GEMM_SWIGLU>(ctx, op, g, s, pdl);
    set_error("GEMM epilogue %d", g.epi);
    return SSD_ERR_ARG;
}

}  // namespace ssd

using namespace ssd;

// ==================================================================== C ABI
extern "C" int ssd_prefill_matmul(ssd_ctx* ctx, const ssd_weight* w, const float* x_dev, int n_tokens,
                                  float* y_dev, void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(w && x_dev && y_dev, SSD_ERR_ARG, "null argument");
    SSD_REQ(w->type == SSD_TYPE_Q4_0 || w->type == SSD_TYPE_Q8_0 || w->type == SSD_TYPE_Q4_K ||
                w->type == SSD_TYPE_Q5_K || w->type == SSD_TYPE_Q6_K || w->type == SSD_TYPE_Q8_K ||
                w->type == SSD_TYPE_F32,
            SSD_ERR_TYPE, "prefill matmul: ggml type %d not supported", w->type);
    SSD_REQ(n_tokens > 0 && n_tokens % 128 == 0, SSD_ERR_SHAPE,
            "n_tokens %d must be a positive multiple of 128", n_tokens);
    SSD_REQ(w->cols % 128 == 0 && w->rows % 128 == 0, SSD_ERR_SHAPE,
            "weight %dx%d: rows and cols must be multiples of 128", w->rows, w->cols);
    cudaStream_t s = pick_stream(ctx, stream);
    const size_t M = n_tokens, N = w->rows, K = w->cols;
    const size_t need = (2 * N * K + 2 * M * K) * 2 + N * 4 + 4096;
    SSD_TRY(ensure_scratch(ctx, need));
    __half* whi = (__half*)ctx->scratch;
    __half* wlo = whi + N * K;
    __half* ahi = wlo + N * K;
    __half* alo = ahi + M * K;
    float* rs = (float*)(alo + M * K);
    SSD_TRY(prepare_weight_split(ctx, w, 0, 0, 0, 0, whi, wlo, rs, s));
    SSD_TRY(prepare_act_split(x_dev, (int)M, (int)K, nullptr, 0.0f, 0, ahi, alo, s, false));
    GemmOperands op{ahi, alo, whi, wlo};
    GemmArgs g = {};
    g.M = (int)M;
    g.N = (int)N;
    g.K = (int)K;
    g.C = y_dev;
    g.ldc = (int)N;
    g.rscale = rs;
    g.epi = GEMM_STORE;
    return launch_gemm(ctx, op, g, s, false);
}
