// gemm.cuh — tensor-core GEMM for batch prefill (internal interface).
#pragma once
#include "common.cuh"

namespace ssd {

enum GemmEpi { GEMM_STORE = 0, GEMM_RESID = 1, GEMM_SWIGLU = 2 };

// C[m][n] = rscale[n] * sum_k A[m][k] W[n][k] with A and W given as fp16 hi / lo splits
// (row-major, K contiguous). GEMM_RESID adds base[m][n]; GEMM_SWIGLU treats each 128-wide
// tile as 64 gate columns followed by the 64 up columns of the same outputs and writes
// silu(gate) * up to C[m][n0/2 + j] (ldc = N / 2). M, N multiples of 128, K of 128.
struct GemmArgs {
    int M, N, K;
    float* C;
    int ldc;
    const float* base;
    int ldb;
    const float* rscale;
    int epi;
    int* status;
    // GEMM_SWIGLU only: when set, the outputs are written as fp16 hi / lo splits
    // (hi = fp16(y), lo = fp16(y - hi), the A-operand form of the next GEMM, ld = ldc)
    // instead of fp32 C (C may then be null).
    __half* c_hi;
    __half* c_lo;
};
struct GemmOperands {
    const __half* a_hi;
    const __half* a_lo;
    const __half* w_hi;
    const __half* w_lo;
};

// Weight -> fp16 hi / lo rows with power-of-two row scales (rscale = 1 / scale).
// map_mode 0 places row r at dst0 + r; map_mode 1 places row r of segment seg (0 gate,
// 1 up) at (r / half) * 2 half + seg half + r % half.
int prepare_weight_split(ssd_ctx* ctx, const ssd_weight* w, int map_mode, int half_tile, int seg,
                         int dst0, __half* hi, __half* lo, float* rscale, cudaStream_t s);
// Activations [M][K] f32 -> fp16 hi / lo, with an optional per-row RMSNorm first.
int prepare_act_split(const float* x, int M, int K, const float* norm_w, float eps, int norm_order,
                      __half* hi, __half* lo, cudaStream_t s, bool pdl);
int launch_gemm(ssd_ctx* ctx, const GemmOperands& op, GemmArgs g, cudaStream_t s, bool pdl);

}  // namespace ssd
