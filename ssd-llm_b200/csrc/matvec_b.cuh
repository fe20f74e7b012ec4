// matvec_b.cuh — batched (continuous-batch decode) dequant-matvec (internal interface).
#pragma once
#include "matvec.cuh"

namespace ssd {

constexpr int kBatchTokens = 16;  // token vectors per batched matvec

// k_bprep: per-token x_eff = x (+ x_add) [written back], optional RMSNorm, then the exact
// fixed-point limbs of every 256-column group in the batched kernel's B layout.
struct BPrepArgs {
    const float* x;        // [16][ldx]
    const float* x_add;    // [16][ldx] or null
    float* x_writeback;    // [16][ldx] or null
    int ldx, cols;
    const float* norm_w;   // [cols] or null
    float eps;
    int norm_order;        // 0: v * (inv * w), 1: (v * inv) * w
    uint8_t* b;            // [cols / 256][16 KB] limbs
    float* cst;            // [cols / 256][256]: 2^-e per block, then X[block][token]
    float* inv;            // [16] inv_rms of each token (written by the stats kernel)
};

// Scratch and per-token layout of one batched matvec launch.
struct BWork {
    const uint8_t* b;      // from k_bprep
    const float* cst;
    unsigned int* counter; // per row tile, zero between launches
    float* partial;        // [kI8MaxGrid][2][16][128]
    int ldy, ldk;          // token strides of y (and of y_k / y_v for QKV)
    const int* pos;        // [16] positions (QKV + RoPE)
    unsigned long long* keys;  // [16] argmax keys
    int n_tiles, nk, n_units, stages;  // filled by the launcher
};

struct I8MapsB {
    CUtensorMap q[3];
    CUtensorMap m[3];
};

// With norm_w set, a stats kernel (inv_rms per token into p.inv) runs first.
int launch_bprep(ssd_ctx* ctx, int type, const BPrepArgs& p, cudaStream_t s, bool pdl);
// Y[t] = f(W X[t]) for the 16 tokens of the B operand prepared by launch_bprep. `a` gives
// the weights and epilogue as for launch_matvec (x / norm fields unused); wk the scratch.
int launch_matvec_batch(ssd_ctx* ctx, int type, int epi, const MvArgs& a, const BWork& wk,
                        cudaStream_t s, bool pdl);

}  // namespace ssd
