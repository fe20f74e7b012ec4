// matvec.cuh — fused GGUF dequant-matvec for sm_100a (internal interface).
#pragma once
#include "common.cuh"

namespace ssd {

// How virtual rows map onto up to three weight tensors of the same type and width.
enum MapMode { MAP_PLAIN = 0, MAP_QKV = 1, MAP_SWIGLU = 2 };
// What the kernel does with each finished row.
enum EpiMode {
    EPI_STORE = 0,
    EPI_RESID = 1,
    EPI_SWIGLU = 2,
    EPI_QKV_ROPE = 3,
    EPI_ARGMAX = 4,
    EPI_PEERS = 5  // partial rows stored into every tensor-parallel rank's buffer
};
constexpr int kMaxPeers = 8;

struct MvArgs {
    // weights (library layout); all segments share type and cols
    const uint8_t* qs[3];
    const uint8_t* meta[3];
    int seg_rows[3];
    int map;
    int rows;  // virtual rows
    int cols;
    // prologue: x_eff = x (+ x_add); optional writeback of x_eff by CTA 0;
    // optional RMSNorm: order 0 = v*(inv*w) (rmsnorm_f32_fast_scalar),
    // order 1 = (v*inv)*w (fused_post_attn_norm / fused_rmsnorm_linear).
    const float* x;
    const float* x_add;
    float* x_writeback;
    const float* norm_w;
    float eps;
    int norm_order;
    // Independent launch (FMA kernel): no kernel enqueued before this one writes x or the
    // other inputs, or touches y; the kernel then does not wait for its predecessor before
    // staging x (consecutive launches overlap) and waits at its end instead, so that its
    // completion still implies the completion of everything before it. Other kernels ignore
    // the flag (they always wait first).
    int x_ready;
    // epilogue
    float* y;           // STORE/RESID/SWIGLU out, QKV q out, ARGMAX logits (may be null)
    const float* base;  // RESID base (may alias y)
    float* y_k;         // QKV k out
    float* y_v;         // QKV v out
    int head_dim;
    float theta;
    int position;
    const int* position_dev;  // if non-null, position is read from device memory
    // optional (cos, sin) table of positions [0, rope_rows), head_dim / 2 pairs each, the
    // values rope_cs gives (filled once per model); other positions compute them
    const float2* rope_cache;
    int rope_rows;
    unsigned long long* argmax_key;
    int index_offset;  // added to row index for ARGMAX (tensor-parallel vocab shards)
    int* status;       // device status word for bounded waits (default: the context's)
    // Peer-memory all-reduce of tensor parallelism (model.cu). Epochs: the producer of
    // call `ar_call` of a step raises flags to *ar_epoch + ar_call + 1.
    // Input side (any epilogue): x_add = sum over r < ar_in_n, in rank order, of the
    // partials at ar_in + r * cols, read after ar_in_flag[r] reaches the epoch.
    const float* ar_in;
    const unsigned long long* ar_in_flag;
    int ar_in_n;
    // Output side (EPI_PEERS): row values go to ar_out[r] + row for every rank r; the
    // last CTA to finish (ar_counter, zero between launches) raises ar_out_flag[r].
    float* ar_out[kMaxPeers];
    unsigned long long* ar_out_flag[kMaxPeers];
    int ar_out_n;
    unsigned int* ar_counter;
    const unsigned long long* ar_epoch;
    int ar_call;
    // Split-K scratch of the tensor-core kernel (matvec_i8.cu): per-tile arrival counters
    // (zero between launches) and per-CTA partial rows, owned by the first weight.
    unsigned int* fix_counter;
    float* fix_partial;
};

// Launches y = f(W x) with the given epilogue. pdl: launch with programmatic
// stream serialization so the weight prefetch overlaps the previous kernel.
int launch_matvec(ssd_ctx* ctx, int type, int epi, const MvArgs& a, cudaStream_t s, bool pdl);

// Fills an MvArgs for a single plain weight.
inline MvArgs mv_plain(const ssd_weight* w, const float* x, float* y) {
    MvArgs a = {};
    a.qs[0] = w->qs;
    a.meta[0] = w->meta;
    a.seg_rows[0] = w->rows;
    a.map = MAP_PLAIN;
    a.rows = w->rows;
    a.cols = w->cols;
    a.x = x;
    a.y = y;
    a.fix_counter = w->fix_counter;
    a.fix_partial = w->fix_partial;
    return a;
}

}  // namespace ssd
