// model.cu — decode engine: HBM-resident quantized layers, INT8 KV cache, row-sharded
// tensor parallelism over NCCL, one CUDA graph per decode token.
//
// Replaces forward_pass and the per-token loop of generate
// (src/inference/transformer.rs:283-399, :681-770) on the compute side: per layer
//   attn_in = rms_norm(h)                                   transformer.rs:323-326
//   q,k,v   = fused_qkv_rope(attn_in)                       attention.rs:188-196
//   kv_cache.append(k, v)   (INT8, quantized_kv_cache.rs:107-110)
//   a       = attention(q, cache) ; o = Wo a                attention.rs:198-239
//   ffn_in  = fused_post_attn_norm(h += o)                  transformer.rs:350-357
//   h      += down(silu(gate ffn_in) * up ffn_in)           feed_forward.rs:17-44
// then logits = output * rmsnorm(h) and the greedy argmax (transformer.rs:690-741).
//
// Kernel sequence per layer (TP = 1): QKV+RoPE (norm folded) -> KV append ->
// attention (2 kernels) -> Wo + residual -> gate/up + SwiGLU (norm folded) ->
// down + residual. With TP = N, Wo and down produce partial sums of the hidden state
// and the residual add is folded into the next kernel's prologue. The partials are
// summed either by an NCCL all-reduce or, once the ranks have exchanged CUDA IPC
// handles (ssd_model_p2p_*), by the kernels themselves over peer memory: Wo / down
// store their rows straight into every rank's receive buffer (plain NVLink stores) and
// the last CTA raises a per-call flag on every rank; the next kernel waits for the
// flags (bounded) and sums the N partials in rank order, so every rank computes the
// same bits. No collective library call sits between the two kernels.
#include <nccl.h>
#include <string.h>

#include <string>
#include <vector>

#include "gemm.cuh"
#include "matvec.cuh"
#include "matvec_b.cuh"
#include "matvec_dev.cuh"
#include "model.cuh"
#include "ops.cuh"

#define SSD_NCCL(call)                                                                \
    do {                                                                              \
        ncclResult_t r_ = (call);                                                     \
        if (r_ != ncclSuccess) {                                                      \
            ::ssd::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call,               \
                             ncclGetErrorString(r_));                                 \
            return SSD_ERR_NCCL;                                                      \
        }                                                                             \
    } while (0)

namespace ssd {
struct Layer {
    ssd_weight *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr;
    ssd_weight *wg = nullptr, *wu = nullptr, *wd = nullptr;
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    ssd_kv_cache* kv = nullptr;
};

// Prefill weights of one layer as fp16 hi / lo splits for the tensor-core GEMMs: QKV
// concatenated ([Wq; Wk; Wv] rows), Wo, gate/up interleaved in 64-row halves of each
// 128-row tile (the SwiGLU epilogue pairs them), down; r* = per-row inverse scales.
struct PfLayer {
    __half *qkv_h = nullptr, *qkv_l = nullptr, *o_h = nullptr, *o_l = nullptr;
    __half *gu_h = nullptr, *gu_l = nullptr, *d_h = nullptr, *d_l = nullptr;
    float *qkv_r = nullptr, *o_r = nullptr, *gu_r = nullptr, *d_r = nullptr;
};

// Prefill RoPE: QKV rows [n][q_rows + 2 kv_rows] of tokens at positions pos0 + t ->
// contiguous Q (rotated), K (rotated), V; pairs (2i, 2i+1) within each head
// (rope_f32_multi_head, src/metal/compute.rs:482-506).
__global__ void __launch_bounds__(256) k_prefill_rope(const float* qkv, int q_rows, int kv_rows,
                                                      int head_dim, float theta, int pos0, float* q,
                                                      float* k, float* v) {
    __shared__ float2 cs[256];
    const int t = blockIdx.x, N = q_rows + 2 * kv_rows;
    pdl_wait();
    for (int i = threadIdx.x; i < head_dim / 2; i += 256) cs[i] = rope_cs(i, head_dim, theta, pos0 + t);
    __syncthreads();
    const float* row = qkv + (size_t)t * N;
    for (int j = 2 * threadIdx.x; j < q_rows + kv_rows; j += 512) {
        float x0 = row[j], x1 = row[j + 1];
        const float2 c = cs[(j % head_dim) >> 1];
        const float a0 = x0, a1 = x1;
        x0 = __fsub_rn(__fmul_rn(a0, c.x), __fmul_rn(a1, c.y));
        x1 = __fadd_rn(__fmul_rn(a0, c.y), __fmul_rn(a1, c.x));
        float* dst = j < q_rows ? q + (size_t)t * q_rows + j : k + (size_t)t * kv_rows + (j - q_rows);
        dst[0] = x0;
        dst[1] = x1;
    }
    for (int j = threadIdx.x; j < kv_rows; j += 256)
        v[(size_t)t * kv_rows + j] = row[q_rows + kv_rows + j];
}

__global__ void k_add(float* out, const float* a, const float* b, int n) {
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fadd_rn(a[i], b[i]);
}

// ---- dense (F16 / BF16 / F32) layer weights: the stages the quantized kernels fuse, as
// separate launches (the dense matvec has no norm prologue, RoPE or argmax epilogue)

// out = rms_norm(x) * w: order 0 x * (inv * w) (transformer.rs:576-579), order 1
// (x * inv) * w (compute.rs:536-577); one CTA.
__global__ void __launch_bounds__(1024) k_dense_norm(const float* x, const float* w, int n,
                                                     float eps, int order, float* out) {
    __shared__ float red[32];
    pdl_wait();
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += 1024) ss = fmaf(x[i], x[i], ss);
    ss = block_sum<1024>(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += 1024)
        out[i] = order == 0 ? __fmul_rn(x[i], __fmul_rn(inv, w[i]))
                            : __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

// (cos, sin) of every RoPE pair at every cache position, the values rope_cs gives: the QKV
// epilogues of the decode steps read their position's row instead of evaluating the
// double-precision power and sincos on every launch.
__global__ void k_rope_table(float2* t, int head_dim, float theta) {
    const int pos = blockIdx.x, half = head_dim / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x)
        t[(size_t)pos * half + i] = rope_cs(i, head_dim, theta, pos);
}
static int fill_rope_table(ssd_ctx* ctx, float2* t, int rows, int head_dim, float theta) {
    k_rope_table<<<rows, 128, 0, ctx->stream>>>(t, head_dim, theta);
    SSD_CK_LAUNCH();
    SSD_CK(cudaStreamSynchronize(ctx->stream));
    return SSD_OK;
}

// act = silu(gate) * up per row (feed_forward.rs:31-39; the SwiGLU epilogue of the fused
// matvecs, for weight types that have none).
__global__ void k_swiglu_rows(const float* gate, const float* up, float* act, int n) {
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) act[i] = swiglu(gate[i], up[i]);
}

// RoPE on the q and k rows at the device-held position (the pair rotation of the fused
// QKV epilogue, rope_f32_multi_head, compute.rs:482-506).
__global__ void k_rope_qk(float* q, int q_rows, float* k, int k_rows, int head_dim, float theta,
                          const int* pos, const float2* tab, int tab_rows) {
    pdl_wait();
    const int half = head_dim / 2;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;  // pair index over q then k
    const int nq = q_rows / 2;
    if (t >= nq + k_rows / 2) return;
    float* x = t < nq ? q : k;
    const int pr = t < nq ? t : t - nq;  // pair within the vector
    const int p = *pos;
    const float2 cs = p >= 0 && p < tab_rows ? tab[(size_t)p * half + pr % half]
                                             : rope_cs(pr % half, head_dim, theta, p);
    float x0 = x[2 * pr], x1 = x[2 * pr + 1];
    rope_apply(x0, x1, cs);
    x[2 * pr] = x0;
    x[2 * pr + 1] = x1;
}

// The packed (value, index) argmax key of n logits (indices index0 ..), max-combined into
// *key (zeroed by the step's finalize): the matvec's argmax epilogue for dense outputs.
__global__ void __launch_bounds__(256) k_argmax_key(const float* v, int n, uint32_t index0,
                                                    unsigned long long* key) {
    __shared__ unsigned long long red[8];
    pdl_wait();
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * 256 + threadIdx.x; i < n; i += gridDim.x * 256) {
        const unsigned long long kk = argmax_key(v[i], index0 + (uint32_t)i);
        best = kk > best ? kk : best;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
        best = t > best ? t : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; w++) best = red[w] > best ? red[w] : best;
        if (best) atomicMax(key, best);
    }
}

// f32 -> F16 / BF16 bits, round to nearest even (synthetic dense weights).
__global__ void k_to16(const float* in, uint16_t* out, size_t n, int bf) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (bf) {
        const uint32_t u = __float_as_uint(in[i]);
        out[i] = (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
    } else {
        out[i] = __half_as_ushort(__float2half_rn(in[i]));
    }
}

__host__ __device__ constexpr bool dense_type(int t) {
    return t == SSD_TYPE_F32 || t == SSD_TYPE_F16 || t == SSD_TYPE_BF16;
}
// Weight types whose matvec has no fused prologue or epilogue (dense, and the low-bit formats
// of matvec_lowbit.cu): the decode engine runs their stages as separate launches (tp_size 1).
__host__ __device__ constexpr bool staged_type(int t) { return dense_type(t) || is_lowbit(t); }
}  // namespace ssd

using namespace ssd;

struct ssd_model {
    ssd_ctx* ctx = nullptr;
    ssd_model_config cfg = {};
    // this rank's shard
    int nq_local = 0, nkv_local = 0, kv_head0 = 0, ff_local = 0, vocab_local = 0, vocab0 = 0;
    int q_rows = 0, kv_rows = 0, embd_cols_local = 0, ff0 = 0, embd0 = 0;
    std::vector<Layer> layers;
    ssd_weight* tok_embd = nullptr;
    ssd_weight* output = nullptr;
    float* out_norm = nullptr;
    // decode state (device)
    void* state = nullptr;
    float *h_a = nullptr, *h_b = nullptr, *q = nullptr, *k = nullptr, *v = nullptr;
    float *attn = nullptr, *act = nullptr, *part = nullptr, *p1 = nullptr, *p2 = nullptr;
    float* logits = nullptr;
    int32_t* token = nullptr;
    int* pos = nullptr;
    unsigned long long* key = nullptr;
    int32_t* pinned = nullptr;  // 2 pinned ints: token in / token out
    // tensor parallel
    ncclComm_t comm = nullptr;
    // peer-memory all-reduce: this rank's exported buffer ([kArSlots][tp][n_embd] floats,
    // then [kArSlots][tp] u64 flags) and every rank's buffer as mapped here
    void* p2p_buf = nullptr;
    float* p2p_rbuf[kMaxPeers] = {};
    unsigned long long* p2p_flag[kMaxPeers] = {};
    // KV absmax exchange slots ([kArSlots][tp][2] tagged words after the flags)
    unsigned long long* p2p_xch[kMaxPeers] = {};
    float* amax = nullptr;  // the (K, V) absmax pair max-reduced by NCCL (no peer path)
    float* xn = nullptr;    // normed input of the dense-weight stages
    float* gu = nullptr;    // gate and up rows of the low-bit FFN stage
    float2* rope = nullptr;  // (cos, sin) of every RoPE pair at every cache position
    void* p2p_mapped[kMaxPeers] = {};
    bool p2p = false;
    unsigned long long* ar_epoch = nullptr;  // advanced by 2 * n_layers per step
    unsigned int* ar_counter = nullptr;      // CTA completion counter of the producers
    // batch prefill: weight splits (prepared on first use) and work buffers
    void* pf_walloc = nullptr;
    std::vector<PfLayer> pf;
    void* pf_buf = nullptr;
    size_t pf_buf_bytes = 0;
    // graph
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int launches = 0;
};

static int tp_size(const ssd_model* m) { return m->cfg.tp_size < 1 ? 1 : m->cfg.tp_size; }

extern "C" int ssd_model_create(ssd_ctx* ctx, const ssd_model_config* c, ssd_model** out) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(c && out, SSD_ERR_ARG, "null argument");
    const int N = c->tp_size < 1 ? 1 : c->tp_size;
    SSD_REQ(c->tp_rank >= 0 && c->tp_rank < N, SSD_ERR_ARG, "tp_rank %d outside [0, %d)",
            c->tp_rank, N);
    SSD_REQ(c->n_layers > 0 && c->n_embd > 0 && c->n_head > 0 && c->n_head_kv > 0 &&
                c->head_dim > 0 && c->n_ff > 0 && c->vocab > 0 && c->kv_capacity > 0,
            SSD_ERR_ARG, "non-positive model dimension");
    SSD_REQ(c->n_head * c->head_dim == c->n_embd, SSD_ERR_SHAPE,
            "n_head*head_dim must equal n_embd (attention.rs:236 projects n_embd x n_embd)");
    SSD_REQ(c->n_head % c->n_head_kv == 0, SSD_ERR_SHAPE, "n_head %% n_head_kv != 0");
    SSD_REQ(c->n_head_kv % N == 0 && c->n_ff % (2 * N) == 0 && c->vocab % N == 0 &&
                c->n_embd % N == 0,
            SSD_ERR_SHAPE, "dimensions do not shard over %d ranks", N);
    const int bs = type_block(c->wtype);
    SSD_REQ(((bs == 32 || bs == 256) && !is_lowbit(c->wtype)) || (staged_type(c->wtype) && N == 1),
            SSD_ERR_TYPE, "layer weight type %d not supported%s", c->wtype,
            staged_type(c->wtype) ? " with tensor parallelism" : "");
    SSD_REQ((c->n_embd / N) % bs == 0 && (c->n_ff / N) % bs == 0, SSD_ERR_SHAPE,
            "column shards must be whole %d-wide blocks", bs);
    SSD_REQ(c->embd_type == SSD_TYPE_F32 || c->embd_type == SSD_TYPE_Q4_0 ||
                c->embd_type == SSD_TYPE_Q8_0 || c->embd_type == SSD_TYPE_Q4_K ||
                c->embd_type == SSD_TYPE_Q5_K || c->embd_type == SSD_TYPE_Q6_K ||
                c->embd_type == SSD_TYPE_Q8_K || c->embd_type == SSD_TYPE_F16 ||
                c->embd_type == SSD_TYPE_BF16,
            SSD_ERR_TYPE, "token_embd type %d not supported", c->embd_type);
    SSD_REQ(((type_block(c->out_type) == 32 || type_block(c->out_type) == 256) &&
             !is_lowbit(c->out_type)) ||
                (staged_type(c->out_type) && N == 1),
            SSD_ERR_TYPE, "output type %d not supported", c->out_type);

    ssd_model* m = new ssd_model();
    m->ctx = ctx;
    m->cfg = *c;
    m->cfg.tp_size = N;
    const int r = c->tp_rank;
    m->nkv_local = c->n_head_kv / N;
    m->kv_head0 = r * m->nkv_local;
    m->nq_local = c->n_head / N;
    m->q_rows = m->nq_local * c->head_dim;
    m->kv_rows = m->nkv_local * c->head_dim;  // this rank's K/V heads
    m->embd_cols_local = c->n_embd / N;
    m->embd0 = r * m->embd_cols_local;
    m->ff_local = c->n_ff / N;
    m->ff0 = r * m->ff_local;
    m->vocab_local = c->vocab / N;
    m->vocab0 = r * m->vocab_local;
    m->layers.resize(c->n_layers);

    // decode state
    const int E = c->n_embd;
    const size_t pf = attn_partial_floats(m->nq_local, c->kv_capacity, c->head_dim);
    size_t floats = 0;
    auto take = [&](size_t n) {
        size_t off = floats;
        floats += (n + 63) & ~(size_t)63;
        return off;
    };
    const size_t o_ha = take(E), o_hb = take(E), o_q = take(m->q_rows), o_k = take(m->kv_rows),
                 o_v = take(m->kv_rows), o_attn = take(m->q_rows), o_act = take(m->ff_local),
                 o_part = take(pf), o_p1 = take(E), o_p2 = take(E), o_log = take(m->vocab_local),
                 o_misc = take(64), o_xn = take(E), o_gu = take(2 * (size_t)m->ff_local),
                 o_rope = take((size_t)c->kv_capacity * c->head_dim);
    if (cudaMalloc(&m->state, floats * 4) != cudaSuccess) {
        cudaGetLastError();
        delete m;
        set_error("decode state allocation failed");
        return SSD_ERR_NOMEM;
    }
    if (zero_device(ctx, m->state, floats * 4) != SSD_OK ||
        fill_rope_table(ctx, reinterpret_cast<float2*>((float*)m->state + o_rope),
                        c->kv_capacity, c->head_dim, c->theta) != SSD_OK) {
        cudaFree(m->state);
        delete m;
        return SSD_ERR_CUDA;
    }
    float* S = (float*)m->state;
    m->h_a = S + o_ha;
    m->h_b = S + o_hb;
    m->q = S + o_q;
    m->k = S + o_k;
    m->v = S + o_v;
    m->attn = S + o_attn;
    m->act = S + o_act;
    m->part = S + o_part;
    m->p1 = S + o_p1;
    m->p2 = S + o_p2;
    m->logits = S + o_log;
    m->key = reinterpret_cast<unsigned long long*>(S + o_misc);
    m->token = reinterpret_cast<int32_t*>(S + o_misc + 4);
    m->pos = reinterpret_cast<int*>(S + o_misc + 8);
    m->ar_epoch = reinterpret_cast<unsigned long long*>(S + o_misc + 16);
    m->ar_counter = reinterpret_cast<unsigned int*>(S + o_misc + 20);
    m->amax = S + o_misc + 24;
    m->xn = S + o_xn;
    m->gu = S + o_gu;
    m->rope = reinterpret_cast<float2*>(S + o_rope);
    if (cudaHostAlloc(&m->pinned, 16, cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(m->state);
        delete m;
        set_error("pinned staging allocation failed");
        return SSD_ERR_NOMEM;
    }
    for (auto& L : m->layers) {
        int st = ssd_kv_create(ctx, c->kv_capacity, m->nkv_local, c->head_dim, &L.kv);
        if (st != SSD_OK) {
            ssd_model_free(m);
            return st;
        }
    }
    *out = m;
    return SSD_OK;
}

extern "C" int ssd_model_free(ssd_model* m) {
    if (!m) return SSD_OK;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    for (auto& L : m->layers) {
        ssd_weight_free(L.wq);
        ssd_weight_free(L.wk);
        ssd_weight_free(L.wv);
        ssd_weight_free(L.wo);
        ssd_weight_free(L.wg);
        ssd_weight_free(L.wu);
        ssd_weight_free(L.wd);
        if (L.attn_norm) cudaFree(L.attn_norm);
        if (L.ffn_norm) cudaFree(L.ffn_norm);
        ssd_kv_free(L.kv);
    }
    ssd_weight_free(m->tok_embd);
    ssd_weight_free(m->output);
    if (m->out_norm) cudaFree(m->out_norm);
    if (m->comm) ncclCommDestroy(m->comm);
    for (int r = 0; r < kMaxPeers; r++)
        if (m->p2p_mapped[r]) cudaIpcCloseMemHandle(m->p2p_mapped[r]);
    if (m->p2p_buf) cudaFree(m->p2p_buf);
    if (m->pf_walloc) cudaFree(m->pf_walloc);
    if (m->pf_buf) cudaFree(m->pf_buf);
    if (m->state) cudaFree(m->state);
    if (m->pinned) cudaFreeHost(m->pinned);
    delete m;
    return SSD_OK;
}

extern "C" int ssd_tp_unique_id(uint8_t out[128]) {
    SSD_REQ(out != nullptr, SSD_ERR_ARG, "null out");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    ncclUniqueId id;
    SSD_NCCL(ncclGetUniqueId(&id));
    memcpy(out, &id, 128);
    return SSD_OK;
}

extern "C" int ssd_model_tp_init(ssd_model* m, const uint8_t uid[128]) {
    SSD_REQ(m && uid, SSD_ERR_ARG, "null argument");
    SSD_TRY(check_ctx(m->ctx));
    if (tp_size(m) == 1) return SSD_OK;
    SSD_REQ(m->comm == nullptr, SSD_ERR_STATE, "communicator already initialised");
    ncclUniqueId id;
    memcpy(&id, uid, 128);
    SSD_NCCL(ncclCommInitRank(&m->comm, tp_size(m), id, m->cfg.tp_rank));
    return SSD_OK;
}

// ------------------------------------------------------ peer-memory all-reduce
constexpr int kArSlots = 4;  // receive slots, used round robin by the producer calls

static size_t p2p_floats(const ssd_model* m) {
    return (size_t)kArSlots * tp_size(m) * m->cfg.n_embd;
}

extern "C" int ssd_model_p2p_handle(ssd_model* m, uint8_t out[64]) {
    SSD_REQ(m && out, SSD_ERR_ARG, "null argument");
    SSD_TRY(check_ctx(m->ctx));
    SSD_REQ(tp_size(m) > 1 && tp_size(m) <= kMaxPeers, SSD_ERR_STATE,
            "peer all-reduce needs 2..%d ranks", kMaxPeers);
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "cudaIpcMemHandle_t size");
    if (!m->p2p_buf) {
        const size_t fl = (p2p_floats(m) * 4 + 255) & ~(size_t)255;
        const size_t bytes = fl + (size_t)kArSlots * tp_size(m) * 8 * 3;  // flags, exchange
        if (cudaMalloc(&m->p2p_buf, bytes) != cudaSuccess) {
            cudaGetLastError();
            m->p2p_buf = nullptr;
            set_error("peer all-reduce buffer allocation (%zu bytes) failed", bytes);
            return SSD_ERR_NOMEM;
        }
        SSD_TRY(zero_device(m->ctx, m->p2p_buf, bytes));
    }
    cudaIpcMemHandle_t h;
    SSD_CK(cudaIpcGetMemHandle(&h, m->p2p_buf));
    memcpy(out, &h, 64);
    return SSD_OK;
}

extern "C" int ssd_model_p2p_open(ssd_model* m, const uint8_t* handles) {
    SSD_REQ(m && handles, SSD_ERR_ARG, "null argument");
    SSD_TRY(check_ctx(m->ctx));
    SSD_REQ(m->p2p_buf != nullptr, SSD_ERR_STATE, "call ssd_model_p2p_handle first");
    SSD_REQ(!m->p2p, SSD_ERR_STATE, "peer buffers already open");
    const int N = tp_size(m), me = m->cfg.tp_rank;
    const size_t fl = (p2p_floats(m) * 4 + 255) & ~(size_t)255;
    for (int r = 0; r < N; r++) {
        void* p = nullptr;
        if (r == me) {
            p = m->p2p_buf;
        } else {
            cudaIpcMemHandle_t h;
            memcpy(&h, handles + (size_t)r * 64, 64);
            cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                cudaGetLastError();
                set_error("opening rank %d's buffer: %s", r, cudaGetErrorString(e));
                return SSD_ERR_CUDA;
            }
            m->p2p_mapped[r] = p;
        }
        m->p2p_rbuf[r] = (float*)p;
        m->p2p_flag[r] = (unsigned long long*)((char*)p + fl);
        m->p2p_xch[r] = m->p2p_flag[r] + (size_t)kArSlots * N;
    }
    m->p2p = true;
    if (m->exec) {  // re-capture with the peer path
        cudaGraphExecDestroy(m->exec);
        cudaGraphDestroy(m->graph);
        m->exec = nullptr;
        m->graph = nullptr;
    }
    return SSD_OK;
}

// A partial sum of the hidden state waiting to be added by the next kernel's prologue:
// an NCCL-reduced buffer, or the peer-memory slot of producer call `call`.
struct Pending {
    bool on = false;
    bool p2p = false;
    float* buf = nullptr;
    int call = 0;
};

static void take_pending(ssd_model* m, MvArgs& a, Pending& p) {
    if (!p.on) return;
    if (p.p2p) {
        const int N = tp_size(m), slot = p.call % kArSlots;
        a.ar_in = m->p2p_rbuf[m->cfg.tp_rank] + (size_t)slot * N * m->cfg.n_embd;
        a.ar_in_flag = m->p2p_flag[m->cfg.tp_rank] + (size_t)slot * N;
        a.ar_in_n = N;
        a.ar_epoch = m->ar_epoch;
        a.ar_call = p.call;
    } else {
        a.x_add = p.buf;
    }
    p = Pending{};
}

// Launches a partial-sum producer (Wo or down at TP > 1) and leaves the pending sum.
static int produce_partial(ssd_model* m, int type, MvArgs a, float* nccl_buf, bool use_p2p,
                           int call, Pending& p, cudaStream_t s) {
    const auto& c = m->cfg;
    if (use_p2p) {
        const int N = tp_size(m), me = c.tp_rank, slot = call % kArSlots;
        a.y = nullptr;
        a.ar_out_n = N;
        for (int r = 0; r < N; r++) {
            a.ar_out[r] = m->p2p_rbuf[r] + ((size_t)slot * N + me) * c.n_embd;
            a.ar_out_flag[r] = m->p2p_flag[r] + (size_t)slot * N + me;
        }
        a.ar_counter = m->ar_counter;
        a.ar_epoch = m->ar_epoch;
        a.ar_call = call;
        SSD_TRY(launch_matvec(m->ctx, type, EPI_PEERS, a, s, true));
        p = Pending{true, true, nullptr, call};
    } else {
        a.y = nccl_buf;
        SSD_TRY(launch_matvec(m->ctx, type, EPI_STORE, a, s, true));
        SSD_NCCL(ncclAllReduce(nccl_buf, nccl_buf, c.n_embd, ncclFloat32, ncclSum, m->comm, s));
        p = Pending{true, false, nccl_buf, call};
    }
    return SSD_OK;
}

// ------------------------------------------------------------------ weights

// Which slice of a global tensor this rank keeps. Row-sharded: attn_q, attn_k, attn_v
// (by heads: n_head / N query heads and n_head_kv / N KV heads per rank, the KV heads those
// query heads read), ffn_gate, ffn_up, output (by vocab rows). Column-sharded: attn_output
// (by the rank's q-head columns), ffn_down (by the rank's FFN columns). Replicated:
// token_embd. The INT8 KV row scale spans all KV heads (quantized_kv_cache.rs:107-110),
// so the ranks exchange the absmax of their K / V slices at every append.
struct Shard {
    int rows, cols;   // global shape
    int row0, nrows;  // kept rows
    int col0, ncols;  // kept cols
    int type;
    uint32_t tid;     // synthetic-generator tensor id
};

static int shard_range(const ssd_model_config& c, const std::string& name, int layer, Shard& s) {
    const int N = c.tp_size < 1 ? 1 : c.tp_size, r = c.tp_rank;
    const int E = c.n_embd, F = c.n_ff, KV = c.n_head_kv * c.head_dim;
    const int qr = (c.n_head / N) * c.head_dim, ec = E / N, fl = F / N, vl = c.vocab / N;
    const int kvl = (c.n_head_kv / N) * c.head_dim;
    if (layer < 0) {
        if (name == "token_embd") {
            s = Shard{c.vocab, E, 0, c.vocab, 0, E, c.embd_type, 1000001u};
            return SSD_OK;
        }
        if (name == "output") {
            s = Shard{c.vocab, E, r * vl, vl, 0, E, c.out_type, 1000002u};
            return SSD_OK;
        }
        set_error("unknown global tensor '%s'", name.c_str());
        return SSD_ERR_ARG;
    }
    SSD_REQ(layer < c.n_layers, SSD_ERR_ARG, "layer %d out of range", layer);
    const uint32_t base = (uint32_t)layer * 16u;
    if (name == "attn_q")
        s = Shard{E, E, r * qr, qr, 0, E, c.wtype, base + 0};
    else if (name == "attn_k")
        s = Shard{KV, E, r * kvl, kvl, 0, E, c.wtype, base + 1};
    else if (name == "attn_v")
        s = Shard{KV, E, r * kvl, kvl, 0, E, c.wtype, base + 2};
    else if (name == "attn_output")
        s = Shard{E, E, 0, E, r * ec, ec, c.wtype, base + 3};
    else if (name == "ffn_gate")
        s = Shard{F, E, r * fl, fl, 0, E, c.wtype, base + 4};
    else if (name == "ffn_up")
        s = Shard{F, E, r * fl, fl, 0, E, c.wtype, base + 5};
    else if (name == "ffn_down")
        s = Shard{E, F, 0, E, r * fl, fl, c.wtype, base + 6};
    else {
        set_error("unknown layer tensor '%s'", name.c_str());
        return SSD_ERR_ARG;
    }
    return SSD_OK;
}

static ssd_weight** slot_of(ssd_model* m, const std::string& name, int layer) {
    if (layer < 0) return name == "token_embd" ? &m->tok_embd : &m->output;
    Layer& L = m->layers[layer];
    if (name == "attn_q") return &L.wq;
    if (name == "attn_k") return &L.wk;
    if (name == "attn_v") return &L.wv;
    if (name == "attn_output") return &L.wo;
    if (name == "ffn_gate") return &L.wg;
    if (name == "ffn_up") return &L.wu;
    return &L.wd;
}

static int shard_of(ssd_model* m, const std::string& name, int layer, Shard& s,
                    ssd_weight**& slot) {
    SSD_TRY(shard_range(m->cfg, name, layer, s));
    slot = slot_of(m, name, layer);
    return SSD_OK;
}

extern "C" int ssd_shard_range(const ssd_model_config* c, const char* name, int layer, int* row0,
                               int* nrows, int* col0, int* ncols) {
    SSD_REQ(c && name, SSD_ERR_ARG, "null argument");
    Shard s;
    SSD_TRY(shard_range(*c, std::string(name), layer, s));
    if (row0) *row0 = s.row0;
    if (nrows) *nrows = s.nrows;
    if (col0) *col0 = s.col0;
    if (ncols) *ncols = s.ncols;
    return SSD_OK;
}

static int set_norm(ssd_model* m, float** slot, const void* host, size_t bytes) {
    const size_t need = (size_t)m->cfg.n_embd * 4;
    SSD_REQ(bytes == need, SSD_ERR_SHAPE, "norm weight needs %zu bytes, got %zu", need, bytes);
    if (!*slot) SSD_CK(cudaMalloc(slot, need));
    // on the context's (non-blocking) stream, complete before any later launch reads it
    SSD_CK(cudaMemcpyAsync(*slot, host, need, cudaMemcpyHostToDevice, m->ctx->stream));
    SSD_CK(cudaStreamSynchronize(m->ctx->stream));
    return SSD_OK;
}

extern "C" int ssd_model_set_tensor_typed(ssd_model* m, const char* cname, int layer,
                                          const void* host, size_t bytes, int ggml_type) {
    SSD_REQ(m && cname && host, SSD_ERR_ARG, "null argument");
    SSD_TRY(check_ctx(m->ctx));
    const std::string name(cname);
    if (layer >= 0 && name == "attn_norm") {
        SSD_REQ(layer < m->cfg.n_layers, SSD_ERR_ARG, "layer out of range");
        return set_norm(m, &m->layers[layer].attn_norm, host, bytes);
    }
    if (layer >= 0 && name == "ffn_norm") {
        SSD_REQ(layer < m->cfg.n_layers, SSD_ERR_ARG, "layer out of range");
        return set_norm(m, &m->layers[layer].ffn_norm, host, bytes);
    }
    if (layer < 0 && name == "output_norm") return set_norm(m, &m->out_norm, host, bytes);
    Shard s;
    ssd_weight** slot = nullptr;
    SSD_TRY(shard_of(m, name, layer, s, slot));
    if (ggml_type >= 0 && ggml_type != s.type) {  // this tensor's own type
        const bool embd = name == "token_embd";
        SSD_REQ(ggml_type == SSD_TYPE_Q4_0 || ggml_type == SSD_TYPE_Q8_0 ||
                    ggml_type == SSD_TYPE_Q4_K || ggml_type == SSD_TYPE_Q5_K ||
                    ggml_type == SSD_TYPE_Q6_K || ggml_type == SSD_TYPE_Q8_K ||
                    (dense_type(ggml_type) && (embd || tp_size(m) == 1)) ||
                    (is_lowbit(ggml_type) && !embd && tp_size(m) == 1),
                SSD_ERR_TYPE, "%s: ggml type %d not supported here", cname, ggml_type);
        const int tb = type_block(ggml_type);
        SSD_REQ(s.cols % tb == 0 && s.col0 % tb == 0 && s.ncols % tb == 0, SSD_ERR_SHAPE,
                "%s: columns (shard %d + %d of %d) not whole %d-wide blocks", cname, s.col0,
                s.ncols, s.cols, tb);
        s.type = ggml_type;
    }
    const size_t rb = ssd_row_bytes(s.type, s.cols);
    SSD_REQ(rb != 0 && bytes == rb * (size_t)s.rows, SSD_ERR_SHAPE,
            "%s: %zu bytes given, %dx%d of type %d needs %zu", cname, bytes, s.rows, s.cols, s.type,
            rb * (size_t)s.rows);
    const int bs = type_block(s.type);
    const size_t kb = ssd_row_bytes(s.type, s.ncols);
    std::vector<uint8_t> buf(kb * (size_t)s.nrows);
    const uint8_t* src = (const uint8_t*)host;
    const size_t coff = (size_t)(s.col0 / bs) * type_block_bytes(s.type);
    for (int r = 0; r < s.nrows; r++)
        memcpy(buf.data() + (size_t)r * kb, src + (size_t)(s.row0 + r) * rb + coff, kb);
    ssd_weight* w = nullptr;
    SSD_TRY(ssd_weight_upload(m->ctx, buf.data(), buf.size(), s.type, s.nrows, s.ncols, &w));
    ssd_weight_free(*slot);
    *slot = w;
    if (m->exec) {  // weights changed: the captured graph holds the old pointers (and types)
        cudaGraphExecDestroy(m->exec);
        cudaGraphDestroy(m->graph);
        m->exec = nullptr;
        m->graph = nullptr;
    }
    return SSD_OK;
}

extern "C" int ssd_model_set_tensor(ssd_model* m, const char* cname, int layer, const void* host,
                                    size_t bytes) {
    return ssd_model_set_tensor_typed(m, cname, layer, host, bytes, -1);
}

extern "C" int ssd_model_synth_weights(ssd_model* m, uint64_t seed, float std_dev) {
    SSD_REQ(m != nullptr, SSD_ERR_ARG, "null model");
    SSD_TRY(check_ctx(m->ctx));
    const auto& c = m->cfg;
    static const char* names[] = {"attn_q", "attn_k", "attn_v", "attn_output",
                                  "ffn_gate", "ffn_up", "ffn_down"};
    auto synth = [&](const char* nm, int layer, float sd) -> int {
        Shard s;
        ssd_weight** slot = nullptr;
        SSD_TRY(shard_of(m, nm, layer, s, slot));
        ssd_weight* w = nullptr;
        if (s.type == SSD_TYPE_F32) {
            SSD_TRY(alloc_weight(m->ctx, SSD_TYPE_F32, s.nrows, s.ncols, &w));
            SSD_TRY(ssd_synth_f32(m->ctx, seed, s.tid, 0.0f, sd, s.cols, s.row0, s.nrows, s.col0,
                                  s.ncols, (float*)w->qs, (void*)m->ctx->stream));
        } else if (s.type == SSD_TYPE_F16 || s.type == SSD_TYPE_BF16) {  // N(0, sd) rounded
            const size_t n = (size_t)s.nrows * s.ncols;
            SSD_TRY(alloc_weight(m->ctx, s.type, s.nrows, s.ncols, &w));
            float* tmp = nullptr;
            SSD_CK(cudaMalloc(&tmp, n * 4));
            int st = ssd_synth_f32(m->ctx, seed, s.tid, 0.0f, sd, s.cols, s.row0, s.nrows, s.col0,
                                   s.ncols, tmp, (void*)m->ctx->stream);
            if (st == SSD_OK) {
                k_to16<<<(unsigned)((n + 255) / 256), 256, 0, m->ctx->stream>>>(
                    tmp, reinterpret_cast<uint16_t*>(w->qs), n, s.type == SSD_TYPE_BF16);
                if (cudaStreamSynchronize(m->ctx->stream) != cudaSuccess) st = SSD_ERR_CUDA;
            }
            cudaFree(tmp);
            if (st != SSD_OK) {
                ssd_weight_free(w);
                return st;
            }
        } else {
            SSD_TRY(ssd_weight_synth(m->ctx, s.type, seed, s.tid, sd, s.cols, s.row0, s.nrows,
                                     s.col0, s.ncols, &w, (void*)m->ctx->stream));
        }
        ssd_weight_free(*slot);
        *slot = w;
        return SSD_OK;
    };
    auto norm = [&](float** slot, uint32_t tid) -> int {
        if (!*slot) SSD_CK(cudaMalloc(slot, (size_t)c.n_embd * 4));
        return ssd_synth_f32(m->ctx, seed, tid, 1.0f, 0.02f, c.n_embd, 0, 1, 0, c.n_embd, *slot,
                             (void*)m->ctx->stream);
    };
    for (int l = 0; l < c.n_layers; l++) {
        for (const char* nm : names) SSD_TRY(synth(nm, l, std_dev));
        SSD_TRY(norm(&m->layers[l].attn_norm, (uint32_t)l * 16u + 8u));
        SSD_TRY(norm(&m->layers[l].ffn_norm, (uint32_t)l * 16u + 9u));
    }
    SSD_TRY(synth("token_embd", -1, 1.0f));
    SSD_TRY(synth("output", -1, std_dev));
    SSD_TRY(norm(&m->out_norm, 1000003u));
    SSD_CK(cudaStreamSynchronize(m->ctx->stream));
    if (m->exec) {
        cudaGraphExecDestroy(m->exec);
        cudaGraphDestroy(m->graph);
        m->exec = nullptr;
        m->graph = nullptr;
    }
    return SSD_OK;
}

extern "C" int ssd_model_synth_kv(ssd_model* m, uint64_t seed, int n) {
    SSD_REQ(m != nullptr, SSD_ERR_ARG, "null model");
    SSD_TRY(check_ctx(m->ctx));
    const auto& c = m->cfg;
    SSD_REQ(n >= 0 && n < c.kv_capacity, SSD_ERR_SHAPE, "n %d outside [0, %d)", n, c.kv_capacity);
    const int kvd = c.n_head_kv * c.head_dim;
    if (n > 0) {
        const int chunk = 256;
        float* tmp = nullptr;
        SSD_CK(cudaMalloc(&tmp, (size_t)2 * chunk * kvd * 4));
        int st = SSD_OK;
        for (int l = 0; l < c.n_layers && st == SSD_OK; l++) {
            for (int p0 = 0; p0 < n && st == SSD_OK; p0 += chunk) {
                const int rows = n - p0 < chunk ? n - p0 : chunk;
                // K and V rows N(0, 1): element (pos, i) of tensors 2000000 + 2l (+1)
                st = ssd_synth_f32(m->ctx, seed, 2000000u + 2u * l, 0.0f, 1.0f, kvd, p0, rows, 0,
                                   kvd, tmp, (void*)m->ctx->stream);
                if (st == SSD_OK)
                    st = ssd_synth_f32(m->ctx, seed, 2000001u + 2u * l, 0.0f, 1.0f, kvd, p0, rows,
                                       0, kvd, tmp + (size_t)chunk * kvd, (void*)m->ctx->stream);
                if (st == SSD_OK)  // whole-row scale, this rank's heads stored
                    st = launch_kv_append_slice(m->layers[l].kv, tmp, tmp + (size_t)chunk * kvd,
                                                kvd, m->kv_head0 * c.head_dim, p0, rows,
                                                m->ctx->stream);
            }
        }
        cudaStreamSynchronize(m->ctx->stream);
        cudaFree(tmp);
        SSD_TRY(st);
    }
    return ssd_model_set_position(m, n);
}

extern "C" int ssd_model_set_position(ssd_model* m, int pos) {
    SSD_REQ(m != nullptr, SSD_ERR_ARG, "null model");
    SSD_TRY(check_ctx(m->ctx));
    SSD_REQ(pos >= 0 && pos < m->cfg.kv_capacity, SSD_ERR_SHAPE, "position %d outside [0, %d)", pos,
            m->cfg.kv_capacity);
    SSD_CK(cudaMemcpyAsync(m->pos, &pos, 4, cudaMemcpyHostToDevice, m->ctx->stream));
    SSD_CK(cudaStreamSynchronize(m->ctx->stream));
    return SSD_OK;
}

extern "C" int ssd_model_get_position(ssd_model* m, int* pos) {
    SSD_REQ(m && pos, SSD_ERR_ARG, "null argument");
    SSD_TRY(check_ctx(m->ctx));
    SSD_CK(cudaMemcpyAsync(pos, m->pos, 4, cudaMemcpyDeviceToHost, m->ctx->stream));
    SSD_CK(cudaStreamSynchronize(m->ctx->stream));
    return SSD_OK;
}

extern "C" int ssd_model_state(ssd_model* m, float** hidden, float** logits, int32_t** token) {
    SSD_REQ(m != nullptr, SSD_ERR_ARG, "null model");
    if (hidden) *hidden = m->h_a;
    if (logits) *logits = m->logits;
    if (token) *token = m->token;
    return SSD_OK;
}

extern "C" int ssd_model_weight(ssd_model* m, const char* name, int layer, ssd_weight** out) {
    SSD_REQ(m && name && out, SSD_ERR_ARG, "null argument");
    Shard s;
    ssd_weight** slot = nullptr;
    SSD_TRY(shard_of(m, std::string(name), layer, s, slot));
    SSD_REQ(*slot != nullptr, SSD_ERR_STATE, "tensor %s (layer %d) not set", name, layer);
    *out = *slot;
    return SSD_OK;
}

extern "C" int ssd_model_norm(ssd_model* m, const char* name, int layer, float** out) {
    SSD_REQ(m && name && out, SSD_ERR_ARG, "null argument");
    const std::string n(name);
    float* p = nullptr;
    if (layer < 0 && n == "output_norm") {
        p = m->out_norm;
    } else {
        SSD_REQ(layer >= 0 && layer < m->cfg.n_layers, SSD_ERR_ARG, "layer out of range");
        if (n == "attn_norm") p = m->layers[layer].attn_norm;
        else if (n == "ffn_norm") p = m->layers[layer].ffn_norm;
        else SSD_REQ(false, SSD_ERR_ARG, "unknown norm '%s'", name);
    }
    SSD_REQ(p != nullptr, SSD_ERR_STATE, "norm %s not set", name);
    *out = p;
    return SSD_OK;
}

extern "C" int ssd_model_kv(ssd_model* m, int layer, ssd_kv_cache** out) {
    SSD_REQ(m && out && layer >= 0 && layer < m->cfg.n_layers, SSD_ERR_ARG, "bad arguments");
    *out = m->layers[layer].kv;
    return SSD_OK;
}

// --------------------------------------------------------------- sequence

static int check_weights(ssd_model* m) {
    for (int l = 0; l < m->cfg.n_layers; l++) {
        const Layer& L = m->layers[l];
        SSD_REQ(L.wq && L.wk && L.wv && L.wo && L.wg && L.wu && L.wd && L.attn_norm && L.ffn_norm,
                SSD_ERR_STATE, "layer %d has unset tensors", l);
    }
    SSD_REQ(m->tok_embd && m->output && m->out_norm, SSD_ERR_STATE, "global tensors unset");
    if (tp_size(m) > 1) SSD_REQ(m->comm != nullptr, SSD_ERR_STATE, "tp_size > 1 needs tp_init");
    return SSD_OK;
}

// Enqueues one layer on stream s. `h` is the residual stream on entry; `pend` a
// pending partial sum (TP) to add first. On return `h` / `pend` describe the new
// residual stream. Producer calls of the step are numbered 2*layer (Wo) and
// 2*layer + 1 (down).
static int enqueue_layer(ssd_model* m, int l, float*& h, Pending& pend, bool use_p2p,
                         cudaStream_t s, int& nl) {
    const auto& c = m->cfg;
    const Layer& L = m->layers[l];
    const bool tp = tp_size(m) > 1;
    float* h_other = (h == m->h_a) ? m->h_b : m->h_a;
    // 1. QKV + RoPE with the pre-attention RMSNorm folded in. Each weight keeps its own
    // type (the reference dispatches every tensor on its dtype, compute.rs:648-675); a V of
    // another type than Q / K gets its own launch after them. Dense (F16 / BF16 / F32)
    // weights, at tp_size 1: norm, the three matvecs, RoPE at the device-held position.
    if (staged_type(L.wq->type) || staged_type(L.wk->type) || staged_type(L.wv->type)) {
        SSD_REQ(!tp && !pend.on, SSD_ERR_TYPE, "dense / low-bit layer weights run at tp_size 1");
        k_dense_norm<<<1, 1024, 0, s>>>(h, L.attn_norm, c.n_embd, c.eps, 0, m->xn);
        SSD_CK_LAUNCH();
        const ssd_weight* ws[3] = {L.wq, L.wk, L.wv};
        float* ys[3] = {m->q, m->k, m->v};
        for (int j = 0; j < 3; j++)
            SSD_TRY(launch_matvec(m->ctx, ws[j]->type, EPI_STORE, mv_plain(ws[j], m->xn, ys[j]),
                                  s, true));
        const int pairs = (m->q_rows + m->kv_rows) / 2;
        k_rope_qk<<<(pairs + 255) / 256, 256, 0, s>>>(m->q, m->q_rows, m->k, m->kv_rows,
                                                      c.head_dim, c.theta, m->pos, m->rope,
                                                      c.kv_capacity);
        SSD_CK_LAUNCH();
        nl += 5;
    } else {
    SSD_REQ(L.wq->type == L.wk->type, SSD_ERR_TYPE, "attn_q and attn_k types differ (%d, %d)",
            L.wq->type, L.wk->type);
    const bool v_apart = L.wv->type != L.wq->type;
    MvArgs a = {};
    a.qs[0] = L.wq->qs;
    a.qs[1] = L.wk->qs;
    a.qs[2] = L.wv->qs;
    a.meta[0] = L.wq->meta;
    a.meta[1] = L.wk->meta;
    a.meta[2] = L.wv->meta;
    a.seg_rows[0] = m->q_rows;
    a.seg_rows[1] = m->kv_rows;
    a.seg_rows[2] = v_apart ? 0 : m->kv_rows;
    a.map = MAP_QKV;
    a.rows = m->q_rows + (v_apart ? 1 : 2) * m->kv_rows;
    a.cols = c.n_embd;
    a.x = h;
    const bool had_pend = pend.on;
    if (had_pend) {  // hidden += partial (all-reduced), written back for the residual path
        take_pending(m, a, pend);
        a.x_writeback = h_other;
    }
    a.norm_w = L.attn_norm;
    a.eps = c.eps;
    a.norm_order = 0;
    a.y = m->q;
    a.y_k = m->k;
    a.y_v = m->v;
    a.head_dim = c.head_dim;
    a.theta = c.theta;
    a.position_dev = m->pos;
    a.rope_cache = m->rope;
    a.rope_rows = c.kv_capacity;
    SSD_TRY(launch_matvec(m->ctx, L.wq->type, EPI_QKV_ROPE, a, s, true));
    nl++;
    if (had_pend) {
        h = h_other;
        h_other = (h == m->h_a) ? m->h_b : m->h_a;
    }
    if (v_apart) {  // the same normed input (any pending sum was added and written back)
        MvArgs va = mv_plain(L.wv, h, m->v);
        va.norm_w = L.attn_norm;
        va.eps = c.eps;
        va.norm_order = 0;
        SSD_TRY(launch_matvec(m->ctx, L.wv->type, EPI_STORE, va, s, true));
        nl++;
    }
    }  // quantized QKV
    // 2-3. INT8 KV append at the current position (fused) and attention over this rank's
    // KV heads
    AttnArgs at = {};
    at.k_new = m->k;
    at.v_new = m->v;
    at.k = L.kv->k;
    at.v = L.kv->v;
    at.ks = L.kv->k_scale;
    at.vs = L.kv->v_scale;
    at.kv_dim = L.kv->kv_dim;
    at.head_dim = c.head_dim;
    at.group = c.n_head / c.n_head_kv;
    at.kv_head0 = 0;  // the cache holds this rank's heads only
    at.n_kv_local = m->nkv_local;
    at.q = m->q;
    at.out = m->attn;
    at.partial = m->part;
    at.pos_dev = m->pos;
    at.max_seq = c.kv_capacity;
    if (tp && use_p2p) {  // global row absmax: exchanged inside the attention kernel
        const int N = tp_size(m), me = c.tp_rank, slot = l % kArSlots;
        at.xch_n = N;
        at.xch_call = l;
        at.xch_epoch = m->ar_epoch;
        at.xch_in = m->p2p_xch[me] + (size_t)slot * N * 2;
        for (int r = 0; r < N; r++) at.xch_out[r] = m->p2p_xch[r] + ((size_t)slot * N + me) * 2;
        at.status = m->ctx->dev_status;
    } else if (tp) {  // local pair, NCCL max-reduce, then the append reads it
        SSD_TRY(launch_kv_absmax(m->k, m->v, m->kv_rows, m->amax, s, true));
        nl++;
        SSD_NCCL(ncclAllReduce(m->amax, m->amax, 2, ncclFloat32, ncclMax, m->comm, s));
        at.amax_in = m->amax;
    }
    SSD_TRY(launch_attention(at, s, true));
    nl += 2;
    // 4. output projection (+ residual, or a partial sum for the all-reduce)
    MvArgs o = mv_plain(L.wo, m->attn, h_other);
    if (tp) {
        SSD_TRY(produce_partial(m, L.wo->type, o, m->p1, use_p2p, 2 * l, pend, s));
    } else {
        o.base = h;
        SSD_TRY(launch_matvec(m->ctx, L.wo->type, EPI_RESID, o, s, true));
        h = h_other;
        h_other = (h == m->h_a) ? m->h_b : m->h_a;
    }
    nl++;
    // 5. gate/up + SwiGLU with the FFN RMSNorm folded in (one fused launch: one type)
    SSD_REQ(L.wg->type == L.wu->type, SSD_ERR_TYPE, "ffn_gate and ffn_up types differ (%d, %d)",
            L.wg->type, L.wu->type);
    if (dense_type(L.wg->type)) {  // dense: the FFN norm, then the gate / up row pairs
        SSD_REQ(!tp && !pend.on, SSD_ERR_TYPE, "dense layer weights run at tp_size 1");
        k_dense_norm<<<1, 1024, 0, s>>>(h, L.ffn_norm, c.n_embd, c.eps, 1, m->xn);
        SSD_CK_LAUNCH();
        MvArgs g = {};
        g.qs[0] = L.wg->qs;
        g.qs[1] = L.wu->qs;
        g.seg_rows[0] = m->ff_local;
        g.seg_rows[1] = m->ff_local;
        g.map = MAP_SWIGLU;
        g.rows = 2 * m->ff_local;
        g.cols = c.n_embd;
        g.x = m->xn;
        g.y = m->act;
        SSD_TRY(launch_matvec(m->ctx, L.wg->type, EPI_SWIGLU, g, s, true));
        nl += 2;
    } else if (is_lowbit(L.wg->type)) {  // low-bit: the FFN norm, gate, up, then SwiGLU
        SSD_REQ(!tp && !pend.on, SSD_ERR_TYPE, "low-bit layer weights run at tp_size 1");
        k_dense_norm<<<1, 1024, 0, s>>>(h, L.ffn_norm, c.n_embd, c.eps, 1, m->xn);
        SSD_CK_LAUNCH();
        float* gate = m->gu;
        float* up = m->gu + m->ff_local;
        SSD_TRY(launch_matvec(m->ctx, L.wg->type, EPI_STORE, mv_plain(L.wg, m->xn, gate), s, true));
        SSD_TRY(launch_matvec(m->ctx, L.wu->type, EPI_STORE, mv_plain(L.wu, m->xn, up), s, true));
        k_swiglu_rows<<<(m->ff_local + 255) / 256, 256, 0, s>>>(gate, up, m->act, m->ff_local);
        SSD_CK_LAUNCH();
        nl += 4;
    } else {
    MvArgs g = {};
    g.qs[0] = L.wg->qs;
    g.qs[1] = L.wu->qs;
    g.meta[0] = L.wg->meta;
    g.meta[1] = L.wu->meta;
    g.seg_rows[0] = m->ff_local;
    g.seg_rows[1] = m->ff_local;
    g.map = MAP_SWIGLU;
    g.rows = 2 * m->ff_local;
    g.cols = c.n_embd;
    g.x = h;
    const bool had_pend2 = pend.on;
    if (had_pend2) {
        take_pending(m, g, pend);
        g.x_writeback = h_other;
    }
    g.norm_w = L.ffn_norm;
    g.eps = c.eps;
    g.norm_order = 1;
    g.y = m->act;
    SSD_TRY(launch_matvec(m->ctx, L.wg->type, EPI_SWIGLU, g, s, true));
    nl++;
    if (had_pend2) {
        h = h_other;
        h_other = (h == m->h_a) ? m->h_b : m->h_a;
    }
    }  // quantized gate / up
    // 6. down projection (+ residual, or a partial sum for the all-reduce)
    MvArgs d = mv_plain(L.wd, m->act, h_other);
    if (tp) {
        SSD_TRY(produce_partial(m, L.wd->type, d, m->p2, use_p2p, 2 * l + 1, pend, s));
    } else {
        d.base = h;
        SSD_TRY(launch_matvec(m->ctx, L.wd->type, EPI_RESID, d, s, true));
        h = h_other;
    }
    nl++;
    return SSD_OK;
}

// Full decode step: embed -> layers -> norm + logits + argmax -> finalize.
static int enqueue_step(ssd_model* m, cudaStream_t s, int& nl, const LayerHooks* hk = nullptr) {
    const auto& c = m->cfg;
    SSD_TRY(launch_embed(m->tok_embd, m->token, m->h_a, s, true));
    nl++;
    float* h = m->h_a;
    Pending pend;
    const bool use_p2p = m->p2p && tp_size(m) > 1;
    for (int l = 0; l < c.n_layers; l++) {
        if (!hk) {
            SSD_TRY(enqueue_layer(m, l, h, pend, use_p2p, s, nl));
            continue;
        }
        // streamed matrices: bound for this layer's enqueue only (the kernels take the
        // pointers by value), so the model never owns them
        ssd_weight* const* w = nullptr;
        SSD_TRY(hk->acquire(hk->user, l, s, w));
        Layer& L = m->layers[l];
        L.wq = w[0], L.wk = w[1], L.wv = w[2], L.wo = w[3], L.wg = w[4], L.wu = w[5], L.wd = w[6];
        const int st = enqueue_layer(m, l, h, pend, use_p2p, s, nl);
        L.wq = L.wk = L.wv = L.wo = L.wg = L.wu = L.wd = nullptr;
        SSD_TRY(st);
        SSD_TRY(hk->release(hk->user, l, s));
    }
    // logits = output * rmsnorm(h) (eps 1e-5 hard-coded at compute.rs:566), argmax
    if (staged_type(m->output->type)) {  // dense / low-bit output (tp_size 1): norm, matvec, key
        SSD_REQ(!pend.on, SSD_ERR_TYPE, "dense / low-bit output weight runs at tp_size 1");
        k_dense_norm<<<1, 1024, 0, s>>>(h, m->out_norm, c.n_embd, 1e-5f, 1, m->xn);
        SSD_CK_LAUNCH();
        SSD_TRY(launch_matvec(m->ctx, m->output->type, EPI_STORE,
                              mv_plain(m->output, m->xn, m->logits), s, true));
        k_argmax_key<<<m->ctx->num_sms, 256, 0, s>>>(m->logits, m->vocab_local,
                                                     (uint32_t)m->vocab0, m->key);
        SSD_CK_LAUNCH();
        nl += 3;
    } else {
        MvArgs a = mv_plain(m->output, h, m->logits);
        take_pending(m, a, pend);
        a.norm_w = m->out_norm;
        a.eps = 1e-5f;
        a.norm_order = 1;
        a.argmax_key = m->key;
        a.index_offset = m->vocab0;
        SSD_TRY(launch_matvec(m->ctx, m->output->type, EPI_ARGMAX, a, s, true));
        nl++;
    }
    if (tp_size(m) > 1)
        SSD_NCCL(ncclAllReduce(m->key, m->key, 1, ncclUint64, ncclMax, m->comm, s));
    SSD_TRY(launch_finalize(m->key, m->token, m->pos, use_p2p ? m->ar_epoch : nullptr,
                            2 * c.n_layers, s, true));
    nl++;
    return SSD_OK;
}

extern "C" int ssd_model_decode_step(ssd_model* m, int use_graph) {
    SSD_REQ(m != nullptr, SSD_ERR_ARG, "null model");
    SSD_TRY(check_ctx(m->ctx));
    SSD_TRY(check_weights(m));
    cudaStream_t s = m->ctx->stream;
    if (!use_graph) {
        int nl = 0;
        SSD_TRY(enqueue_step(m, s, nl));
        m->launches = nl;
        return SSD_OK;
    }
    if (!m->exec) {
        int nl = 0;
        SSD_CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        int st = enqueue_step(m, s, nl);
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamEndCapture(s, &g);
        SSD_TRY(st);
        SSD_CK(e);
        cudaGraphExec_t ex = nullptr;
        e = cudaGraphInstantiate(&ex, g, 0);
        if (e != cudaSuccess) {
            cudaGraphDestroy(g);
            SSD_CK(e);
        }
        m->graph = g;
        m->exec = ex;
        m->launches = nl;
    }
    SSD_CK(cudaGraphLaunch(m->exec, s));
    return SSD_OK;
}

extern "C" int ssd_model_decode_token(ssd_model* m, int32_t token_in, int32_t* token_out,
                                      int use_graph) {
    SSD_REQ(m && token_out, SSD_ERR_ARG, "null argument");
    SSD_TRY(check_ctx(m->ctx));
    SSD_REQ(token_in >= 0 && token_in < m->cfg.vocab, SSD_ERR_ARG, "token %d outside vocab",
            token_in);
    cudaStream_t s = m->ctx->stream;
    m->pinned[0] = token_in;  // the previous call synchronised: the slot is free
    SSD_CK(cudaMemcpyAsync(m->token, &m->pinned[0], 4, cudaMemcpyHostToDevice, s));
    SSD_TRY(ssd_model_decode_step(m, use_graph));
    SSD_CK(cudaMemcpyAsync(&m->pinned[1], m->token, 4, cudaMemcpyDeviceToHost, s));
    SSD_CK(cudaStreamSynchronize(s));
    *token_out = m->pinned[1];
    return SSD_OK;
}

namespace ssd {
ssd_ctx* model_ctx(const ssd_model* m) { return m->ctx; }
bool model_has_layer_matrices(const ssd_model* m) {
    for (const Layer& L : m->layers)
        if (L.wq || L.wk || L.wv || L.wo || L.wg || L.wu || L.wd) return true;
    return false;
}
const ssd_model_config& model_cfg(const ssd_model* m) { return m->cfg; }

int model_decode_token_hooked(ssd_model* m, int32_t token_in, int32_t* token_out,
                              const LayerHooks& hk) {
    SSD_REQ(m && token_out, SSD_ERR_ARG, "null argument");
    SSD_TRY(check_ctx(m->ctx));
    SSD_REQ(tp_size(m) == 1, SSD_ERR_ARG, "the streaming tier runs at tp_size 1");
    SSD_REQ(token_in >= 0 && token_in < m->cfg.vocab, SSD_ERR_ARG, "token %d outside vocab",
            token_in);
    for (int l = 0; l < m->cfg.n_layers; l++)
        SSD_REQ(m->layers[l].attn_norm && m->layers[l].ffn_norm, SSD_ERR_STATE,
                "layer %d norms unset", l);
    SSD_REQ(m->tok_embd && m->output && m->out_norm, SSD_ERR_STATE, "global tensors unset");
    cudaStream_t s = m->ctx->stream;
    m->pinned[0] = token_in;
    SSD_CK(cudaMemcpyAsync(m->token, &m->pinned[0], 4, cudaMemcpyHostToDevice, s));
    int nl = 0;
    SSD_TRY(enqueue_step(m, s, nl, &hk));
    m->launches = nl;
    SSD_CK(cudaMemcpyAsync(&m->pinned[1], m->token, 4, cudaMemcpyDeviceToHost, s));
    SSD_CK(cudaStreamSynchronize(s));
    *token_out = m->pinned[1];
    return SSD_OK;
}
}  // namespace ssd

extern "C" int ssd_model_layer_step(ssd_model* m, int layer) {
    SSD_REQ(m != nullptr, SSD_ERR_ARG, "null model");
    SSD_TRY(check_ctx(m->ctx));
    SSD_REQ(layer >= 0 && layer < m->cfg.n_layers, SSD_ERR_ARG, "layer out of range");
    const Layer& L = m->layers[layer];
    SSD_REQ(L.wq && L.wk && L.wv && L.wo && L.wg && L.wu && L.wd && L.attn_norm && L.ffn_norm,
            SSD_ERR_STATE, "layer %d has unset tensors", layer);
    if (tp_size(m) > 1) SSD_REQ(m->comm != nullptr, SSD_ERR_STATE, "tp_size > 1 needs tp_init");
    cudaStream_t s = m->ctx->stream;
    float* h = m->h_a;
    Pending pend;
    int nl = 0;
    SSD_TRY(enqueue_layer(m, layer, h, pend, false, s, nl));  // NCCL path for partials
    // leave the layer's output in h_a, with any pending partial sum applied
    if (pend.on) {
        k_add<<<(m->cfg.n_embd + 255) / 256, 256, 0, s>>>(m->h_a, h, pend.buf, m->cfg.n_embd);
        SSD_CK_LAUNCH();
    } else if (h != m->h_a) {
        SSD_CK(cudaMemcpyAsync(m->h_a, h, (size_t)m->cfg.n_embd * 4, cudaMemcpyDeviceToDevice, s));
    }
    SSD_CK(cudaStreamSynchronize(s));
    return SSD_OK;
}

extern "C" int ssd_model_launches_per_step(ssd_model* m, int* launches) {
    SSD_REQ(m && launches, SSD_ERR_ARG, "null argument");
    *launches = m->launches;
    return SSD_OK;
}

// ================================================================ batch prefill
// Layer-major batch prefill (batch_prefill_lora, src/inference/transformer.rs:120-250):
// the n prompt tokens go through each layer together, every projection one tensor-core
// GEMM over the n token rows (gemm.cu), attention causal over the INT8 cache.

static int prepare_prefill_weights(ssd_model* m, cudaStream_t s) {
    if (m->pf_walloc) return SSD_OK;
    const auto& c = m->cfg;
    const size_t E = c.n_embd, F = m->ff_local, NQ = (size_t)m->q_rows + 2 * m->kv_rows;
    auto pad = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t per = pad(NQ * E * 2) * 2 + pad(NQ * 4) + pad(E * E * 2) * 2 + pad(E * 4) +
                       pad(2 * F * E * 2) * 2 + pad(2 * F * 4) + pad(E * F * 2) * 2 + pad(E * 4);
    const size_t total = per * c.n_layers;
    if (cudaMalloc(&m->pf_walloc, total) != cudaSuccess) {
        cudaGetLastError();
        m->pf_walloc = nullptr;
        set_error("prefill weight splits (%zu bytes) do not fit", total);
        return SSD_ERR_NOMEM;
    }
    m->pf.assign(c.n_layers, PfLayer{});
    char* p = (char*)m->pf_walloc;
    auto take = [&](size_t b) {
        char* r = p;
        p += pad(b);
        return r;
    };
    for (int l = 0; l < c.n_layers; l++) {
        PfLayer& P = m->pf[l];
        const Layer& L = m->layers[l];
        P.qkv_h = (__half*)take(NQ * E * 2);
        P.qkv_l = (__half*)take(NQ * E * 2);
        P.qkv_r = (float*)take(NQ * 4);
        P.o_h = (__half*)take(E * E * 2);
        P.o_l = (__half*)take(E * E * 2);
        P.o_r = (float*)take(E * 4);
        P.gu_h = (__half*)take(2 * F * E * 2);
        P.gu_l = (__half*)take(2 * F * E * 2);
        P.gu_r = (float*)take(2 * F * 4);
        P.d_h = (__half*)take(E * F * 2);
        P.d_l = (__half*)take(E * F * 2);
        P.d_r = (float*)take(E * 4);
        SSD_TRY(prepare_weight_split(m->ctx, L.wq, 0, 0, 0, 0, P.qkv_h, P.qkv_l, P.qkv_r, s));
        SSD_TRY(prepare_weight_split(m->ctx, L.wk, 0, 0, 0, m->q_rows, P.qkv_h, P.qkv_l, P.qkv_r, s));
        SSD_TRY(prepare_weight_split(m->ctx, L.wv, 0, 0, 0, m->q_rows + m->kv_rows, P.qkv_h,
                                     P.qkv_l, P.qkv_r, s));
        SSD_TRY(prepare_weight_split(m->ctx, L.wo, 0, 0, 0, 0, P.o_h, P.o_l, P.o_r, s));
        SSD_TRY(prepare_weight_split(m->ctx, L.wg, 1, 64, 0, 0, P.gu_h, P.gu_l, P.gu_r, s));
        SSD_TRY(prepare_weight_split(m->ctx, L.wu, 1, 64, 1, 0, P.gu_h, P.gu_l, P.gu_r, s));
        SSD_TRY(prepare_weight_split(m->ctx, L.wd, 0, 0, 0, 0, P.d_h, P.d_l, P.d_r, s));
    }
    return SSD_OK;
}

extern "C" int ssd_model_prefill(ssd_model* m, const int32_t* tokens, int n, int32_t* next_token) {
    SSD_REQ(m && tokens && next_token, SSD_ERR_ARG, "null argument");
    SSD_TRY(check_ctx(m->ctx));
    SSD_TRY(check_weights(m));
    const auto& c = m->cfg;
    SSD_REQ(tp_size(m) == 1, SSD_ERR_STATE, "batch prefill runs at tp_size 1");
    for (const Layer& L : m->layers)
        for (const ssd_weight* w : {L.wq, L.wk, L.wv, L.wo, L.wg, L.wu, L.wd})
            SSD_REQ(!is_lowbit(w->type), SSD_ERR_TYPE,
                    "batch prefill: low-bit layer weights (type %d) run in the decode step only",
                    w->type);
    SSD_REQ(!is_lowbit(m->output->type), SSD_ERR_TYPE,
            "batch prefill: a low-bit output weight runs in the decode step only");
    SSD_REQ(n > 0 && n % 128 == 0, SSD_ERR_SHAPE, "prefill of %d tokens: a multiple of 128", n);
    const int E = c.n_embd, F = m->ff_local, NQ = m->q_rows + 2 * m->kv_rows;
    SSD_REQ(E % 128 == 0 && F % 128 == 0 && NQ % 128 == 0 && m->q_rows == E, SSD_ERR_SHAPE,
            "prefill needs n_embd, n_ff and the QKV rows in multiples of 128");
    for (int i = 0; i < n; i++)
        SSD_REQ(tokens[i] >= 0 && tokens[i] < c.vocab, SSD_ERR_ARG, "token %d outside vocab",
                tokens[i]);
    cudaStream_t s = m->ctx->stream;
    int pos0 = 0;  // after the stream's pending work (a decode step may advance it)
    SSD_CK(cudaMemcpyAsync(&pos0, m->pos, 4, cudaMemcpyDeviceToHost, s));
    SSD_CK(cudaStreamSynchronize(s));
    SSD_REQ(pos0 + n <= c.kv_capacity, SSD_ERR_SHAPE, "positions [%d, %d) exceed capacity %d", pos0,
            pos0 + n, c.kv_capacity);
    SSD_TRY(prepare_prefill_weights(m, s));

    // work buffers
    const size_t KM = (size_t)(F > E ? F : E);
    const size_t pf = (size_t)n * attn_partial_floats(m->nq_local, pos0 + n, c.head_dim);
    auto pad = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t bytes = pad((size_t)n * E * 4) + 2 * pad((size_t)n * KM * 2) +
                         pad((size_t)n * NQ * 4) + pad((size_t)n * m->q_rows * 4) +
                         2 * pad((size_t)n * m->kv_rows * 4) + pad((size_t)n * m->q_rows * 4) +
                         2 * pad((size_t)n * F * 2) + pad(pf * 4) + pad((size_t)n * 4);
    if (bytes > m->pf_buf_bytes) {
        if (m->pf_buf) {
            SSD_CK(cudaStreamSynchronize(s));
            cudaFree(m->pf_buf);
        }
        m->pf_buf = nullptr;
        m->pf_buf_bytes = 0;
        if (cudaMalloc(&m->pf_buf, bytes) != cudaSuccess) {
            cudaGetLastError();
            m->pf_buf = nullptr;
            set_error("prefill buffers (%zu bytes) do not fit", bytes);
            return SSD_ERR_NOMEM;
        }
        m->pf_buf_bytes = bytes;
    }
    char* p = (char*)m->pf_buf;
    auto take = [&](size_t b) {
        char* r = p;
        p += pad(b);
        return r;
    };
    float* H = (float*)take((size_t)n * E * 4);
    __half* Ah = (__half*)take((size_t)n * KM * 2);
    __half* Al = (__half*)take((size_t)n * KM * 2);
    float* QKV = (float*)take((size_t)n * NQ * 4);
    float* Q = (float*)take((size_t)n * m->q_rows * 4);
    float* Kr = (float*)take((size_t)n * m->kv_rows * 4);
    float* Vr = (float*)take((size_t)n * m->kv_rows * 4);
    float* AO = (float*)take((size_t)n * m->q_rows * 4);
    __half* ACTh = (__half*)take((size_t)n * F * 2);  // SwiGLU output, split for the down GEMM
    __half* ACTl = (__half*)take((size_t)n * F * 2);
    float* PART = (float*)take(pf * 4);
    int32_t* TOK = (int32_t*)take((size_t)n * 4);

    SSD_CK(cudaMemcpyAsync(TOK, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, s));
    SSD_TRY(launch_embed_rows(m->tok_embd, TOK, n, H, s));
    GemmOperands op{Ah, Al, nullptr, nullptr};
    for (int l = 0; l < c.n_layers; l++) {
        const Layer& L = m->layers[l];
        const PfLayer& P = m->pf[l];
        // attn_in = rms_norm(h) (transformer.rs:323-326); q, k, v = W attn_in
        SSD_TRY(prepare_act_split(H, n, E, L.attn_norm, c.eps, 0, Ah, Al, s, false));
        GemmArgs g = {};
        g.M = n;
        g.K = E;
        g.N = NQ;
        g.C = QKV;
        g.ldc = NQ;
        g.rscale = P.qkv_r;
        g.epi = GEMM_STORE;
        op.w_hi = P.qkv_h;
        op.w_lo = P.qkv_l;
        SSD_TRY(launch_gemm(m->ctx, op, g, s, false));
        k_prefill_rope<<<n, 256, 0, s>>>(QKV, m->q_rows, m->kv_rows, c.head_dim, c.theta, pos0, Q,
                                         Kr, Vr);
        SSD_CK_LAUNCH();
        // the tokens' K / V rows into the INT8 cache, then causal attention over it
        SSD_TRY(launch_kv_append(L.kv, Kr, Vr, pos0, nullptr, n, s, false));
        AttnArgs at = {};
        at.k = L.kv->k;
        at.v = L.kv->v;
        at.ks = L.kv->k_scale;
        at.vs = L.kv->v_scale;
        at.kv_dim = L.kv->kv_dim;
        at.head_dim = c.head_dim;
        at.group = c.n_head / c.n_head_kv;
        at.kv_head0 = 0;
        at.n_kv_local = m->nkv_local;
        at.q = Q;
        at.out = AO;
        at.partial = PART;
        at.max_seq = pos0 + n;
        at.n_q = n;
        at.q_stride = m->q_rows;
        at.out_stride = m->q_rows;
        at.seq0 = pos0;
        // the tensor-core kernel writes the output as the Wo GEMM's hi / lo operand (the
        // QKV GEMM, the last reader of Ah / Al, precedes it on the stream)
        const bool ao_split = prefill_attention_uses_tc(at);
        if (ao_split) {
            at.out_hi = Ah;
            at.out_lo = Al;
        }
        SSD_TRY(launch_prefill_attention(m->ctx, at, s, false));
        // h += Wo attn (transformer.rs:350-352)
        if (!ao_split) SSD_TRY(prepare_act_split(AO, n, m->q_rows, nullptr, 0.0f, 0, Ah, Al, s, false));
        g.K = m->q_rows;
        g.N = E;
        g.C = H;
        g.ldc = E;
        g.base = H;
        g.ldb = E;
        g.rscale = P.o_r;
        g.epi = GEMM_RESID;
        op.w_hi = P.o_h;
        op.w_lo = P.o_l;
        SSD_TRY(launch_gemm(m->ctx, op, g, s, false));
        // ffn_in = h * inv_rms * w (fused_post_attn_norm, compute.rs:536-555); SwiGLU
        SSD_TRY(prepare_act_split(H, n, E, L.ffn_norm, c.eps, 1, Ah, Al, s, false));
        g.K = E;
        g.N = 2 * F;
        g.C = nullptr;
        g.c_hi = ACTh;  // the epilogue writes act as the down GEMM's hi / lo operand
        g.c_lo = ACTl;
        g.ldc = F;
        g.base = nullptr;
        g.rscale = P.gu_r;
        g.epi = GEMM_SWIGLU;
        op.w_hi = P.gu_h;
        op.w_lo = P.gu_l;
        SSD_TRY(launch_gemm(m->ctx, op, g, s, false));
        // h += down(act) (feed_forward.rs:40-43, transformer.rs:392)
        g.c_hi = g.c_lo = nullptr;
        op.a_hi = ACTh;
        op.a_lo = ACTl;
        g.K = F;
        g.N = E;
        g.C = H;
        g.ldc = E;
        g.base = H;
        g.ldb = E;
        g.rscale = P.d_r;
        g.epi = GEMM_RESID;
        op.w_hi = P.d_h;
        op.w_lo = P.d_l;
        SSD_TRY(launch_gemm(m->ctx, op, g, s, false));
        op.a_hi = Ah;
        op.a_lo = Al;
    }
    // the last token's hidden state is the decode state; logits, greedy argmax, position
    SSD_CK(cudaMemcpyAsync(m->h_a, H + (size_t)(n - 1) * E, (size_t)E * 4, cudaMemcpyDeviceToDevice,
                           s));
    const int last = pos0 + n - 1;
    m->pinned[2] = last;
    SSD_CK(cudaMemcpyAsync(m->pos, &m->pinned[2], 4, cudaMemcpyHostToDevice, s));
    MvArgs a = mv_plain(m->output, m->h_a, m->logits);
    a.norm_w = m->out_norm;
    a.eps = 1e-5f;  // compute.rs:566
    a.norm_order = 1;
    a.argmax_key = m->key;
    a.index_offset = m->vocab0;
    SSD_TRY(launch_matvec(m->ctx, m->output->type, EPI_ARGMAX, a, s, false));
    SSD_TRY(launch_finalize(m->key, m->token, m->pos, nullptr, 0, s, false));
    SSD_CK(cudaMemcpyAsync(&m->pinned[1], m->token, 4, cudaMemcpyDeviceToHost, s));
    SSD_CK(cudaStreamSynchronize(s));
    *next_token = m->pinned[1];
    return SSD_OK;
}


// ====================================================== continuous-batch decode
// BatchScheduler::step (src/inference/batch_scheduler.rs:149-403) runs its decoding
// requests layer-major: each layer's weights are loaded once and applied to every request
// in turn (:236-296), each request with its own KV cache and position. Here the 16 slots of
// a batch go through each layer together: every projection is one batched tensor-core
// matvec over the 16 hidden vectors (matvec_b.cu, the weights streamed once for all), the
// attention one launch over the slots' own INT8 caches (the new K/V rows appended at each
// slot's position inside it). A slot whose request ends is given a new one between steps
// (ssd_batch_set_position + its tokens in the next steps' input), which is the scheduler's
// admission of queued requests (:157-166).

__global__ void k_batch_finalize(unsigned long long* keys, int32_t* tokens, int* pos, int n,
                                 int capacity) {
    pdl_wait();
    const int t = threadIdx.x;
    if (t < n) {
        tokens[t] = (int32_t)(uint32_t)(keys[t] & 0xFFFFFFFFull);
        keys[t] = 0ull;
        pos[t] = pos[t] + 1 < capacity ? pos[t] + 1 : capacity;
    }
}

struct ssd_batch {
    ssd_model* m = nullptr;
    int slots = kBatchTokens, capacity = 0;
    void* alloc = nullptr;
    int8_t *kk = nullptr, *vv = nullptr;  // [layer][slot][capacity][kv_dim]
    float *ks = nullptr, *vs = nullptr;   // [layer][slot][capacity]
    float *h_a = nullptr, *h_b = nullptr, *q = nullptr, *k = nullptr, *v = nullptr;
    float *attn = nullptr, *act = nullptr, *part = nullptr;
    uint8_t* bop = nullptr;
    float* cst = nullptr;
    unsigned int* counter = nullptr;
    float* partial = nullptr;
    int32_t* tokens = nullptr;
    int* pos = nullptr;
    unsigned long long* keys = nullptr;
    float* inv = nullptr;       // [slots] inv_rms of the current RMSNorm
    int32_t* pinned = nullptr;  // [2][slots]: tokens in, tokens out
    size_t part_stride = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int launches = 0;
};

static int batch_check_weight(const ssd_weight* w, const char* what) {
    SSD_REQ(w->type == SSD_TYPE_Q4_0 || w->type == SSD_TYPE_Q8_0 || w->type == SSD_TYPE_Q4_K,
            SSD_ERR_TYPE, "batch decode: %s type %d (Q4_0, Q8_0, Q4_K)", what, w->type);
    SSD_REQ(w->cols % 256 == 0, SSD_ERR_SHAPE, "batch decode: %s cols %d %% 256", what, w->cols);
    return SSD_OK;
}

extern "C" int ssd_batch_create(ssd_model* m, int capacity, ssd_batch** out) {
    SSD_REQ(m && out, SSD_ERR_ARG, "null argument");
    SSD_TRY(check_ctx(m->ctx));
    SSD_TRY(check_weights(m));
    const auto& c = m->cfg;
    SSD_REQ(tp_size(m) == 1, SSD_ERR_ARG, "batch decode runs on one GPU (tp_size 1)");
    SSD_REQ(capacity > 0, SSD_ERR_SHAPE, "capacity %d", capacity);
    SSD_REQ(c.head_dim <= 128 && c.head_dim % 16 == 0, SSD_ERR_SHAPE, "batch decode: head_dim %d",
            c.head_dim);
    SSD_REQ(m->q_rows % 128 == 0 && m->kv_rows % 128 == 0 && m->ff_local % 64 == 0, SSD_ERR_SHAPE,
            "batch decode: q / kv rows multiples of 128, n_ff of 64");
    for (int l = 0; l < c.n_layers; l++) {
        const Layer& L = m->layers[l];
        for (const ssd_weight* w : {L.wq, L.wk, L.wv, L.wo, L.wg, L.wu, L.wd})
            SSD_TRY(batch_check_weight(w, "layer weight"));
        SSD_REQ(L.wq->type == L.wk->type && L.wk->type == L.wv->type && L.wg->type == L.wu->type,
                SSD_ERR_TYPE, "batch decode: fused QKV / gate-up weights of one type");
    }
    SSD_TRY(batch_check_weight(m->output, "output"));
    ssd_batch* b = new ssd_batch();
    b->m = m;
    b->capacity = capacity;
    const int S = b->slots, E = c.n_embd, kvd = m->kv_rows, Q = m->q_rows, F = m->ff_local;
    const int maxc = E > F ? (E > Q ? E : Q) : (F > Q ? F : Q);
    b->part_stride = attn_partial_floats(m->nq_local, capacity, c.head_dim);
    auto pad = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t kvb = (size_t)c.n_layers * S * capacity * kvd;
    const size_t scb = (size_t)c.n_layers * S * capacity * 4;
    const int max_tiles = 2 * ((F > c.vocab ? F : c.vocab) / 64 + 16);
    size_t off[24], o = 0;
    int i = 0;
    auto take = [&](size_t bytes) { off[i++] = o; o += pad(bytes); };
    take(kvb);                                   // 0 kk
    take(kvb);                                   // 1 vv
    take(scb);                                   // 2 ks
    take(scb);                                   // 3 vs
    take((size_t)S * E * 4);                     // 4 h_a
    take((size_t)S * E * 4);                     // 5 h_b
    take((size_t)S * Q * 4);                     // 6 q
    take((size_t)S * kvd * 4);                   // 7 k
    take((size_t)S * kvd * 4);                   // 8 v
    take((size_t)S * Q * 4);                     // 9 attn
    take((size_t)S * F * 4);                     // 10 act
    take((size_t)S * b->part_stride * 4);        // 11 attention partials
    take((size_t)(maxc / 256) * 16384);          // 12 B operand
    take((size_t)(maxc / 256) * 1024);           // 13 B scale tables
    take((size_t)max_tiles * 4);                 // 14 counters
    take((size_t)kI8MaxGrid * 2 * S * 128 * 4);  // 15 split-K partials
    take((size_t)S * 4);                         // 16 tokens
    take((size_t)S * 4);                         // 17 positions
    take((size_t)S * 8);                         // 18 keys
    take((size_t)S * 4);                         // 19 inv_rms per slot
    if (cudaMalloc(&b->alloc, o) != cudaSuccess) {
        cudaGetLastError();
        delete b;
        set_error("batch allocation of %zu bytes failed", o);
        return SSD_ERR_NOMEM;
    }
    uint8_t* p = (uint8_t*)b->alloc;
    b->kk = (int8_t*)(p + off[0]);
    b->vv = (int8_t*)(p + off[1]);
    b->ks = (float*)(p + off[2]);
    b->vs = (float*)(p + off[3]);
    b->h_a = (float*)(p + off[4]);
    b->h_b = (float*)(p + off[5]);
    b->q = (float*)(p + off[6]);
    b->k = (float*)(p + off[7]);
    b->v = (float*)(p + off[8]);
    b->attn = (float*)(p + off[9]);
    b->act = (float*)(p + off[10]);
    b->part = (float*)(p + off[11]);
    b->bop = p + off[12];
    b->cst = (float*)(p + off[13]);
    b->counter = (unsigned*)(p + off[14]);
    b->partial = (float*)(p + off[15]);
    b->tokens = (int32_t*)(p + off[16]);
    b->pos = (int*)(p + off[17]);
    b->keys = (unsigned long long*)(p + off[18]);
    b->inv = (float*)(p + off[19]);
    int st = SSD_OK;
    if (zero_device(m->ctx, b->alloc, o) != SSD_OK ||
        cudaMallocHost(&b->pinned, (size_t)2 * S * 4) != cudaSuccess) {
        cudaGetLastError();
        set_error("batch initialisation failed");
        st = SSD_ERR_CUDA;
    }
    if (st != SSD_OK) {
        cudaFree(b->alloc);
        delete b;
        return st;
    }
    *out = b;
    return SSD_OK;
}

extern "C" int ssd_batch_free(ssd_batch* b) {
    if (!b) return SSD_OK;
    cudaSetDevice(b->m->ctx->device);
    cudaStreamSynchronize(b->m->ctx->stream);
    if (b->exec) cudaGraphExecDestroy(b->exec);
    if (b->graph) cudaGraphDestroy(b->graph);
    if (b->pinned) cudaFreeHost(b->pinned);
    cudaFree(b->alloc);
    delete b;
    return SSD_OK;
}

extern "C" int ssd_batch_slots(ssd_batch* b, int* slots) {
    SSD_REQ(b && slots, SSD_ERR_ARG, "null argument");
    *slots = b->slots;
    return SSD_OK;
}

// The cache of (layer, slot) as a view (no allocation of its own).
static ssd_kv_cache batch_kv_view(ssd_batch* b, int layer, int slot) {
    const auto& c = b->m->cfg;
    ssd_kv_cache kv;
    kv.ctx = b->m->ctx;
    kv.capacity = b->capacity;
    kv.n_head_kv = c.n_head_kv;
    kv.head_dim = c.head_dim;
    kv.kv_dim = b->m->kv_rows;
    const size_t ls = (size_t)layer * b->slots + slot;
    kv.k = b->kk + ls * b->capacity * kv.kv_dim;
    kv.v = b->vv + ls * b->capacity * kv.kv_dim;
    kv.k_scale = b->ks + ls * b->capacity;
    kv.v_scale = b->vs + ls * b->capacity;
    return kv;
}

extern "C" int ssd_batch_kv_pointers(ssd_batch* b, int layer, int slot, int8_t** k, int8_t** v,
                                     float** ks, float** vs) {
    SSD_REQ(b && layer >= 0 && layer < b->m->cfg.n_layers && slot >= 0 && slot < b->slots,
            SSD_ERR_ARG, "bad arguments");
    const ssd_kv_cache kv = batch_kv_view(b, layer, slot);
    if (k) *k = kv.k;
    if (v) *v = kv.v;
    if (ks) *ks = kv.k_scale;
    if (vs) *vs = kv.v_scale;
    return SSD_OK;
}

extern "C" int ssd_batch_set_position(ssd_batch* b, int slot, int pos) {
    SSD_REQ(b && slot >= 0 && slot < b->slots, SSD_ERR_ARG, "bad slot");
    SSD_TRY(check_ctx(b->m->ctx));
    SSD_REQ(pos >= 0 && pos < b->capacity, SSD_ERR_SHAPE, "position %d outside [0, %d)", pos,
            b->capacity);
    SSD_CK(cudaMemcpyAsync(b->pos + slot, &pos, 4, cudaMemcpyHostToDevice, b->m->ctx->stream));
    SSD_CK(cudaStreamSynchronize(b->m->ctx->stream));
    return SSD_OK;
}

extern "C" int ssd_batch_positions(ssd_batch* b, int* pos) {
    SSD_REQ(b && pos, SSD_ERR_ARG, "null argument");
    SSD_TRY(check_ctx(b->m->ctx));
    SSD_CK(cudaMemcpyAsync(pos, b->pos, (size_t)b->slots * 4, cudaMemcpyDeviceToHost,
                           b->m->ctx->stream));
    SSD_CK(cudaStreamSynchronize(b->m->ctx->stream));
    return SSD_OK;
}

extern "C" int ssd_batch_synth_kv(ssd_batch* b, uint64_t seed, int n) {
    SSD_REQ(b != nullptr, SSD_ERR_ARG, "null batch");
    ssd_model* m = b->m;
    SSD_TRY(check_ctx(m->ctx));
    SSD_REQ(n >= 0 && n < b->capacity, SSD_ERR_SHAPE, "n %d outside [0, %d)", n, b->capacity);
    const int kvd = m->kv_rows;
    cudaStream_t s = m->ctx->stream;
    if (n > 0) {
        const int chunk = 1024;
        float* tmp = nullptr;
        SSD_CK(cudaMalloc(&tmp, (size_t)2 * chunk * kvd * 4));
        int st = SSD_OK;
        for (int l = 0; l < m->cfg.n_layers && st == SSD_OK; l++) {
            for (int sl = 0; sl < b->slots && st == SSD_OK; sl++) {
                ssd_kv_cache kv = batch_kv_view(b, l, sl);
                for (int p0 = 0; p0 < n && st == SSD_OK; p0 += chunk) {
                    const int rows = n - p0 < chunk ? n - p0 : chunk;
                    // K / V rows N(0, 1): tensors 3000000 + 128 l + 2 slot (+1)
                    const uint32_t tk = 3000000u + 128u * l + 2u * sl;
                    st = ssd_synth_f32(m->ctx, seed, tk, 0.0f, 1.0f, kvd, p0, rows, 0, kvd, tmp,
                                       (void*)s);
                    if (st == SSD_OK)
                        st = ssd_synth_f32(m->ctx, seed, tk + 1, 0.0f, 1.0f, kvd, p0, rows, 0, kvd,
                                           tmp + (size_t)chunk * kvd, (void*)s);
                    if (st == SSD_OK)
                        st = launch_kv_append(&kv, tmp, tmp + (size_t)chunk * kvd, p0, nullptr, rows,
                                              s, false);
                }
            }
        }
        cudaStreamSynchronize(s);
        cudaFree(tmp);
        SSD_TRY(st);
    }
    for (int sl = 0; sl < b->slots; sl++) SSD_TRY(ssd_batch_set_position(b, sl, n));
    return SSD_OK;
}

// One batched matvec: B operand from x (+ norm), then the tensor-core launch.
static int batch_mv(ssd_batch* b, const ssd_weight* w0, int epi, MvArgs a, const float* x, int ldx,
                    const float* norm_w, float eps, int norm_order, int ldy, cudaStream_t s,
                    int& nl) {
    ssd_ctx* ctx = b->m->ctx;
    BPrepArgs p = {};
    p.x = x;
    p.ldx = ldx;
    p.cols = a.cols;
    p.norm_w = norm_w;
    p.eps = eps;
    p.norm_order = norm_order;
    p.b = b->bop;
    p.cst = b->cst;
    p.inv = b->inv;
    SSD_TRY(launch_bprep(ctx, w0->type, p, s, true));
    if (norm_w) nl++;
    BWork wk = {};
    wk.b = b->bop;
    wk.cst = b->cst;
    wk.counter = b->counter;
    wk.partial = b->partial;
    wk.ldy = ldy;
    wk.ldk = b->m->kv_rows;
    wk.pos = b->pos;
    wk.keys = b->keys;
    SSD_TRY(launch_matvec_batch(ctx, w0->type, epi, a, wk, s, true));
    nl += 2;
    return SSD_OK;
}

static int enqueue_batch_step(ssd_batch* b, cudaStream_t s, int& nl) {
    ssd_model* m = b->m;
    const auto& c = m->cfg;
    const int S = b->slots, E = c.n_embd;
    SSD_TRY(launch_embed_rows(m->tok_embd, b->tokens, S, b->h_a, s));
    nl++;
    float* h = b->h_a;
    float* ho = b->h_b;
    for (int l = 0; l < c.n_layers; l++) {
        const Layer& L = m->layers[l];
        // QKV + RoPE (each slot at its own position), pre-attention RMSNorm in the B prep
        MvArgs a = {};
        a.qs[0] = L.wq->qs;
        a.qs[1] = L.wk->qs;
        a.qs[2] = L.wv->qs;
        a.meta[0] = L.wq->meta;
        a.meta[1] = L.wk->meta;
        a.meta[2] = L.wv->meta;
        a.seg_rows[0] = m->q_rows;
        a.seg_rows[1] = m->kv_rows;
        a.seg_rows[2] = m->kv_rows;
        a.map = MAP_QKV;
        a.rows = m->q_rows + 2 * m->kv_rows;
        a.cols = E;
        a.y = b->q;
        a.y_k = b->k;
        a.y_v = b->v;
        a.head_dim = c.head_dim;
        a.theta = c.theta;
        a.rope_cache = m->rope;
        a.rope_rows = c.kv_capacity;
        SSD_TRY(batch_mv(b, L.wq, EPI_QKV_ROPE, a, h, E, L.attn_norm, c.eps, 0, m->q_rows, s, nl));
        // attention over each slot's cache, its new K / V row appended at its position
        ssd_kv_cache kv0 = batch_kv_view(b, l, 0);
        AttnArgs at = {};
        at.k_new = b->k;
        at.v_new = b->v;
        at.k = kv0.k;
        at.v = kv0.v;
        at.ks = kv0.k_scale;
        at.vs = kv0.v_scale;
        at.kv_dim = m->kv_rows;
        at.head_dim = c.head_dim;
        at.group = c.n_head / c.n_head_kv;
        at.kv_head0 = 0;
        at.n_kv_local = m->nkv_local;
        at.q = b->q;
        at.out = b->attn;
        at.partial = b->part;
        at.pos_dev = b->pos;
        at.max_seq = b->capacity;
        at.n_q = S;
        at.q_stride = m->q_rows;
        at.out_stride = m->q_rows;
        at.n_slots = S;
        at.slot_kv = (size_t)b->capacity * m->kv_rows;
        at.slot_sc = b->capacity;
        at.slot_new = m->kv_rows;
        SSD_TRY(launch_attention(at, s, true));
        nl += 2;
        // o_proj + residual
        MvArgs o = mv_plain(L.wo, nullptr, ho);
        o.base = h;
        SSD_TRY(batch_mv(b, L.wo, EPI_RESID, o, b->attn, m->q_rows, nullptr, 0.0f, 0, E, s, nl));
        std::swap(h, ho);
        // gate / up + SwiGLU, FFN RMSNorm in the B prep
        MvArgs g = {};
        g.qs[0] = L.wg->qs;
        g.qs[1] = L.wu->qs;
        g.meta[0] = L.wg->meta;
        g.meta[1] = L.wu->meta;
        g.seg_rows[0] = m->ff_local;
        g.seg_rows[1] = m->ff_local;
        g.map = MAP_SWIGLU;
        g.rows = 2 * m->ff_local;
        g.cols = E;
        g.y = b->act;
        SSD_TRY(batch_mv(b, L.wg, EPI_SWIGLU, g, h, E, L.ffn_norm, c.eps, 1, m->ff_local, s, nl));
        // down + residual
        MvArgs d = mv_plain(L.wd, nullptr, ho);
        d.base = h;
        SSD_TRY(batch_mv(b, L.wd, EPI_RESID, d, b->act, m->ff_local, nullptr, 0.0f, 0, E, s, nl));
        std::swap(h, ho);
    }
    // logits = output * rmsnorm(h) (eps 1e-5, compute.rs:566), argmax per slot
    MvArgs a = mv_plain(m->output, nullptr, nullptr);
    a.y = nullptr;
    a.index_offset = 0;
    SSD_TRY(batch_mv(b, m->output, EPI_ARGMAX, a, h, E, m->out_norm, 1e-5f, 1, c.vocab, s, nl));
    SSD_CK(launch_pdl(k_batch_finalize, dim3(1), dim3(32), 0, s, true, b->keys, b->tokens, b->pos,
                      S, b->capacity));
    nl++;
    return SSD_OK;
}

// One decode step of every slot: tokens_in (host, one per slot, or null to continue from
// each slot's last output) -> next tokens (host, may be null). Graph-captured on first use.
extern "C" int ssd_batch_step(ssd_batch* b, const int32_t* tokens_in, int32_t* tokens_out,
                              int use_graph) {
    SSD_REQ(b != nullptr, SSD_ERR_ARG, "null batch");
    ssd_model* m = b->m;
    SSD_TRY(check_ctx(m->ctx));
    const int S = b->slots;
    cudaStream_t s = m->ctx->stream;
    if (tokens_in) {
        for (int i = 0; i < S; i++)
            SSD_REQ(tokens_in[i] >= 0 && tokens_in[i] < m->cfg.vocab, SSD_ERR_ARG,
                    "slot %d token %d outside vocab", i, tokens_in[i]);
        memcpy(b->pinned, tokens_in, (size_t)S * 4);  // the previous call synchronised
        SSD_CK(cudaMemcpyAsync(b->tokens, b->pinned, (size_t)S * 4, cudaMemcpyHostToDevice, s));
    }
    if (!use_graph) {
        int nl = 0;
        SSD_TRY(enqueue_batch_step(b, s, nl));
        b->launches = nl;
    } else {
        if (!b->exec) {
            int nl = 0;
            SSD_CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
            int st = enqueue_batch_step(b, s, nl);
            cudaGraph_t g = nullptr;
            cudaError_t e = cudaStreamEndCapture(s, &g);
            SSD_TRY(st);
            SSD_CK(e);
            cudaGraphExec_t ex = nullptr;
            e = cudaGraphInstantiate(&ex, g, 0);
            if (e != cudaSuccess) {
                cudaGraphDestroy(g);
                SSD_CK(e);
            }
            b->graph = g;
            b->exec = ex;
            b->launches = nl;
        }
        SSD_CK(cudaGraphLaunch(b->exec, s));
    }
    if (tokens_out) {
        SSD_CK(cudaMemcpyAsync(b->pinned + S, b->tokens, (size_t)S * 4, cudaMemcpyDeviceToHost, s));
        SSD_CK(cudaStreamSynchronize(s));
        memcpy(tokens_out, b->pinned + S, (size_t)S * 4);
    }
    return SSD_OK;
}

extern "C" int ssd_batch_launches_per_step(ssd_batch* b, int* launches) {
    SSD_REQ(b && launches, SSD_ERR_ARG, "null argument");
    *launches = b->launches;
    return SSD_OK;
}

extern "C" int ssd_batch_state(ssd_batch* b, float** hidden) {
    SSD_REQ(b && hidden, SSD_ERR_ARG, "null argument");
    *hidden = b->h_a;  // after a step with an even number of swaps per layer
    return SSD_OK;
}
