// host.cu — the host-slice operators of MetalCompute (src/metal/compute.rs:145-375) and
// MetalGpu::feed_forward_f32 (src/metal/gpu.rs:789-838), plus the windowed attention over
// f32 K/V rows that flash_attention_f32 needs.
//
// Every *_host call takes host slices exactly as the reference method does: it stages the
// inputs in the context's scratch (one region per operand, 256-byte aligned), runs the
// device kernels on the context's stream, copies the results back and synchronises. The
// weights of the f32 calls are host slices too (the reference uploads them per call,
// gpu.rs:169-205), so they are copied per call; a caller that keeps weights resident
// uploads them once with ssd_weight_upload and uses the device-pointer entry points.
#include "common.cuh"
#include "matvec.cuh"
#include "matvec_dev.cuh"

namespace ssd {

// ---------------------------------------------------------------- f32 attention

constexpr int kFaWarps = 4;
constexpr int kFaMaxDim = 256;  // the shader's accumulator bound (kernels.metal:1385-1386)
constexpr int kFaMaxSplit = 64;

struct FaArgs {
    const float* q;  // [n_head][head_dim]
    const float* k;  // [seq][n_head_kv * head_dim]
    const float* v;
    float* out;      // [n_head][head_dim]
    float* partial;  // [n_head][n_split][head_dim + 2] (m, l, acc) when n_split > 1
    int n_head, n_head_kv, head_dim, group;
    int p0, p1;      // window [p0, p1)
    int chunk;       // positions per split
    float scale;
};

// One CTA per (head, split): its warps take the split's positions round-robin, four at a
// time, lane l holding dims l, l + 32, ... of q, of the K / V rows and of the accumulator.
// Online softmax per warp (running max m, running sum l, accumulator rescaled when m
// grows), then the warps' states are merged in shared memory into the split's (m, l, acc).
template <int DJ>
__global__ void __launch_bounds__(kFaWarps * 32) k_fa_f32(const FaArgs a) {
    __shared__ float sm_m[kFaWarps], sm_l[kFaWarps];
    __shared__ float sm_acc[kFaWarps][DJ * 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int h = blockIdx.x, split = blockIdx.y;
    const int kvh = h / a.group;
    const int kv_dim = a.n_head_kv * a.head_dim;
    const int s0 = a.p0 + split * a.chunk;
    const int s1 = min(a.p1, s0 + a.chunk);
    float q[DJ], acc[DJ];
#pragma unroll
    for (int j = 0; j < DJ; j++) {
        const int d = lane + 32 * j;
        q[j] = d < a.head_dim ? a.q[(size_t)h * a.head_dim + d] * a.scale : 0.0f;
        acc[j] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    const float* kb = a.k + (size_t)kvh * a.head_dim;
    const float* vb = a.v + (size_t)kvh * a.head_dim;
    constexpr int P = 4;
    for (int p = s0 + warp * P; p < s1; p += kFaWarps * P) {
        float sc[P];
#pragma unroll
        for (int i = 0; i < P; i++) {
            float dot = 0.0f;
            if (p + i < s1) {
                const float* kr = kb + (size_t)(p + i) * kv_dim;
#pragma unroll
                for (int j = 0; j < DJ; j++) {
                    const int d = lane + 32 * j;
                    if (d < a.head_dim) dot = fmaf(q[j], __ldg(kr + d), dot);
                }
            }
            sc[i] = dot;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int i = 0; i < P; i++) sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], off);
        float mn = m;
#pragma unroll
        for (int i = 0; i < P; i++)
            if (p + i < s1) mn = fmaxf(mn, sc[i]);
        const float corr = m == -INFINITY ? 0.0f : expf(m - mn);
        l *= corr;
#pragma unroll
        for (int j = 0; j < DJ; j++) acc[j] *= corr;
        m = mn;
#pragma unroll
        for (int i = 0; i < P; i++) {
            if (p + i >= s1) break;
            const float wgt = expf(sc[i] - m);
            l += wgt;
            const float* vr = vb + (size_t)(p + i) * kv_dim;
#pragma unroll
            for (int j = 0; j < DJ; j++) {
                const int d = lane + 32 * j;
                if (d < a.head_dim) acc[j] = fmaf(wgt, __ldg(vr + d), acc[j]);
            }
        }
    }
    if (lane == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
    }
#pragma unroll
    for (int j = 0; j < DJ; j++) sm_acc[warp][lane + 32 * j] = acc[j];
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kFaWarps; w++) M = fmaxf(M, sm_m[w]);
    float L = 0.0f, f[kFaWarps];
#pragma unroll
    for (int w = 0; w < kFaWarps; w++) {
        f[w] = sm_m[w] == -INFINITY ? 0.0f : expf(sm_m[w] - M);
        L += sm_l[w] * f[w];
    }
    const bool direct = gridDim.y == 1;
    float* dst = direct ? a.out + (size_t)h * a.head_dim
                        : a.partial + ((size_t)h * gridDim.y + split) * (a.head_dim + 2);
    for (int d = threadIdx.x; d < a.head_dim; d += blockDim.x) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kFaWarps; w++) s += sm_acc[w][d] * f[w];
        if (direct)
            dst[d] = L > 0.0f ? s / L : 0.0f;  // empty window: zeros (kernels.metal:1435-1438)
        else
            dst[2 + d] = s;
    }
    if (!direct && threadIdx.x == 0) {
        dst[0] = M;
        dst[1] = L;
    }
}

// Merge of the splits of one head: out = sum_s acc_s e^(m_s - M) / sum_s l_s e^(m_s - M).
__global__ void k_fa_f32_combine(const FaArgs a, int n_split) {
    const int h = blockIdx.x;
    const float* base = a.partial + (size_t)h * n_split * (a.head_dim + 2);
    float M = -INFINITY;
    for (int s = 0; s < n_split; s++) M = fmaxf(M, base[(size_t)s * (a.head_dim + 2)]);
    float L = 0.0f;
    for (int s = 0; s < n_split; s++) {
        const float* ps = base + (size_t)s * (a.head_dim + 2);
        if (ps[0] != -INFINITY) L += ps[1] * expf(ps[0] - M);
    }
    for (int d = threadIdx.x; d < a.head_dim; d += blockDim.x) {
        float acc = 0.0f;
        for (int s = 0; s < n_split; s++) {
            const float* ps = base + (size_t)s * (a.head_dim + 2);
            if (ps[0] != -INFINITY) acc += ps[2 + d] * expf(ps[0] - M);
        }
        a.out[(size_t)h * a.head_dim + d] = L > 0.0f ? acc / L : 0.0f;
    }
}

static int fa_splits(const ssd_ctx* ctx, int n_head, int len) {
    int want = (2 * ctx->num_sms + n_head - 1) / n_head;
    int by_len = (len + 63) / 64;
    int n = want < by_len ? want : by_len;
    if (n > kFaMaxSplit) n = kFaMaxSplit;
    return n < 1 ? 1 : n;
}

static size_t fa_partial_bytes(int n_head, int n_split, int head_dim) {
    return n_split > 1 ? (size_t)n_head * n_split * (head_dim + 2) * 4 : 0;
}

static int fa_check(int n_head, int n_head_kv, int head_dim, int seq_len, int ws, int we) {
    SSD_REQ(n_head > 0 && n_head_kv > 0 && n_head % n_head_kv == 0, SSD_ERR_SHAPE,
            "n_head %d must be a positive multiple of n_head_kv %d", n_head, n_head_kv);
    SSD_REQ(head_dim > 0 && head_dim <= kFaMaxDim, SSD_ERR_SHAPE, "head_dim %d outside (0, %d]",
            head_dim, kFaMaxDim);
    SSD_REQ(seq_len >= 0 && ws >= 0 && we >= 0, SSD_ERR_ARG, "negative length or window");
    return SSD_OK;
}

static int launch_fa_f32(ssd_ctx* ctx, const float* q, const float* k, const float* v,
                         int n_head, int n_head_kv, int head_dim, int seq_len, int ws, int we,
                         float* out, float* partial, int n_split, cudaStream_t s) {
    FaArgs a;
    a.q = q;
    a.k = k;
    a.v = v;
    a.out = out;
    a.partial = partial;
    a.n_head = n_head;
    a.n_head_kv = n_head_kv;
    a.head_dim = head_dim;
    a.group = n_head / n_head_kv;
    a.p0 = ws;
    a.p1 = we < seq_len ? we : seq_len;
    if (a.p1 < a.p0) a.p1 = a.p0;
    const int len = a.p1 - a.p0;
    a.chunk = (len + n_split - 1) / n_split;
    if (a.chunk < 1) a.chunk = 1;
    a.scale = 1.0f / sqrtf((float)head_dim);
    const dim3 grid(n_head, n_split);
    const int dj = (head_dim + 31) / 32;
    if (dj <= 2)
        k_fa_f32<2><<<grid, kFaWarps * 32, 0, s>>>(a);
    else if (dj <= 4)
        k_fa_f32<4><<<grid, kFaWarps * 32, 0, s>>>(a);
    else
        k_fa_f32<8><<<grid, kFaWarps * 32, 0, s>>>(a);
    SSD_CK_LAUNCH();
    if (n_split > 1) {
        k_fa_f32_combine<<<n_head, head_dim < 128 ? 128 : 256, 0, s>>>(a, n_split);
        SSD_CK_LAUNCH();
    }
    return SSD_OK;
}

// ---------------------------------------------------------------- helpers

// out = x * inv_rms * w, inv_rms over n elements (fused_rmsnorm_linear_f32_cpu,
// src/metal/compute.rs:557-578: (x * inv_rms) * w, eps 1e-5).
__global__ void __launch_bounds__(1024) k_norm_into(const float* x, const float* w, int n,
                                                    float eps, float* out) {
    __shared__ float red[32];
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += 1024) ss = fmaf(x[i], x[i], ss);
    ss = block_sum<1024>(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += 1024) out[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

// Carves 256-byte-aligned regions out of the context scratch.
struct Stage {
    size_t off = 0;
    size_t take(size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) & ~(size_t)255;
        return o;
    }
};

static int h2d(ssd_ctx* ctx, void* dst, const void* src, size_t bytes) {
    if (bytes) SSD_CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    return SSD_OK;
}

static int d2h(ssd_ctx* ctx, void* dst, const void* src, size_t bytes) {
    if (bytes) SSD_CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    return SSD_OK;
}

static int finish(ssd_ctx* ctx, const char* what) {
    const cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        set_error("%s: %s", what, cudaGetErrorString(e));
        return SSD_ERR_CUDA;
    }
    return SSD_OK;
}

static float* at(ssd_ctx* ctx, size_t off) {
    return reinterpret_cast<float*>(static_cast<char*>(ctx->scratch) + off);
}

// y = W x over a dense f32 W already on the device.
static int dense_f32(ssd_ctx* ctx, const float* w, const float* x, float* y, int rows, int cols) {
    MvArgs a = {};
    a.qs[0] = reinterpret_cast<const uint8_t*>(w);
    a.seg_rows[0] = rows;
    a.map = MAP_PLAIN;
    a.rows = rows;
    a.cols = cols;
    a.x = x;
    a.y = y;
    return launch_matvec(ctx, SSD_TYPE_F32, EPI_STORE, a, ctx->stream, false);
}

}  // namespace ssd

using namespace ssd;

extern "C" int ssd_flash_attention_f32(ssd_ctx* ctx, const float* q, const float* k,
                                       const float* v, int n_head, int n_head_kv, int head_dim,
                                       int seq_len, int window_start, int window_end, float* out,
                                       void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(q && out && (seq_len == 0 || (k && v)), SSD_ERR_ARG, "null pointer");
    SSD_TRY(fa_check(n_head, n_head_kv, head_dim, seq_len, window_start, window_end));
    const int end = window_end < seq_len ? window_end : seq_len;
    const int len = end > window_start ? end - window_start : 0;
    const int n_split = fa_splits(ctx, n_head, len);
    float* partial = nullptr;
    if (n_split > 1) {
        SSD_TRY(ensure_scratch(ctx, fa_partial_bytes(n_head, n_split, head_dim)));
        partial = static_cast<float*>(ctx->scratch);
    }
    return launch_fa_f32(ctx, q, k, v, n_head, n_head_kv, head_dim, seq_len, window_start,
                         window_end, out, partial, n_split, pick_stream(ctx, stream));
}

extern "C" int ssd_flash_attention_f32_host(ssd_ctx* ctx, const float* q, const float* k,
                                            const float* v, int n_head, int n_head_kv,
                                            int head_dim, int seq_len, int window_start,
                                            int window_end, float* out) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(q && out && (seq_len == 0 || (k && v)), SSD_ERR_ARG, "null pointer");
    SSD_TRY(fa_check(n_head, n_head_kv, head_dim, seq_len, window_start, window_end));
    const int end = window_end < seq_len ? window_end : seq_len;
    const int len = end > window_start ? end - window_start : 0;
    const int n_split = fa_splits(ctx, n_head, len);
    const size_t qb = (size_t)n_head * head_dim * 4;
    // only the window's rows travel: rows [window_start, end) of K and V
    const size_t row = (size_t)n_head_kv * head_dim * 4;
    const size_t kvb = (size_t)len * row;
    Stage st;
    const size_t oq = st.take(qb), ok = st.take(kvb), ov = st.take(kvb), oo = st.take(qb),
                 op = st.take(fa_partial_bytes(n_head, n_split, head_dim));
    SSD_TRY(ensure_scratch(ctx, st.off));
    SSD_TRY(h2d(ctx, at(ctx, oq), q, qb));
    if (len) {
        SSD_TRY(h2d(ctx, at(ctx, ok), k + (size_t)window_start * n_head_kv * head_dim, kvb));
        SSD_TRY(h2d(ctx, at(ctx, ov), v + (size_t)window_start * n_head_kv * head_dim, kvb));
    }
    // the staged rows start at the window: positions [0, len)
    SSD_TRY(launch_fa_f32(ctx, at(ctx, oq), at(ctx, ok), at(ctx, ov), n_head, n_head_kv,
                          head_dim, len, 0, len, at(ctx, oo), at(ctx, op), n_split, ctx->stream));
    SSD_TRY(d2h(ctx, out, at(ctx, oo), qb));
    return finish(ctx, "flash_attention_f32");
}

extern "C" int ssd_matvec_f32_host(ssd_ctx* ctx, const float* w, const float* x, float* y,
                                   int out_dim, int in_dim) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(w && x && y, SSD_ERR_ARG, "null pointer");
    SSD_REQ(out_dim > 0 && in_dim > 0, SSD_ERR_SHAPE, "empty matrix %dx%d", out_dim, in_dim);
    Stage st;
    const size_t ow = st.take((size_t)out_dim * in_dim * 4), ox = st.take((size_t)in_dim * 4),
                 oy = st.take((size_t)out_dim * 4);
    SSD_TRY(ensure_scratch(ctx, st.off));
    SSD_TRY(h2d(ctx, at(ctx, ow), w, (size_t)out_dim * in_dim * 4));
    SSD_TRY(h2d(ctx, at(ctx, ox), x, (size_t)in_dim * 4));
    SSD_TRY(dense_f32(ctx, at(ctx, ow), at(ctx, ox), at(ctx, oy), out_dim, in_dim));
    SSD_TRY(d2h(ctx, y, at(ctx, oy), (size_t)out_dim * 4));
    return finish(ctx, "matvec_f32");
}

static int qkv_host(ssd_ctx* ctx, const float* wq, const float* wk, const float* wv,
                    const float* x, int q_dim, int kv_dim, int n_embd, int head_dim,
                    int position, float theta, bool rope, float* q, float* k, float* v) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(wq && wk && wv && x && q && k && v, SSD_ERR_ARG, "null pointer");
    SSD_REQ(q_dim > 0 && kv_dim > 0 && n_embd > 0, SSD_ERR_SHAPE, "empty projection");
    SSD_REQ(!rope || (head_dim > 1 && q_dim % head_dim == 0 && kv_dim % head_dim == 0),
            SSD_ERR_SHAPE, "head_dim %d must divide q_dim %d and kv_dim %d", head_dim, q_dim,
            kv_dim);
    const size_t wqb = (size_t)q_dim * n_embd * 4, wkb = (size_t)kv_dim * n_embd * 4;
    Stage st;
    const size_t owq = st.take(wqb), owk = st.take(wkb), owv = st.take(wkb),
                 ox = st.take((size_t)n_embd * 4), oq = st.take((size_t)q_dim * 4),
                 ok = st.take((size_t)kv_dim * 4), ov = st.take((size_t)kv_dim * 4);
    SSD_TRY(ensure_scratch(ctx, st.off));
    SSD_TRY(h2d(ctx, at(ctx, owq), wq, wqb));
    SSD_TRY(h2d(ctx, at(ctx, owk), wk, wkb));
    SSD_TRY(h2d(ctx, at(ctx, owv), wv, wkb));
    SSD_TRY(h2d(ctx, at(ctx, ox), x, (size_t)n_embd * 4));
    SSD_TRY(dense_f32(ctx, at(ctx, owq), at(ctx, ox), at(ctx, oq), q_dim, n_embd));
    SSD_TRY(dense_f32(ctx, at(ctx, owk), at(ctx, ox), at(ctx, ok), kv_dim, n_embd));
    SSD_TRY(dense_f32(ctx, at(ctx, owv), at(ctx, ox), at(ctx, ov), kv_dim, n_embd));
    if (rope) {  // fused_qkv_rope_f32_cpu: RoPE on Q and K only (compute.rs:509-533)
        SSD_TRY(ssd_rope(ctx, at(ctx, oq), q_dim, head_dim, q_dim / head_dim, position, theta,
                         ctx->stream));
        SSD_TRY(ssd_rope(ctx, at(ctx, ok), kv_dim, head_dim, kv_dim / head_dim, position, theta,
                         ctx->stream));
    }
    SSD_TRY(d2h(ctx, q, at(ctx, oq), (size_t)q_dim * 4));
    SSD_TRY(d2h(ctx, k, at(ctx, ok), (size_t)kv_dim * 4));
    SSD_TRY(d2h(ctx, v, at(ctx, ov), (size_t)kv_dim * 4));
    return finish(ctx, rope ? "fused_qkv_rope_f32" : "fused_qkv_f32");
}

extern "C" int ssd_fused_qkv_f32_host(ssd_ctx* ctx, const float* wq, const float* wk,
                                      const float* wv, const float* x, int q_dim, int kv_dim,
                                      int n_embd, float* q, float* k, float* v) {
    return qkv_host(ctx, wq, wk, wv, x, q_dim, kv_dim, n_embd, 0, 0, 0.0f, false, q, k, v);
}

extern "C" int ssd_fused_qkv_rope_f32_host(ssd_ctx* ctx, const float* wq, const float* wk,
                                           const float* wv, const float* x, int q_dim,
                                           int kv_dim, int n_embd, int head_dim, int position,
                                           float theta, float* q, float* k, float* v) {
    return qkv_host(ctx, wq, wk, wv, x, q_dim, kv_dim, n_embd, head_dim, position, theta, true,
                    q, k, v);
}

extern "C" int ssd_fused_rmsnorm_linear_f32_host(ssd_ctx* ctx, const float* x,
                                                 const float* norm_w, const float* out_w,
                                                 int vocab, int n_embd, float* logits) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(x && norm_w && out_w && logits, SSD_ERR_ARG, "null pointer");
    SSD_REQ(vocab > 0 && n_embd > 0, SSD_ERR_SHAPE, "empty projection");
    const size_t wb = (size_t)vocab * n_embd * 4, eb = (size_t)n_embd * 4;
    Stage st;
    const size_t ow = st.take(wb), ox = st.take(eb), on = st.take(eb), oxn = st.take(eb),
                 oy = st.take((size_t)vocab * 4);
    SSD_TRY(ensure_scratch(ctx, st.off));
    SSD_TRY(h2d(ctx, at(ctx, ow), out_w, wb));
    SSD_TRY(h2d(ctx, at(ctx, ox), x, eb));
    SSD_TRY(h2d(ctx, at(ctx, on), norm_w, eb));
    k_norm_into<<<1, 1024, 0, ctx->stream>>>(at(ctx, ox), at(ctx, on), n_embd, 1e-5f,
                                             at(ctx, oxn));
    SSD_CK_LAUNCH();
    SSD_TRY(dense_f32(ctx, at(ctx, ow), at(ctx, oxn), at(ctx, oy), vocab, n_embd));
    SSD_TRY(d2h(ctx, logits, at(ctx, oy), (size_t)vocab * 4));
    return finish(ctx, "fused_rmsnorm_linear_f32");
}

extern "C" int ssd_feed_forward_f32_host(ssd_ctx* ctx, const float* x, const float* w_gate,
                                         const float* w_up, const float* w_down, int n_embd,
                                         int n_ff, float* out) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(x && out && (n_ff == 0 || (w_gate && w_up && w_down)), SSD_ERR_ARG, "null pointer");
    SSD_REQ(n_embd > 0 && n_ff >= 0, SSD_ERR_SHAPE, "bad sizes n_embd %d n_ff %d", n_embd, n_ff);
    if (n_ff == 0) {  // feed_forward returns zeros when the weights are empty (:25-28)
        for (int i = 0; i < n_embd; i++) out[i] = 0.0f;
        return SSD_OK;
    }
    const size_t wb = (size_t)n_ff * n_embd * 4;
    Stage st;
    const size_t og = st.take(wb), ou = st.take(wb), od = st.take(wb),
                 ox = st.take((size_t)n_embd * 4), oa = st.take((size_t)n_ff * 4),
                 oy = st.take((size_t)n_embd * 4);
    SSD_TRY(ensure_scratch(ctx, st.off));
    SSD_TRY(h2d(ctx, at(ctx, og), w_gate, wb));
    SSD_TRY(h2d(ctx, at(ctx, ou), w_up, wb));
    SSD_TRY(h2d(ctx, at(ctx, od), w_down, wb));
    SSD_TRY(h2d(ctx, at(ctx, ox), x, (size_t)n_embd * 4));
    // gate and up rows share each x load; act = silu(gate) * up
    MvArgs a = {};
    a.qs[0] = reinterpret_cast<const uint8_t*>(at(ctx, og));
    a.qs[1] = reinterpret_cast<const uint8_t*>(at(ctx, ou));
    a.seg_rows[0] = n_ff;
    a.seg_rows[1] = n_ff;
    a.map = MAP_SWIGLU;
    a.rows = 2 * n_ff;
    a.cols = n_embd;
    a.x = at(ctx, ox);
    a.y = at(ctx, oa);
    SSD_TRY(launch_matvec(ctx, SSD_TYPE_F32, EPI_SWIGLU, a, ctx->stream, false));
    SSD_TRY(dense_f32(ctx, at(ctx, od), at(ctx, oa), at(ctx, oy), n_embd, n_ff));
    SSD_TRY(d2h(ctx, out, at(ctx, oy), (size_t)n_embd * 4));
    return finish(ctx, "feed_forward_f32");
}

extern "C" int ssd_rmsnorm_f32_host(ssd_ctx* ctx, float* x, const float* weight, int n,
                                    float eps) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(x && weight && n > 0, SSD_ERR_ARG, "bad arguments");
    Stage st;
    const size_t ox = st.take((size_t)n * 4), ow = st.take((size_t)n * 4);
    SSD_TRY(ensure_scratch(ctx, st.off));
    SSD_TRY(h2d(ctx, at(ctx, ox), x, (size_t)n * 4));
    SSD_TRY(h2d(ctx, at(ctx, ow), weight, (size_t)n * 4));
    SSD_TRY(ssd_rmsnorm(ctx, at(ctx, ox), at(ctx, ow), n, eps, ctx->stream));
    SSD_TRY(d2h(ctx, x, at(ctx, ox), (size_t)n * 4));
    return finish(ctx, "rmsnorm_f32");
}

extern "C" int ssd_softmax_f32_host(ssd_ctx* ctx, float* x, int n) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(x != nullptr && n >= 0, SSD_ERR_ARG, "bad arguments");
    if (n == 0) return SSD_OK;
    SSD_TRY(ensure_scratch(ctx, (size_t)n * 4));
    SSD_TRY(h2d(ctx, at(ctx, 0), x, (size_t)n * 4));
    SSD_TRY(ssd_softmax(ctx, at(ctx, 0), n, ctx->stream));
    SSD_TRY(d2h(ctx, x, at(ctx, 0), (size_t)n * 4));
    return finish(ctx, "softmax_f32");
}

extern "C" int ssd_fused_post_attn_norm_f32_host(ssd_ctx* ctx, float* hidden, const float* attn,
                                                 const float* norm_w, int n, float eps,
                                                 float* out) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(hidden && attn && norm_w && out && n > 0, SSD_ERR_ARG, "bad arguments");
    const size_t b = (size_t)n * 4;
    Stage st;
    const size_t oh = st.take(b), oa = st.take(b), ow = st.take(b), oo = st.take(b);
    SSD_TRY(ensure_scratch(ctx, st.off));
    SSD_TRY(h2d(ctx, at(ctx, oh), hidden, b));
    SSD_TRY(h2d(ctx, at(ctx, oa), attn, b));
    SSD_TRY(h2d(ctx, at(ctx, ow), norm_w, b));
    SSD_TRY(ssd_fused_post_attn_norm(ctx, at(ctx, oh), at(ctx, oa), at(ctx, ow), n, eps,
                                     at(ctx, oo), ctx->stream));
    SSD_TRY(d2h(ctx, hidden, at(ctx, oh), b));
    SSD_TRY(d2h(ctx, out, at(ctx, oo), b));
    return finish(ctx, "fused_post_attn_norm_f32");
}
