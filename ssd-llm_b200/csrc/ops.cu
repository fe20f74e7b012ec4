// ops.cu — RMSNorm, softmax, RoPE, SiLU, argmax, INT8 KV cache and split-K decode
// attention for sm_100a.
//
// Reference: MetalCompute::{rmsnorm_f32, softmax_f32, fused_post_attn_norm_f32,
// flash_attention_f32} (src/metal/compute.rs:193-258, :328-346), their CPU forms
// (:536-555, :580-645), QuantizedLayerKvCache (src/inference/quantized_kv_cache.rs:23-130),
// flash_attention_cached (src/inference/flash_attention.rs:40-143) and the greedy
// argmax of src/inference/sampler.rs:572-578.
#include <math.h>

#include <mutex>

#include <cstring>

#include "ops.cuh"

namespace ssd {

constexpr float kQ80Magic = 8388736.0f;  // 2^23 + 128: (byte ^ 0x80) under 0x4B -> int8 exact

template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = -INFINITY;
#pragma unroll
    for (int w = 0; w < NT / 32; w++) t = fmaxf(t, red[w]);
    return t;
}

// ------------------------------------------------------------ norms
// rmsnorm_f32_fast_scalar (src/metal/compute.rs:580-588): x *= inv_rms * w.
__global__ void __launch_bounds__(1024) k_rmsnorm(float* x, const float* w, int n, float eps) {
    __shared__ float red[32];
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += 1024) ss = fmaf(x[i], x[i], ss);
    ss = block_sum<1024>(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += 1024) x[i] = __fmul_rn(x[i], __fmul_rn(inv, w[i]));
}

// fused_post_attn_norm_f32_cpu (src/metal/compute.rs:536-555): h += a; out = h*inv*w.
__global__ void __launch_bounds__(1024) k_post_attn_norm(float* h, const float* a, const float* w,
                                                         int n, float eps, float* out) {
    __shared__ float red[32];
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += 1024) {
        const float v = __fadd_rn(h[i], a[i]);
        h[i] = v;
        ss = fmaf(v, v, ss);
    }
    ss = block_sum<1024>(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += 1024) out[i] = __fmul_rn(__fmul_rn(h[i], inv), w[i]);
}

// softmax_f32_fast_scalar (src/metal/compute.rs:604-620).
__global__ void __launch_bounds__(1024) k_softmax(float* x, int n) {
    __shared__ float red[32];
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += 1024) m = fmaxf(m, x[i]);
    m = block_max<1024>(m, red);
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += 1024) {
        const float e = expf(__fsub_rn(x[i], m));
        x[i] = e;
        s += e;
    }
    s = block_sum<1024>(s, red);
    if (s > 0.0f) {
        const float inv = __fdiv_rn(1.0f, s);
        for (int i = threadIdx.x; i < n; i += 1024) x[i] = __fmul_rn(x[i], inv);
    }
}

// rope_f32_multi_head (src/metal/compute.rs:482-506): one thread per adjacent pair.
__global__ void k_rope(float* x, int len, int head_dim, int n_heads, int pos, float theta) {
    const int half = head_dim / 2;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n_heads * half) return;
    const int h = t / half, i = t % half;
    const int i0 = h * head_dim + 2 * i, i1 = i0 + 1;
    if (i1 >= len) return;
    const float e = __fdiv_rn(__fmul_rn(2.0f, (float)i), (float)head_dim);
    const float freq = __fdiv_rn(1.0f, (float)pow((double)theta, (double)e));
    const float ang = __fmul_rn((float)pos, freq);
    double sd, cd;
    sincos((double)ang, &sd, &cd);
    const float sn = (float)sd, cs = (float)cd;
    const float x0 = x[i0], x1 = x[i1];
    x[i0] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
    x[i1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
}

// silu_f32 (src/metal/compute.rs:641-645): v / (1 + exp(-v)).
__global__ void k_silu(float* x, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fdiv_rn(x[i], __fadd_rn(1.0f, expf(-x[i])));
}

__device__ __forceinline__ unsigned long long amax_key(float v, uint32_t idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | idx;
}

// argmax with the LAST index on ties (Iterator::max_by, src/inference/sampler.rs:572-578).
__global__ void __launch_bounds__(1024) k_argmax(const float* v, int n, int32_t* idx) {
    __shared__ unsigned long long red[32];
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < n; i += 1024) {
        const unsigned long long k = amax_key(v[i], (uint32_t)i);
        best = k > best ? k : best;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
        best = t > best ? t : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < 32; w++) b = red[w] > b ? red[w] : b;
        *idx = (int32_t)(uint32_t)(b & 0xFFFFFFFFull);
    }
}

// ------------------------------------------------------------- INT8 KV
// QuantizedVec::quantize (src/inference/quantized_kv_cache.rs:23-41), bit-exact:
// absmax = max |v|; zero row -> scale 0; scale = absmax/127; q = clamp(round(v*127/absmax)).
// Rows of src_dim floats; the scale spans the whole row, columns [col0, col0 + kv_dim) are
// stored (the whole row when col0 == 0 and src_dim == kv_dim).
__global__ void __launch_bounds__(256) k_kv_append(const float* __restrict__ k,
                                                   const float* __restrict__ v, int8_t* kc,
                                                   int8_t* vc, float* ksc, float* vsc, int kv_dim,
                                                   int pos, const int* pos_dev, int capacity,
                                                   int src_dim, int col0) {
    __shared__ float red[8];
    pdl_wait();
    const int base_pos = pos_dev ? *pos_dev : pos;
    const int r = blockIdx.x, which = blockIdx.y;
    const int p = base_pos + r;
    if (p < 0 || p >= capacity) return;  // host checks bounds for the direct API
    const float* src = (which == 0 ? k : v) + (size_t)r * src_dim;
    int8_t* dst = (which == 0 ? kc : vc) + (size_t)p * kv_dim;
    float am = 0.0f;
    for (int i = threadIdx.x; i < src_dim; i += 256) am = fmaxf(am, fabsf(src[i]));
    am = block_max<256>(am, red);
    if (am == 0.0f) {
        for (int i = threadIdx.x; i < kv_dim; i += 256) dst[i] = 0;
        if (threadIdx.x == 0) (which == 0 ? ksc : vsc)[p] = 0.0f;
        return;
    }
    const float scale = __fdiv_rn(am, 127.0f);
    const float inv = __fdiv_rn(127.0f, am);
    for (int i = threadIdx.x; i < kv_dim; i += 256) {
        float q = roundf(__fmul_rn(src[col0 + i], inv));
        q = fminf(127.0f, fmaxf(-127.0f, q));
        dst[i] = (int8_t)(int)q;
    }
    if (threadIdx.x == 0) (which == 0 ? ksc : vsc)[p] = scale;
}

__global__ void __launch_bounds__(256) k_kv_absmax(const float* __restrict__ k,
                                                   const float* __restrict__ v, int n,
                                                   float* out) {
    __shared__ float red[8];
    pdl_wait();
    float ak = 0.0f, av = 0.0f;
    for (int i = threadIdx.x; i < n; i += 256) {
        ak = fmaxf(ak, fabsf(k[i]));
        av = fmaxf(av, fabsf(v[i]));
    }
    ak = block_max<256>(ak, red);
    __syncthreads();
    av = block_max<256>(av, red);
    if (threadIdx.x == 0) {
        out[0] = ak;
        out[1] = av;
    }
}

// ------------------------------------------------ split-K decode attention
// CTA (local kv head, chunk of ATT_P = 128 positions), 4 warps of 32 positions. The
// GROUP query heads that share the kv head (GQA kv_h = h / group,
// flash_attention.rs:79-80) are processed together:
//  * scores: lane = position. Each lane streams its own int8 K row (16-byte loads) and
//    dots it with the group's q, broadcast from shared memory. The int8 values are
//    decoded exactly with the denormal trick of the matvec (byte b of a word read as
//    the fp32 (k+128) * 2^(s-149), q pre-scaled by 2^(85-s), the +128 removed by a
//    per-head bias), two FMAs per instruction (fma.rn.f32x2);
//    score = (q . k) * k_scale * 1/sqrt(d) (flash_attention.rs:87-95 over the
//    INT8 rows of quantized_kv_cache.rs:118-130);
//  * warp softmax statistics per head: max, sum of exp (flash_attention.rs:96-118);
//  * P V: lane = head dimensions; weights exp(s - m) * v_scale broadcast from shared
//    memory, V decoded exactly as signed integers;
//  * the 4 warps' (m, l, acc) are merged with the online-softmax rescaling into one
//    partial per (head, chunk); k_attn_combine merges the chunks (:106-134).
// With few KV heads per GPU (tensor parallelism) a KV head's query group is split over
// a.hsplit CTAs (template G = group / hsplit query heads each), which read the same K/V
// chunk (the second and later reads hit L2), so the grid fills the SMs at any head count.
constexpr int ATT_P = 128;
constexpr int ATT_NW = ATT_P / 32;
constexpr float kAttUnscale = 18446744073709551616.0f;  // 2^64
constexpr float kAttS0 = 38685626227668133590597632.0f;  // 2^85: byte at bit 0
constexpr float kAttS8 = 151115727451828646838272.0f;    // 2^77: byte at bit 8

__device__ __forceinline__ float att_den(uint32_t bits) { return __uint_as_float(bits); }
__device__ __forceinline__ void att_ffma2(float& d0, float& d1, float a0, float a1, float b0,
                                          float b1) {
    uint64_t d, a, b;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(d0), "f"(d1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(b0), "f"(b1));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}
__device__ __forceinline__ uint32_t att_word(const uint4& q, int m) {
    return m == 0 ? q.x : (m == 1 ? q.y : (m == 2 ? q.z : q.w));
}

template <int HD, int G>
__global__ void __launch_bounds__(128) k_attn_partial(const AttnArgs a0) {
    AttnArgs a = a0;
    if (a0.n_slots > 0) {  // this query's slot: its own cache, position and new rows
        const int sl = blockIdx.z;
        a.k += (size_t)sl * a0.slot_kv;
        a.v += (size_t)sl * a0.slot_kv;
        a.ks += (size_t)sl * a0.slot_sc;
        a.vs += (size_t)sl * a0.slot_sc;
        a.pos_dev += sl;
        a.k_new += (size_t)sl * a0.slot_new;
        a.v_new += (size_t)sl * a0.slot_new;
    }
    constexpr int DPL = HD / 32;  // dims per lane in the P V phase
    __shared__ __align__(16) float qs[G][HD];         // q * 2^85 / 2^77 by byte position
    __shared__ __align__(16) float2 pw[ATT_NW][G][32];  // (weight, weight)
    __shared__ __align__(16) float red[ATT_NW][G][HD];
    __shared__ float mlw[ATT_NW][G][2];  // warp max, sum exp
    __shared__ float fac[ATT_NW][G];
    __shared__ float qbias[G];
    __shared__ float amred[2][ATT_NW > 8 ? ATT_NW : 8];
    __shared__ __align__(16) int8_t nkv[2][HD];  // the new position's K / V bytes (this head)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = a.hsplit > 0 ? a.hsplit : 1;
    // hg: this CTA's query-head group (local heads hg*G ..); gl: its KV head; hs: its part
    const int hg = blockIdx.x, gl = hg / S, hs = hg % S;
    const int chunk = blockIdx.y, nchunks = gridDim.y, qi = blockIdx.z;
    const int g_kv = a.kv_head0 + gl;
    // Decode with the append fused (k_new set): the new K/V row is quantized and written
    // by the CTAs of its chunk. No kernel before this one writes the cache then, so the
    // old rows are loaded before griddepcontrol.wait, overlapping the previous kernel; the
    // position itself was written by the previous step's last kernel, long complete.
    const bool fused = a.k_new != nullptr;
    int pnew = -1;
    if (!fused) pdl_wait();
    // positions [0, seq); never beyond the cache (max_seq is its capacity on the
    // graph path), so a position past the end reads nothing out of bounds. A batch of
    // causal queries (prefill): query qi sees positions [0, seq0 + qi].
    int seq;
    if (fused) {
        pnew = *a.pos_dev;
        seq = min(pnew + 1, a.max_seq);
    } else {
        seq = min(a.n_q > 1 ? a.seq0 + qi + 1 : (a.pos_dev ? (*a.pos_dev + 1) : a.seq_len),
                  a.max_seq);
    }
    const int p0 = chunk * ATT_P;
    const size_t qpart = (size_t)a.n_kv_local * S * G * nchunks * (HD + 2);
    float* part = a.partial + qpart * qi + ((size_t)(hg * G) * nchunks + chunk) * (HD + 2);
    const size_t head_stride = (size_t)nchunks * (HD + 2);
    const int p = p0 + 32 * warp + lane;
    // this lane's K row and position scales, and its bytes of the warp's 32 V rows: all in
    // flight at once (the new row, if in this chunk, is loaded once written below)
    const int pw0 = p0 + 32 * warp;
    const int npos = max(0, min(32, seq - pw0));
    uint4 krow[HD / 16];
    uint32_t vw[32];
    float ksc = 0.0f, vsc = 0.0f;
    const int8_t* vbase = a.v + (size_t)g_kv * HD + DPL * lane + (size_t)pw0 * a.kv_dim;
    if (p0 < seq) {
        if (p < seq && p != pnew) {
            const uint4* kr =
                reinterpret_cast<const uint4*>(a.k + (size_t)p * a.kv_dim + (size_t)g_kv * HD);
#pragma unroll
            for (int j = 0; j < HD / 16; j++) krow[j] = __ldg(kr + j);
            ksc = __ldg(a.ks + p);
            vsc = __ldg(a.vs + p);
        }
#pragma unroll
        for (int t = 0; t < 32; t++) {
            vw[t] = 0x80808080u;
            if (t < npos && pw0 + t != pnew) {
                const int8_t* vr = vbase + (size_t)t * a.kv_dim;
                if constexpr (DPL == 4)
                    vw[t] = __ldg(reinterpret_cast<const uint32_t*>(vr));
                else
                    vw[t] = (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(vr));
            }
        }
    }
    if (fused) pdl_wait();
    if (p0 >= seq) {
        if (tid < G) {
            part[tid * head_stride + 0] = -INFINITY;
            part[tid * head_stride + 1] = 0.0f;
        }
        return;
    }
    // q of the group: all float4 loads issued at once; each HD/4 consecutive float4 are
    // one head, so sub-groups of HD/4 lanes reduce that head's sum for the decode bias
    const float4* qg4 =
        reinterpret_cast<const float4*>(a.q + (size_t)qi * a.q_stride + (size_t)hg * G * HD);
    constexpr int QV = G * HD / 4 / 128 > 0 ? G * HD / 4 / 128 : 1;  // float4 per thread
    float4 qv[QV];
#pragma unroll
    for (int j = 0; j < QV; j++)
        if (tid + 128 * j < G * HD / 4) qv[j] = __ldg(qg4 + tid + 128 * j);
#pragma unroll
    for (int j = 0; j < QV; j++) {
        const int u = tid + 128 * j;  // float4 index
        const bool in = u < G * HD / 4;
        float t = 0.0f;
        if (in) {
            const float4 v = qv[j];
            reinterpret_cast<float4*>(&qs[0][0])[u] =
                make_float4(__fmul_rn(v.x, kAttS0), __fmul_rn(v.y, kAttS8),
                            __fmul_rn(v.z, kAttS0), __fmul_rn(v.w, kAttS8));
            t = (v.x + v.y) + (v.z + v.w);
        }
        // every lane shuffles (uniform control flow); groups of HD/4 lanes = one head
#pragma unroll
        for (int o = 1; o < HD / 4 && o < 32; o <<= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (in && (u % (HD / 4)) == 0)  // -128 * sum_d q[d], scaled by 2^-64
            qbias[u / (HD / 4)] = __fmul_rn(-128.0f, __fmul_rn(t, 1.0f / kAttUnscale));
    }
    if (fused && pnew >= p0 && pnew < p0 + ATT_P && pnew < a.max_seq) {
        // ---- the new position is in this chunk: quantize its K and V rows exactly as
        // k_kv_append (QuantizedVec::quantize, quantized_kv_cache.rs:23-41; the scale spans
        // every KV head), write this head's bytes (the CTA of local head 0 the scales), and
        // load them back
        float amk = 0.0f, amv = 0.0f;
        for (int i = tid; i < a.kv_dim; i += 128) {
            amk = fmaxf(amk, fabsf(a.k_new[i]));
            amv = fmaxf(amv, fabsf(a.v_new[i]));
        }
        amk = warp_max(amk);
        amv = warp_max(amv);
        if (lane == 0) {
            amred[0][warp] = amk;
            amred[1][warp] = amv;
        }
        __syncthreads();
        amk = 0.0f;
        amv = 0.0f;
#pragma unroll
        for (int w = 0; w < ATT_NW; w++) {
            amk = fmaxf(amk, amred[0][w]);
            amv = fmaxf(amv, amred[1][w]);
        }
        if (a.amax_in) {  // the global pair, max-reduced by the caller
            amk = a.amax_in[0];
            amv = a.amax_in[1];
        } else if (a.xch_n > 1) {
            // publish this rank's pair to every rank (local head 0's CTA), then take the max
            // of all ranks' pairs once every word carries this call's tag (bounded wait)
            const uint32_t tag = (uint32_t)(*a.xch_epoch + (unsigned long long)a.xch_call) + 1u;
            if (gl == 0 && hs == 0 && tid < 2 * a.xch_n) {
                const float val = (tid & 1) ? amv : amk;
                const unsigned long long w =
                    ((unsigned long long)__float_as_uint(val) << 32) | (unsigned long long)tag;
                asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a.xch_out[tid >> 1] +
                                                                        (tid & 1)),
                             "l"(w)
                             : "memory");
            }
            __syncthreads();  // amred is reused below
            if (tid < 2 * a.xch_n) {
                float val = 0.0f;
                if (*(volatile int*)a.status == SSD_OK) {  // fail fast after a timeout
                    bool done = false;
                    for (uint32_t it = 0; it < (1u << 21) && !done; it++) {
                        unsigned long long w;
                        asm volatile("ld.acquire.sys.global.u64 %0, [%1];"
                                     : "=l"(w)
                                     : "l"(a.xch_in + tid)
                                     : "memory");
                        done = (uint32_t)w == tag;
                        if (done)
                            val = __uint_as_float((uint32_t)(w >> 32));
                        else
                            __nanosleep(100);
                    }
                    if (!done) atomicExch(a.status, SSD_ERR_TIMEOUT);  // bytes below are then stale
                }
                amred[tid & 1][tid >> 1] = val;
            }
            __syncthreads();
            amk = 0.0f;
            amv = 0.0f;
            for (int r = 0; r < a.xch_n; r++) {
                amk = fmaxf(amk, amred[0][r]);
                amv = fmaxf(amv, amred[1][r]);
            }
        }
        const float sk = amk == 0.0f ? 0.0f : __fdiv_rn(amk, 127.0f);
        const float sv = amv == 0.0f ? 0.0f : __fdiv_rn(amv, 127.0f);
        const float ik = amk == 0.0f ? 0.0f : __fdiv_rn(127.0f, amk);
        const float iv = amv == 0.0f ? 0.0f : __fdiv_rn(127.0f, amv);
        // every CTA of the head quantizes the row into shared memory; the first (hs 0)
        // stores it in the cache
        int8_t* kc = const_cast<int8_t*>(a.k) + (size_t)pnew * a.kv_dim + (size_t)g_kv * HD;
        int8_t* vc = const_cast<int8_t*>(a.v) + (size_t)pnew * a.kv_dim + (size_t)g_kv * HD;
        for (int d = tid; d < HD; d += 128) {
            const float fk = fminf(127.0f, fmaxf(-127.0f, roundf(__fmul_rn(a.k_new[g_kv * HD + d], ik))));
            const float fv = fminf(127.0f, fmaxf(-127.0f, roundf(__fmul_rn(a.v_new[g_kv * HD + d], iv))));
            nkv[0][d] = (int8_t)(int)fk;
            nkv[1][d] = (int8_t)(int)fv;
            if (hs == 0) {
                kc[d] = (int8_t)(int)fk;
                vc[d] = (int8_t)(int)fv;
            }
        }
        if (gl == 0 && hs == 0 && tid == 0) {
            const_cast<float*>(a.ks)[pnew] = sk;
            const_cast<float*>(a.vs)[pnew] = sv;
        }
        __syncthreads();  // the row's bytes are visible to the whole CTA
        if (p == pnew) {
            const uint4* kr = reinterpret_cast<const uint4*>(&nkv[0][0]);
#pragma unroll
            for (int j = 0; j < HD / 16; j++) krow[j] = kr[j];
            ksc = sk;
            vsc = sv;
        }
#pragma unroll
        for (int t = 0; t < 32; t++) {
            if (pw0 + t == pnew) {
                const int8_t* vr = &nkv[1][0] + DPL * lane;
                if constexpr (DPL == 4)
                    vw[t] = *reinterpret_cast<const uint32_t*>(vr);
                else
                    vw[t] = (uint32_t)*reinterpret_cast<const uint16_t*>(vr);
            }
        }
    }
    __syncthreads();

    // ---- scores: lane = position
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
    float sc[G];
    {
        float e[G], o[G];
#pragma unroll
        for (int i = 0; i < G; i++) {
            e[i] = qbias[i];
            o[i] = 0.0f;
        }
        if (p < seq) {
#pragma unroll
            for (int j = 0; j < HD / 16; j++) {
                const uint4 kk = krow[j];  // dims 16j .. 16j+15
#pragma unroll
                for (int m = 0; m < 4; m++) {
                    const uint32_t w = att_word(kk, m) ^ 0x80808080u, w2 = w >> 16;
                    const float f0 = att_den(w & 0xFFu), f1 = att_den(w & 0xFF00u);
                    const float f2 = att_den(w2 & 0xFFu), f3 = att_den(w2 & 0xFF00u);
#pragma unroll
                    for (int i = 0; i < G; i++) {
                        const float4 q4 = *reinterpret_cast<const float4*>(&qs[i][16 * j + 4 * m]);
                        att_ffma2(e[i], o[i], f0, f1, q4.x, q4.y);
                        att_ffma2(e[i], o[i], f2, f3, q4.z, q4.w);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < G; i++)
                sc[i] = __fmul_rn(__fmul_rn(__fmul_rn(e[i] + o[i], kAttUnscale), ksc), scale);
        } else {
#pragma unroll
            for (int i = 0; i < G; i++) sc[i] = -INFINITY;
        }
    }
    // ---- warp softmax statistics; weights exp(s - m) * v_scale for P V
#pragma unroll
    for (int i = 0; i < G; i++) {
        const float m = warp_max(sc[i]);
        const float ex = sc[i] == -INFINITY ? 0.0f : expf(__fsub_rn(sc[i], m));
        const float wgt = __fmul_rn(ex, vsc);
        const float l = warp_sum(ex);
        pw[warp][i][lane] = make_float2(wgt, wgt);
        if (lane == 0) {
            mlw[warp][i][0] = m;
            mlw[warp][i][1] = l;
        }
    }
    __syncwarp();

    // ---- P V over this warp's 32 positions: lane = dims DPL*lane ..; V values decoded
    // exactly as signed integers (byte ^ 0x80 under exponent 0x4B, minus 2^23 + 128):
    // the weights are all positive, so an offset decode would not cancel.
    float acc[G][DPL];
#pragma unroll
    for (int i = 0; i < G; i++)
#pragma unroll
        for (int j = 0; j < DPL; j++) acc[i][j] = 0.0f;
#pragma unroll
    for (int t = 0; t < 32; t++) {
        if (t >= npos) break;
        float f[DPL];
        const uint32_t w = vw[t] ^ 0x80808080u;
#pragma unroll
        for (int j = 0; j < DPL; j++) f[j] = magic_byte(w, j) - kQ80Magic;
#pragma unroll
        for (int i = 0; i < G; i++) {
            const float2 wp = pw[warp][i][t];
#pragma unroll
            for (int j = 0; j < DPL; j += 2) att_ffma2(acc[i][j], acc[i][j + 1], f[j], f[j + 1], wp.x, wp.y);
        }
    }
#pragma unroll
    for (int i = 0; i < G; i++)
#pragma unroll
        for (int j = 0; j < DPL; j++) red[warp][i][DPL * lane + j] = acc[i][j];
    __syncthreads();
    // ---- merge the 4 warps: M = max m_w, factor exp(m_w - M) (0 for empty warps)
    if (tid < ATT_NW * G) {
        const int w = tid / G, i = tid % G;
        float M = -INFINITY;
#pragma unroll
        for (int v = 0; v < ATT_NW; v++) M = fmaxf(M, mlw[v][i][0]);
        fac[w][i] = mlw[w][i][1] == 0.0f ? 0.0f : expf(__fsub_rn(mlw[w][i][0], M));
    }
    __syncthreads();
    for (int idx = tid; idx < G * HD; idx += 128) {
        const int i = idx / HD, d = idx % HD;
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < ATT_NW; w++) s = fmaf(red[w][i][d], fac[w][i], s);
        part[i * head_stride + 2 + d] = s;
    }
    if (tid < G) {
        float M = -INFINITY, L = 0.0f;
#pragma unroll
        for (int w = 0; w < ATT_NW; w++) M = fmaxf(M, mlw[w][tid][0]);
#pragma unroll
        for (int w = 0; w < ATT_NW; w++) L = fmaf(mlw[w][tid][1], fac[w][tid], L);
        part[tid * head_stride + 0] = M;
        part[tid * head_stride + 1] = L;
    }
}

// Merges the chunk partials of one query head (flash_attention.rs:106-134): the chunk
// statistics are loaded in parallel, the rescale factors exp(m_c - M) shared through
// shared memory, then thread d sums its dimension over the chunks. (Issuing every load of
// the head at once, with one barrier, measured no faster inside the PDL chain: the partial
// kernel's tail already hides these round trips.)
template <int HD>
__global__ void __launch_bounds__(HD) k_attn_combine(const AttnArgs a, int nchunks) {
    __shared__ float fac[1024];
    __shared__ float red[HD / 32];
    __shared__ float lsum[HD / 32];
    const int h = blockIdx.x, d = threadIdx.x, lane = d & 31, warp = d >> 5, qi = blockIdx.y;
    pdl_wait();
    const float* part = a.partial + (size_t)qi * gridDim.x * nchunks * (HD + 2) +
                        (size_t)h * nchunks * (HD + 2);
    float m = -INFINITY;
    for (int c = d; c < nchunks; c += HD) m = fmaxf(m, part[(size_t)c * (HD + 2)]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < HD / 32; w++) M = fmaxf(M, red[w]);
    float L = 0.0f;
    for (int c = d; c < nchunks; c += HD) {
        const float* pc = part + (size_t)c * (HD + 2);
        const float l = pc[1];
        const float f = l == 0.0f ? 0.0f : expf(__fsub_rn(pc[0], M));
        fac[c] = f;
        L = fmaf(l, f, L);
    }
    L = warp_sum(L);
    if (lane == 0) lsum[warp] = L;
    __syncthreads();
    L = 0.0f;
#pragma unroll
    for (int w = 0; w < HD / 32; w++) L += lsum[w];
    // chunks past the sequence (factor 0) hold stale data: their values are loaded (the
    // buffer holds all nchunks records) but not used
    float acc = 0.0f;
    const float* pd = part + 2 + d;
    int c = 0;
    for (; c + 8 <= nchunks; c += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = pd[(size_t)(c + j) * (HD + 2)];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float f = fac[c + j];
            acc = f != 0.0f ? fmaf(v[j], f, acc) : acc;
        }
    }
    for (; c < nchunks; c++) {
        const float v = pd[(size_t)c * (HD + 2)], f = fac[c];
        acc = f != 0.0f ? fmaf(v, f, acc) : acc;
    }
    // output_acc[d] * (1 / running_sum)  (flash_attention.rs:126-133)
    a.out[(size_t)qi * a.out_stride + (size_t)h * HD + d] =
        L > 0.0f ? __fmul_rn(acc, __fdiv_rn(1.0f, L)) : 0.0f;
}

size_t attn_partial_floats(int n_heads, int max_seq, int head_dim) {
    const int nchunks = (max_seq + ATT_P - 1) / ATT_P;
    return (size_t)n_heads * nchunks * (head_dim + 2);
}

// G = query heads per CTA (a.group / a.hsplit).
template <int HD, int G>
static int launch_attn_t(const AttnArgs& a, cudaStream_t s, bool pdl) {
    const int nchunks = (a.max_seq + ATT_P - 1) / ATT_P;
    const int nq = a.n_q > 1 ? a.n_q : 1;
    SSD_CK(launch_pdl(k_attn_partial<HD, G>, dim3(a.n_kv_local * a.hsplit, nchunks, nq), dim3(128),
                      0, s, pdl, a));
    SSD_CK(launch_pdl(k_attn_combine<HD>, dim3(a.n_kv_local * a.group, nq), dim3(HD), 0, s, pdl,
                      a, nchunks));
    return SSD_OK;
}

static int sm_count() {
    static int n = [] {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    return n;
}

template <int HD>
static int launch_attn_hd(const AttnArgs& a0, cudaStream_t s, bool pdl) {
    SSD_REQ(a0.group == 1 || a0.group == 2 || a0.group == 4 || a0.group == 8, SSD_ERR_SHAPE,
            "GQA group %d not supported (1, 2, 4, 8)", a0.group);
    AttnArgs a = a0;
    // decode: split the query group while the grid would still hold under ~one CTA per SM
    // (measured, 70B heads at 4096 positions: 8 KV heads best unsplit, 14.6 us against 17.7
    // split in two; 1 KV head best split in four, 7.9 us against 10.4 unsplit and 8.9 split in
    // eight: each split repeats the K decode, so it pays only while SMs would sit idle)
    const int nchunks = (a.max_seq + ATT_P - 1) / ATT_P;
    a.hsplit = 1;
    static const int forced = [] {  // SSD_ATTN_HSPLIT=n: a fixed split (tuning sweeps)
        const char* e = getenv("SSD_ATTN_HSPLIT");
        return e ? atoi(e) : 0;
    }();
    if (a.n_q <= 1) {
        if (forced > 0)
            while (a.hsplit < forced && a.hsplit < a.group) a.hsplit *= 2;
        else
            while (a.hsplit < a.group && 2 * a.n_kv_local * a.hsplit * nchunks <= sm_count())
                a.hsplit *= 2;
    }
    switch (a.group / a.hsplit) {
        case 1: return launch_attn_t<HD, 1>(a, s, pdl);
        case 2: return launch_attn_t<HD, 2>(a, s, pdl);
        case 4: return launch_attn_t<HD, 4>(a, s, pdl);
        default: return launch_attn_t<HD, 8>(a, s, pdl);
    }
}

int launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
    SSD_REQ(a.max_seq > 0, SSD_ERR_SHAPE, "empty attention");
    SSD_REQ(!a.k_new || (a.v_new && a.pos_dev && (a.n_q <= 1 || a.n_slots == a.n_q)), SSD_ERR_ARG,
            "fused KV append needs v_new, pos_dev and one query per cache");
    SSD_REQ(a.n_slots == 0 || (a.k_new && a.n_q == a.n_slots), SSD_ERR_ARG,
            "batch attention: one query per slot, with the fused append");
    SSD_REQ((a.max_seq + ATT_P - 1) / ATT_P <= 1024, SSD_ERR_SHAPE,
            "attention over %d positions exceeds %d", a.max_seq, 1024 * ATT_P);
    SSD_REQ(a.xch_n <= 1 || (a.k_new && a.status && a.xch_in && a.xch_epoch && a.xch_n <= 8),
            SSD_ERR_ARG, "absmax exchange needs the fused append, a status word and its slots");
    for (int r = 0; r < (a.xch_n > 1 ? a.xch_n : 0); r++)
        SSD_REQ(a.xch_out[r] != nullptr, SSD_ERR_ARG, "null exchange slot of rank %d", r);
    if (a.head_dim == 128) return launch_attn_hd<128>(a, s, pdl);
    if (a.head_dim == 64) return launch_attn_hd<64>(a, s, pdl);
    set_error("head_dim %d not supported (64, 128)", a.head_dim);
    return SSD_ERR_SHAPE;
}

int launch_kv_append(const ssd_kv_cache* kv, const float* k, const float* v, int pos,
                     const int* pos_dev, int rows, cudaStream_t s, bool pdl) {
    SSD_CK(launch_pdl(k_kv_append, dim3(rows, 2), dim3(256), 0, s, pdl, k, v, kv->k, kv->v,
                      kv->k_scale, kv->v_scale, kv->kv_dim, pos, pos_dev, kv->capacity,
                      kv->kv_dim, 0));
    return SSD_OK;
}

int launch_kv_append_slice(const ssd_kv_cache* kv, const float* k, const float* v, int src_dim,
                           int col0, int pos, int rows, cudaStream_t s) {
    SSD_REQ(col0 >= 0 && col0 + kv->kv_dim <= src_dim, SSD_ERR_SHAPE,
            "slice [%d, %d) outside rows of %d", col0, col0 + kv->kv_dim, src_dim);
    SSD_CK(launch_pdl(k_kv_append, dim3(rows, 2), dim3(256), 0, s, false, k, v, kv->k, kv->v,
                      kv->k_scale, kv->v_scale, kv->kv_dim, pos, (const int*)nullptr,
                      kv->capacity, src_dim, col0));
    return SSD_OK;
}

int launch_kv_absmax(const float* k, const float* v, int n, float* out, cudaStream_t s,
                     bool pdl) {
    SSD_CK(launch_pdl(k_kv_absmax, dim3(1), dim3(256), 0, s, pdl, k, v, n, out));
    return SSD_OK;
}

// ---------------------------------------------------------- embed / finalize
__global__ void __launch_bounds__(256) k_embed(const ssd_weight e, const int32_t* token,
                                               float* hidden) {
    pdl_wait();
    int t = token[blockIdx.x];  // one row per block (one block on the decode path)
    hidden += (size_t)blockIdx.x * e.cols;
    t = t < 0 ? 0 : (t >= e.rows ? e.rows - 1 : t);  // out-of-range ids clamp (no OOB read)
    const int n = e.cols;
    // dequant8: the element values of the matvec decoders (bit-exact dequantization)
    for (int i = 8 * threadIdx.x; i < n; i += 8 * 256) {
        float v[8];
        dequant8(e, (int64_t)t * n + i, v);
#pragma unroll
        for (int j = 0; j < 8; j++) hidden[i + j] = v[j];
    }
}

__global__ void k_finalize(unsigned long long* key, int32_t* token, int* pos,
                           unsigned long long* epoch, int epoch_inc) {
    pdl_wait();
    const unsigned long long k = *key;
    *token = (int32_t)(uint32_t)(k & 0xFFFFFFFFull);
    *key = 0ull;
    *pos += 1;
    if (epoch) *epoch += (unsigned long long)epoch_inc;
}

int launch_embed(const ssd_weight* emb, const int32_t* token_dev, float* hidden, cudaStream_t s,
                 bool pdl) {
    SSD_REQ(type_block(emb->type) != 0 && !is_lowbit(emb->type) && emb->cols % 8 == 0, SSD_ERR_TYPE,
            "token_embd type %d not supported (F32, F16, BF16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K)",
            emb->type);
    SSD_CK(launch_pdl(k_embed, dim3(1), dim3(256), 0, s, pdl, *emb, token_dev, hidden));
    return SSD_OK;
}

int launch_embed_rows(const ssd_weight* emb, const int32_t* tokens_dev, int n, float* hidden,
                      cudaStream_t s) {
    SSD_REQ(type_block(emb->type) != 0 && !is_lowbit(emb->type) && emb->cols % 8 == 0, SSD_ERR_TYPE,
            "token_embd type %d not supported (F32, F16, BF16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K)",
            emb->type);
    SSD_CK(launch_pdl(k_embed, dim3(n), dim3(256), 0, s, false, *emb, tokens_dev, hidden));
    return SSD_OK;
}

int launch_finalize(unsigned long long* key, int32_t* token, int* pos, unsigned long long* epoch,
                    int epoch_inc, cudaStream_t s, bool pdl) {
    SSD_CK(launch_pdl(k_finalize, dim3(1), dim3(1), 0, s, pdl, key, token, pos, epoch, epoch_inc));
    return SSD_OK;
}

}  // namespace ssd

using namespace ssd;

// =================================================================== C ABI

extern "C" int ssd_rmsnorm(ssd_ctx* ctx, float* x, const float* w, int n, float eps, void* s) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(x && w && n > 0, SSD_ERR_ARG, "bad arguments");
    k_rmsnorm<<<1, 1024, 0, pick_stream(ctx, s)>>>(x, w, n, eps);
    SSD_CK_LAUNCH();
    return SSD_OK;
}

extern "C" int ssd_fused_post_attn_norm(ssd_ctx* ctx, float* h, const float* a, const float* w,
                                        int n, float eps, float* out, void* s) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(h && a && w && out && n > 0, SSD_ERR_ARG, "bad arguments");
    k_post_attn_norm<<<1, 1024, 0, pick_stream(ctx, s)>>>(h, a, w, n, eps, out);
    SSD_CK_LAUNCH();
    return SSD_OK;
}

extern "C" int ssd_softmax(ssd_ctx* ctx, float* x, int n, void* s) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(x != nullptr && n >= 0, SSD_ERR_ARG, "bad arguments");
    if (n == 0) return SSD_OK;  // the reference returns early on empty input
    k_softmax<<<1, 1024, 0, pick_stream(ctx, s)>>>(x, n);
    SSD_CK_LAUNCH();
    return SSD_OK;
}

extern "C" int ssd_rope(ssd_ctx* ctx, float* x, int len, int head_dim, int n_heads, int position,
                        float theta, void* s) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(x && head_dim > 1 && n_heads > 0 && len > 0, SSD_ERR_ARG, "bad arguments");
    const int pairs = n_heads * (head_dim / 2);
    k_rope<<<(pairs + 255) / 256, 256, 0, pick_stream(ctx, s)>>>(x, len, head_dim, n_heads,
                                                                 position, theta);
    SSD_CK_LAUNCH();
    return SSD_OK;
}

extern "C" int ssd_silu(ssd_ctx* ctx, float* x, int n, void* s) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(x && n > 0, SSD_ERR_ARG, "bad arguments");
    k_silu<<<(n + 255) / 256, 256, 0, pick_stream(ctx, s)>>>(x, n);
    SSD_CK_LAUNCH();
    return SSD_OK;
}

extern "C" int ssd_argmax(ssd_ctx* ctx, const float* v, int n, int32_t* idx, void* s) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(v && idx && n > 0, SSD_ERR_ARG, "bad arguments");
    k_argmax<<<1, 1024, 0, pick_stream(ctx, s)>>>(v, n, idx);
    SSD_CK_LAUNCH();
    return SSD_OK;
}

extern "C" int ssd_kv_create(ssd_ctx* ctx, int capacity, int n_head_kv, int head_dim,
                             ssd_kv_cache** out) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(out && capacity > 0 && n_head_kv > 0 && head_dim > 0, SSD_ERR_ARG, "bad arguments");
    SSD_REQ(head_dim % 16 == 0, SSD_ERR_SHAPE, "head_dim %d must be a multiple of 16", head_dim);
    const int kv_dim = n_head_kv * head_dim;
    const size_t kb = (size_t)capacity * kv_dim;
    const size_t kb_pad = (kb + 255) & ~(size_t)255;
    const size_t sb_pad = ((size_t)capacity * 4 + 255) & ~(size_t)255;
    const size_t total = 2 * kb_pad + 2 * sb_pad;
    void* p = nullptr;
    if (cudaMalloc(&p, total) != cudaSuccess) {
        cudaGetLastError();
        set_error("KV cache allocation of %zu bytes failed", total);
        return SSD_ERR_NOMEM;
    }
    if (zero_device(ctx, p, total) != SSD_OK) {
        cudaFree(p);
        return SSD_ERR_CUDA;
    }
    ssd_kv_cache* kv = new ssd_kv_cache();
    kv->ctx = ctx;
    kv->capacity = capacity;
    kv->n_head_kv = n_head_kv;
    kv->head_dim = head_dim;
    kv->kv_dim = kv_dim;
    kv->base = p;
    kv->k = (int8_t*)p;
    kv->v = (int8_t*)p + kb_pad;
    kv->k_scale = (float*)((char*)p + 2 * kb_pad);
    kv->v_scale = (float*)((char*)p + 2 * kb_pad + sb_pad);
    *out = kv;
    return SSD_OK;
}

extern "C" int ssd_kv_free(ssd_kv_cache* kv) {
    if (!kv) return SSD_OK;
    cudaSetDevice(kv->ctx->device);
    cudaFree(kv->base);
    delete kv;
    return SSD_OK;
}

extern "C" int ssd_kv_pointers(ssd_kv_cache* kv, int8_t** k, int8_t** v, float** ks, float** vs) {
    SSD_REQ(kv != nullptr, SSD_ERR_ARG, "null cache");
    if (k) *k = kv->k;
    if (v) *v = kv->v;
    if (ks) *ks = kv->k_scale;
    if (vs) *vs = kv->v_scale;
    return SSD_OK;
}

extern "C" int ssd_kv_append_rows(ssd_ctx* ctx, ssd_kv_cache* kv, const float* k, const float* v,
                                  int position, int rows, void* s) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(kv && k && v && rows > 0, SSD_ERR_ARG, "bad arguments");
    SSD_REQ(position >= 0 && position + rows <= kv->capacity, SSD_ERR_SHAPE,
            "positions [%d, %d) exceed capacity %d", position, position + rows, kv->capacity);
    return launch_kv_append(kv, k, v, position, nullptr, rows, pick_stream(ctx, s), false);
}

extern "C" int ssd_kv_append(ssd_ctx* ctx, ssd_kv_cache* kv, const float* k, const float* v,
                             int position, void* s) {
    return ssd_kv_append_rows(ctx, kv, k, v, position, 1, s);
}

extern "C" int ssd_attention_int8(ssd_ctx* ctx, const ssd_kv_cache* kv, const float* q,
                                  int n_head, int seq_len, float* out, void* s) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(kv && q && out, SSD_ERR_ARG, "null pointer");
    SSD_REQ(seq_len > 0 && seq_len <= kv->capacity, SSD_ERR_SHAPE, "seq_len %d outside (0, %d]",
            seq_len, kv->capacity);
    SSD_REQ(n_head % kv->n_head_kv == 0, SSD_ERR_SHAPE, "n_head %d not a multiple of n_head_kv %d",
            n_head, kv->n_head_kv);
    const size_t pf = attn_partial_floats(n_head, seq_len, kv->head_dim);
    SSD_TRY(ensure_scratch(ctx, pf * 4));
    AttnArgs a = {};
    a.k = kv->k;
    a.v = kv->v;
    a.ks = kv->k_scale;
    a.vs = kv->v_scale;
    a.kv_dim = kv->kv_dim;
    a.head_dim = kv->head_dim;
    a.group = n_head / kv->n_head_kv;
    a.kv_head0 = 0;
    a.n_kv_local = kv->n_head_kv;
    a.q = q;
    a.out = out;
    a.partial = (float*)ctx->scratch;
    a.seq_len = seq_len;
    a.pos_dev = nullptr;
    a.max_seq = seq_len;
    return launch_attention(a, pick_stream(ctx, s), false);
}

// Causal attention of n_q consecutive queries (a prompt batch) at positions pos0 .. over
// the cache rows [0, pos0 + n_q): on the tcgen05 tensor cores when head_dim is 128 and n_q
// a multiple of 128 (SSD_PREFILL_ATTN=decode forces the per-query kernels), else the
// batched split-K decode kernels.
bool ssd::prefill_attention_uses_tc(const AttnArgs& a) {
    const char* e = getenv("SSD_PREFILL_ATTN");
    const bool per_query = e && strcmp(e, "decode") == 0;
    return !per_query && a.head_dim == 128 && a.n_q % 128 == 0 && a.q_stride % 4 == 0 &&
           a.out_stride % 4 == 0 && a.kv_dim % 16 == 0;
}

int ssd::launch_prefill_attention(ssd_ctx* ctx, const AttnArgs& a, cudaStream_t s, bool pdl) {
    if (prefill_attention_uses_tc(a)) return launch_attention_prefill_tc(ctx, a, s, pdl);
    SSD_REQ(!a.out_hi, SSD_ERR_ARG, "fp16 split output needs the tensor-core prefill attention");
    return launch_attention(a, s, pdl);
}

extern "C" int ssd_attention_prefill(ssd_ctx* ctx, const ssd_kv_cache* kv, const float* q,
                                     int n_q, int q_stride, int pos0, int n_head, float* out,
                                     int out_stride, void* s) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(kv && q && out, SSD_ERR_ARG, "null pointer");
    SSD_REQ(n_q > 0 && pos0 >= 0 && pos0 + n_q <= kv->capacity, SSD_ERR_SHAPE,
            "queries [%d, %d) outside the cache of %d", pos0, pos0 + n_q, kv->capacity);
    SSD_REQ(n_head % kv->n_head_kv == 0, SSD_ERR_SHAPE, "n_head %d not a multiple of n_head_kv %d",
            n_head, kv->n_head_kv);
    SSD_REQ(q_stride >= n_head * kv->head_dim && out_stride >= n_head * kv->head_dim, SSD_ERR_SHAPE,
            "row strides shorter than n_head * head_dim");
    AttnArgs a = {};
    a.k = kv->k;
    a.v = kv->v;
    a.ks = kv->k_scale;
    a.vs = kv->v_scale;
    a.kv_dim = kv->kv_dim;
    a.head_dim = kv->head_dim;
    a.group = n_head / kv->n_head_kv;
    a.kv_head0 = 0;
    a.n_kv_local = kv->n_head_kv;
    a.q = q;
    a.out = out;
    a.max_seq = pos0 + n_q;
    a.n_q = n_q;
    a.q_stride = q_stride;
    a.out_stride = out_stride;
    a.seq0 = pos0;
    const size_t pf = (size_t)n_q * attn_partial_floats(n_head, pos0 + n_q, kv->head_dim);
    const char* e = getenv("SSD_PREFILL_ATTN");
    if (kv->head_dim != 128 || n_q % 128 != 0 || (e && strcmp(e, "decode") == 0)) {
        SSD_TRY(ensure_scratch(ctx, pf * 4));  // partials of the per-query kernels
        a.partial = (float*)ctx->scratch;
    }
    return launch_prefill_attention(ctx, a, pick_stream(ctx, s), false);
}

// ============================================ allocation-free attention variant
// Some callers cannot allocate device memory: code that runs while a CUDA graph is
// being captured elsewhere in the process, hosts whose allocator is owned by a
// framework that forbids foreign cudaMalloc/cudaFree (a cudaFree synchronises the
// whole device), and real-time loops that must not block in the driver. For them,
// ssd_attention_int8_noalloc keeps the split-K partials in this fixed device array
// instead of the context's growable scratch buffer. The array is part of the
// library image: every GPU that loads the library holds its 4 MiB until the process
// exits. Nothing in it needs to start at zero: k_attn_partial writes every
// (head, chunk) record that k_attn_combine reads, on every call.
constexpr size_t kNoAllocPartialFloats = (size_t)1 << 20;  // 4 MiB
static __device__ __align__(256) float g_noalloc_partial[kNoAllocPartialFloats];

// Device address of g_noalloc_partial on each device, looked up once per device with
// that device current. In host code the array's name is only a host-side stand-in,
// never a device address.
static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64] = {nullptr};

// Loads every attention kernel the entry point may launch (each head_dim and GQA group)
// on the current device. With lazy module loading a kernel's code is otherwise loaded at
// its first launch, which would make the first call with a new (head_dim, group) do more
// than launch.
static int noalloc_preload_kernels() {
    cudaFuncAttributes fa;
    const void* fns[] = {
        (const void*)k_attn_partial<128, 1>, (const void*)k_attn_partial<128, 2>,
        (const void*)k_attn_partial<128, 4>, (const void*)k_attn_partial<128, 8>,
        (const void*)k_attn_partial<64, 1>,  (const void*)k_attn_partial<64, 2>,
        (const void*)k_attn_partial<64, 4>,  (const void*)k_attn_partial<64, 8>,
        (const void*)k_attn_combine<128>,    (const void*)k_attn_combine<64>};
    for (const void* f : fns) SSD_CK(cudaFuncGetAttributes(&fa, f));
    return SSD_OK;
}

static int noalloc_partial_ptr(int device, float** out) {
    SSD_REQ(device >= 0 && device < 64, SSD_ERR_ARG, "device %d out of range", device);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[device]) {
        void* p = nullptr;
        SSD_CK(cudaGetSymbolAddress(&p, g_noalloc_partial));  // check_ctx made `device` current
        SSD_TRY(noalloc_preload_kernels());
        g_noalloc_ptr[device] = (float*)p;
    }
    *out = g_noalloc_ptr[device];
    return SSD_OK;
}

extern "C" int ssd_attention_int8_noalloc(ssd_ctx* ctx, const ssd_kv_cache* kv, const float* q,
                                          int n_head, int seq_len, float* out, void* s) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(kv && q && out, SSD_ERR_ARG, "null pointer");
    SSD_REQ(seq_len > 0 && seq_len <= kv->capacity, SSD_ERR_SHAPE, "seq_len %d outside (0, %d]",
            seq_len, kv->capacity);
    SSD_REQ(n_head % kv->n_head_kv == 0, SSD_ERR_SHAPE, "n_head %d not a multiple of n_head_kv %d",
            n_head, kv->n_head_kv);
    const size_t pf = attn_partial_floats(n_head, seq_len, kv->head_dim);
    SSD_REQ(pf <= kNoAllocPartialFloats, SSD_ERR_SHAPE,
            "attention_int8_noalloc: %d heads x %d positions need %zu partial floats; the fixed "
            "buffer holds %zu (n_head * ceil(seq_len/128) * (head_dim+2) must not exceed it)",
            n_head, seq_len, pf, kNoAllocPartialFloats);
    float* partial = nullptr;
    SSD_TRY(noalloc_partial_ptr(ctx->device, &partial));
    AttnArgs a = {};
    a.k = kv->k;
    a.v = kv->v;
    a.ks = kv->k_scale;
    a.vs = kv->v_scale;
    a.kv_dim = kv->kv_dim;
    a.head_dim = kv->head_dim;
    a.group = n_head / kv->n_head_kv;
    a.kv_head0 = 0;
    a.n_kv_local = kv->n_head_kv;
    a.q = q;
    a.out = out;
    a.partial = partial;
    a.seq_len = seq_len;
    a.pos_dev = nullptr;
    a.max_seq = seq_len;
    return launch_attention(a, pick_stream(ctx, s), false);
}
