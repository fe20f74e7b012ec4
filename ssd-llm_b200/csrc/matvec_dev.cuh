// matvec_dev.cuh — device pieces shared by the two matvec kernels (matvec.cu: the
// FMA kernel for any shape; matvec_tc.cu: the integer tensor-core kernel for the
// common shapes): row mapping, cp.async staging, the x prologue, epilogue helpers.
#pragma once
#include <mutex>

#include "matvec.cuh"

namespace ssd {

constexpr int kMaxRopePairs = 256;  // head_dim <= 512

// The row map each epilogue is launched with: QKV + RoPE reads the three projections,
// SwiGLU interleaves gate and up rows, every other epilogue reads one matrix.
__host__ __device__ constexpr int epi_map(int epi) {
    return epi == EPI_QKV_ROPE ? MAP_QKV : (epi == EPI_SWIGLU ? MAP_SWIGLU : MAP_PLAIN);
}

// Virtual row v -> (segment, row within the segment). R is the number of rows a warp
// computes together; MAP_SWIGLU puts R/2 gate rows then the R/2 matching up rows in
// each group of R. MAP >= 0 fixes the map at compile time (it must equal a.map).
template <int MAP = -1>
__device__ __forceinline__ void map_row(const MvArgs& a, int R, int v, int& seg, int& lr) {
    const int map = MAP >= 0 ? MAP : a.map;
    if (map == MAP_PLAIN) {
        seg = 0;
        lr = v;
    } else if (map == MAP_QKV) {
        if (v < a.seg_rows[0]) {
            seg = 0;
            lr = v;
        } else if (v < a.seg_rows[0] + a.seg_rows[1]) {
            seg = 1;
            lr = v - a.seg_rows[0];
        } else {
            seg = 2;
            lr = v - a.seg_rows[0] - a.seg_rows[1];
        }
    } else {  // MAP_SWIGLU: rows R*g .. R*g+R/2-1 are gate rows (R/2)g.., the rest up rows
        const int h = R >> 1;
        const int g = v / R, j = v % R;
        seg = j >= h;
        lr = h * g + (j - (j >= h ? h : 0));
    }
}

// ---- cp.async (global -> shared, bypassing registers)
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void rope_apply(float& x0, float& x1, float2 cs) {
    const float a0 = x0, a1 = x1;
    x0 = __fsub_rn(__fmul_rn(a0, cs.x), __fmul_rn(a1, cs.y));
    x1 = __fadd_rn(__fmul_rn(a0, cs.y), __fmul_rn(a1, cs.x));
}

// Orderable (value, index) key: larger value wins, then larger index (the sampler's
// LAST index on ties, sampler.rs:572-578).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | idx;
}

// silu(g) * up (feed_forward.rs:31-39, compute.rs:641-645)
__device__ __forceinline__ float swiglu(float g, float up) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), up);
}

// EPI_PEERS publication, called by every thread of the CTA after its peer stores: the
// barrier orders all of the CTA's stores before thread 0's system-scope fence (a fence is
// cumulative over the writes the barrier made visible to its thread), so one fence per CTA
// does what a fence in every thread did at a fraction of the cost; the completion counter's
// atomics between two fences carry that order to the last CTA, whose release stores raise
// this call's flag on every rank.
__device__ __forceinline__ void peers_publish(const MvArgs& a) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned prev = atomicAdd(a.ar_counter, 1u);
        if (prev == gridDim.x - 1) {
            __threadfence_system();
            *a.ar_counter = 0u;  // zero for the next launch (stream-ordered)
            const unsigned long long ep = *a.ar_epoch + (unsigned long long)a.ar_call + 1ull;
            for (int p = 0; p < a.ar_out_n; p++)
                asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a.ar_out_flag[p]), "l"(ep)
                             : "memory");
        }
    }
}

// x''[unit] += the sum, in rank order, of the n <= NMAX vectors at in + p * cols (the ranks'
// partials, or one added vector) for the units this thread owns (tid, tid + NTH, ...). The
// loads of B units (B * NMAX <= 8 float4) are issued together, so a thread waits for one L2
// round trip per B units instead of one per unit.
template <int B, int NMAX, int NTH>
__device__ __forceinline__ void add_partials(const float* in_f, int n, int cols, float4* xs4,
                                             int nunits, int tid) {
    const float4* in = reinterpret_cast<const float4*>(in_f);
    const size_t stride = (size_t)cols / 4;
    for (int i0 = tid; i0 < nunits; i0 += NTH * B) {
        float4 t[B][NMAX];
#pragma unroll
        for (int b = 0; b < B; b++)
            if (i0 + b * NTH < nunits)
#pragma unroll
                for (int p = 0; p < NMAX; p++)
                    if (p < n) t[b][p] = __ldcg(in + p * stride + i0 + b * NTH);
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int i = i0 + b * NTH;
            if (i < nunits) {
                float4 r = t[b][0];
#pragma unroll
                for (int p = 1; p < NMAX; p++) {
                    if (p < n) {
                        r.x = __fadd_rn(r.x, t[b][p].x);
                        r.y = __fadd_rn(r.y, t[b][p].y);
                        r.z = __fadd_rn(r.z, t[b][p].z);
                        r.w = __fadd_rn(r.w, t[b][p].w);
                    }
                }
                const int c = i >> 3, ph = c * 8 + ((i & 7) ^ (c & 7));
                float4 v = xs4[ph];
                v.x = __fadd_rn(v.x, r.x);
                v.y = __fadd_rn(v.y, r.y);
                v.z = __fadd_rn(v.z, r.z);
                v.w = __fadd_rn(v.w, r.w);
                xs4[ph] = v;
            }
        }
    }
}

// (cos, sin) of RoPE pair i at position pos: from the model's table when it covers pos (the
// table holds rope_cs values, so both give the same bits), else computed.
__device__ __forceinline__ float2 rope_pair(const MvArgs& a, int i, int pos) {
    if (a.rope_cache && pos >= 0 && pos < a.rope_rows)
        return __ldg(a.rope_cache + (size_t)pos * (a.head_dim >> 1) + i);
    return rope_cs(i, a.head_dim, a.theta, pos);
}

// The x prologue of both kernels, run after the first weight copies are in flight and
// the barrier is initialised: waits for the previous kernel (PDL), stages x (nc rows of
// 128 B, 128-byte swizzle: unit u of chunk c at slot c*8 + (u ^ (c & 7))) by TMA, fills
// the RoPE pairs of this position meanwhile, waits for the peers' partials (bounded), then applies
//   x_eff = x (+ x_add or the sum of the peers' partials), written back by CTA 0,
//   optional RMSNorm (order 0: x * (inv * w); order 1: (x * inv) * w),
// and hands every 16-byte unit i (chunk c, slot ph, values v) to finish(i, c, ph, v,
// gmask), where the 8 units of a chunk are consecutive threads of one warp (gmask).
// Returns false, after recording the status, if a bounded wait gave up (every thread
// of the CTA then returns false).
template <int NTH, int EPI, typename Finish>
__device__ __forceinline__ bool mv_prologue(const MvArgs& a, const CUtensorMap* tm_x,
                                            uint8_t* xs, int nc, int xrows, float* red,
                                            uint64_t* bar, float2* rope_tab, Finish&& finish) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = NTH / 32;
    const bool has_add = a.x_add != nullptr || a.ar_in_n > 0, has_norm = a.norm_w != nullptr;
    float4* xs4 = reinterpret_cast<float4*>(xs);
    const int nunits = nc * 8;  // 16-byte units
    // The norm weights are weights: like the matrix they never depend on the previous
    // kernel, so this thread's first kNwPre units load before the wait.
    constexpr int kNwPre = 4;
    const float4* nw4 = reinterpret_cast<const float4*>(a.norm_w);
    float4 nwp[kNwPre];
#pragma unroll
    for (int j = 0; j < kNwPre; j++) {
        nwp[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (has_norm && tid + j * NTH < nunits) nwp[j] = __ldg(nw4 + tid + j * NTH);
    }
    if (!a.x_ready) pdl_wait();
    if (tid == 0) {
        const int nbox = xrows / kVecBoxRows;
        mbar_expect_tx(bar, (uint32_t)xrows * 128u);
        for (int b = 0; b < nbox; b++)
            tma_load_2d(xs + (size_t)b * kVecBoxRows * 128, tm_x, 0, b * kVecBoxRows, bar);
    }
    if constexpr (EPI == EPI_QKV_ROPE) {  // (cos, sin) of every pair at this position
        const int pos = a.position_dev ? *a.position_dev : a.position;
        for (int i = tid; i < (a.head_dim >> 1); i += NTH) rope_tab[i] = rope_pair(a, i, pos);
    }
    if (a.ar_in_n > 0) {  // wait for every rank's partial of this call (bounded)
        // fail fast: once any wait of this context has timed out, later ones do not wait
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
            if (!done) atomicExch(a.status, SSD_ERR_TIMEOUT);  // data below is then stale
        }
        __syncthreads();
    }
    const bool ok = mbar_wait(bar, 0, a.status);
    if (__syncthreads_or(!ok)) return false;  // timed out: status recorded

    const unsigned gmask = 0xFFu << (lane & 24);
    float inv = 1.0f;
    if (has_add || has_norm) {
        const bool wb = a.x_writeback != nullptr && blockIdx.x == 0;
        // hidden[i] += attn_output[i] (src/metal/compute.rs:547-549): the ranks' partials
        // (summed in rank order) or one added vector, into x'' in place
        if (has_add) {
            const int n = a.ar_in_n;
            if (n == 0)
                add_partials<8, 1, NTH>(a.x_add, 1, a.cols, xs4, nunits, tid);
            else if (n == 1)
                add_partials<8, 1, NTH>(a.ar_in, 1, a.cols, xs4, nunits, tid);
            else if (n == 2)
                add_partials<4, 2, NTH>(a.ar_in, 2, a.cols, xs4, nunits, tid);
            else if (n <= 4)
                add_partials<2, 4, NTH>(a.ar_in, n, a.cols, xs4, nunits, tid);
            else
                add_partials<1, kMaxPeers, NTH>(a.ar_in, n, a.cols, xs4, nunits, tid);
        }
        float ss = 0.0f;
        for (int i = tid; i < nunits; i += NTH) {  // this thread's own units: no barrier needed
            const int c = i >> 3, ph = c * 8 + ((i & 7) ^ (c & 7));
            const float4 v = xs4[ph];
            if (has_add && wb) reinterpret_cast<float4*>(a.x_writeback)[i] = v;
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
        if (has_norm) {
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; w++) tot += red[w];
            // inv_rms = 1 / sqrt(sum_sq / n + eps)   (src/metal/compute.rs:583-584)
            inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.cols), a.eps)));
        }
    }
    auto unit = [&](int i, float4 w) {
        const int c = i >> 3, ph = c * 8 + ((i & 7) ^ (c & 7));
        float4 v = xs4[ph];
        if (has_norm) {
            if (a.norm_order == 0) {  // x * (inv_rms * w)
                v.x = __fmul_rn(v.x, __fmul_rn(inv, w.x));
                v.y = __fmul_rn(v.y, __fmul_rn(inv, w.y));
                v.z = __fmul_rn(v.z, __fmul_rn(inv, w.z));
                v.w = __fmul_rn(v.w, __fmul_rn(inv, w.w));
            } else {  // (x * inv_rms) * w
                v.x = __fmul_rn(__fmul_rn(v.x, inv), w.x);
                v.y = __fmul_rn(__fmul_rn(v.y, inv), w.y);
                v.z = __fmul_rn(__fmul_rn(v.z, inv), w.z);
                v.w = __fmul_rn(__fmul_rn(v.w, inv), w.w);
            }
        }
        finish(i, c, ph, v, gmask);
    };
#pragma unroll
    for (int j = 0; j < kNwPre; j++)
        if (tid + j * NTH < nunits) unit(tid + j * NTH, nwp[j]);
    for (int i = tid + kNwPre * NTH; i < nunits; i += NTH)
        unit(i, has_norm ? __ldg(nw4 + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f));
    __syncthreads();
    pdl_trigger();
    return true;
}

// Resident CTAs per SM of one kernel at a given dynamic shared-memory size, cached
// per (kernel, device, size); sets the shared-memory opt-in attribute on first use.
template <typename K>
static int occupancy(ssd_ctx* ctx, K kern, int threads, size_t smem, int* out) {
    struct Entry {
        const void* fn;
        int dev;
        size_t smem;
        int blocks;
    };
    static Entry cache[512];
    static int n = 0;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    const void* fn = reinterpret_cast<const void*>(kern);
    bool attr_set = false;
    for (int i = 0; i < n; i++) {
        if (cache[i].fn != fn || cache[i].dev != ctx->device) continue;
        attr_set = true;
        if (cache[i].smem == smem) {
            *out = cache[i].blocks;
            return SSD_OK;
        }
    }
    if (!attr_set)
        SSD_CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)ctx->smem_optin));
    int nb = 0;
    SSD_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, threads, smem));
    SSD_REQ(nb > 0, SSD_ERR_SHAPE, "matvec kernel does not fit on an SM (%zu B smem)", smem);
    if (n < 512) cache[n++] = Entry{fn, ctx->device, smem, nb};
    *out = nb;
    return SSD_OK;
}

// Integer tensor-core kernel (matvec_tc.cu): launches it, or returns kTcNotCovered
// without launching when the shape is not one it covers.
constexpr int kTcNotCovered = -1000;
int launch_matvec_tc(ssd_ctx* ctx, int type, int epi, const MvArgs& a, cudaStream_t s, bool pdl);
// tcgen05 integer tensor-core kernel (matvec_i8.cu): launches it, or returns kI8NotCovered
// without launching when the type, shape or row map is not one it covers.
constexpr int kI8NotCovered = -1001;
int launch_matvec_i8(ssd_ctx* ctx, int type, int epi, const MvArgs& a, cudaStream_t s, bool pdl);
// Low-bit formats in the reference's block layouts (matvec_lowbit.cu): plain or residual.
int launch_matvec_lowbit(ssd_ctx* ctx, int type, int epi, const MvArgs& a, cudaStream_t s,
                         bool pdl);

}  // namespace ssd
