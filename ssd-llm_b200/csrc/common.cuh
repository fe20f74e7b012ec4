// common.cuh — shared definitions of the sm_100a backend (internal).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <string>

#include "../../include/ssdllm_cuda.h"

namespace ssd {

// --------------------------------------------------------------- errors
void set_error(const char* fmt, ...);

#define SSD_CK(call)                                                                  \
    do {                                                                              \
        cudaError_t e_ = (call);                                                      \
        if (e_ != cudaSuccess) {                                                      \
            ::ssd::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call,               \
                             cudaGetErrorString(e_));                                 \
            return SSD_ERR_CUDA;                                                      \
        }                                                                             \
    } while (0)

#define SSD_REQ(cond, code, ...)                                                      \
    do {                                                                              \
        if (!(cond)) {                                                                \
            ::ssd::set_error(__VA_ARGS__);                                            \
            return (code);                                                            \
        }                                                                             \
    } while (0)

#define SSD_TRY(expr)                                                                 \
    do {                                                                              \
        int s_ = (expr);                                                              \
        if (s_ != SSD_OK) return s_;                                                  \
    } while (0)

// Checks the last launch error (async errors surface at the next sync).
#define SSD_CK_LAUNCH() SSD_CK(cudaGetLastError())

// ------------------------------------------------------------- handles
}  // namespace ssd

struct ssd_ctx {
    int device = 0;
    int num_sms = 0;
    size_t smem_optin = 0;
    size_t smem_per_sm = 0;  // shared memory per SM usable by resident CTAs
    char name[256] = {0};
    cudaStream_t stream = nullptr;
    bool cached = false;  // owned by the process-wide cache; destroy is a no-op
    bool pdl = false;     // standalone launches use programmatic dependent launch
    // Scratch for the host-slice operators and split-K attention partials.
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    unsigned long long* argmax_key = nullptr;  // 8-byte (value, index) slot
    int* dev_status = nullptr;                 // device status word (bounded waits)
};

// Device layout of a quantized tensor (library-owned): structure of arrays so that
// every lane's load is an aligned 16-byte vector and a warp reads contiguous bytes.
//   Q4_0: qs = [rows][cols/32][16 B nibbles], meta = [rows][cols/32] f16 scales
//   Q8_0: qs = [rows][cols/32][32 B int8],   meta = [rows][cols/32] f16 scales
//   Q4_K: qs = [rows][cols/256][128 B],      meta = [rows][cols/256][16 B: d, dmin, 12 B sc]
//   Q5_K: qs = [rows][cols/32][32 B: q ^ 0x80, q = low4 | hbit << 4, element order],
//         meta = [rows][cols/256][16 B: d, dmin, 12 B 6-bit scales] (as Q4_K)
//   Q6_K: qs = [rows][cols/32][32 B int8 q - 32, element order],
//         meta = [rows][cols/32][4 B: int8 scale of elements 0-15, of 16-31, f16 d]
//   Q8_K: qs = [rows][cols/32][32 B int8], meta = [rows][cols/32] f32 d, then the
//         block sums of every super-block ([rows][cols/256][32 B], kept for the download)
//   F16 / BF16: qs = [rows][cols] 2 bytes each (as in the file)
//   F32 : qs = [rows][cols] f32
// The bytes are the reference's bytes, regrouped; nothing is re-quantized (Q5_K's and Q6_K's
// two bit fields are joined into one byte per weight; Q6_K's d is repeated per 32 weights).
struct ssd_weight {
    ssd_ctx* ctx = nullptr;
    int type = 0;
    int rows = 0, cols = 0;
    uint8_t* qs = nullptr;
    uint8_t* meta = nullptr;
    void* base = nullptr;  // allocation
    size_t alloc_bytes = 0;
    // Split-K scratch of the tensor-core matvec (matvec_i8.cu), inside the same allocation:
    // arrival counters per row tile (zeroed at allocation, reset by each launch's last
    // arrival) and two partial rows of 128 floats per CTA. Calls that use the same weight
    // must not overlap on the GPU.
    unsigned int* fix_counter = nullptr;
    float* fix_partial = nullptr;
};

struct ssd_kv_cache {
    ssd_ctx* ctx = nullptr;
    int capacity = 0, n_head_kv = 0, head_dim = 0, kv_dim = 0;
    int8_t* k = nullptr;
    int8_t* v = nullptr;
    float* k_scale = nullptr;
    float* v_scale = nullptr;
    void* base = nullptr;
};

namespace ssd {

// ------------------------------------------------------ device helpers
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// 2^23 + byte k of `b` (an unsigned byte), exact: byte_perm puts the byte in the low
// mantissa byte under exponent byte 0x4B.
__device__ __forceinline__ float magic_byte(uint32_t b, int k) {
    return __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7440u | k));
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ldg_u16(const void* p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// Programmatic dependent launch: wait for the producer grid / let dependents launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Counter-based generator: splitmix64 finaliser of (seed, tensor, index).
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
// N(0,1) for element `idx` of tensor `tid` (Box-Muller on two 24-bit uniforms).
__device__ __forceinline__ float synth_normal(uint64_t seed, uint32_t tid, uint64_t idx) {
    uint64_t h = mix64(seed ^ mix64(((uint64_t)tid << 40) ^ idx));
    float u1 = ((float)(uint32_t)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    float u2 = (float)((uint32_t)(h >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// Elements e0 .. e0+7 (e0 a multiple of 8) of a weight in the library layout, flat
// row-major index, dequantized exactly as dequantize_to_f32 (src/ssd/streamer.rs:93-180)
// and the Q4_K element formula of matvec_q4_k_cpu (src/metal/compute.rs:718-744).
__device__ __forceinline__ void dequant8(const ssd_weight& w, int64_t e0, float (&v)[8]) {
    if (w.type == SSD_TYPE_F32) {
        for (int t = 0; t < 8; t++) v[t] = reinterpret_cast<const float*>(w.qs)[e0 + t];
    } else if (w.type == SSD_TYPE_F16) {
        for (int t = 0; t < 8; t++)
            v[t] = f16_bits_to_f32(reinterpret_cast<const uint16_t*>(w.qs)[e0 + t]);
    } else if (w.type == SSD_TYPE_BF16) {  // bits << 16, compute.rs:2250-2253
        for (int t = 0; t < 8; t++)
            v[t] = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(w.qs)[e0 + t] << 16);
    } else if (w.type == SSD_TYPE_Q4_0) {
        const int64_t blk = e0 / 32;
        const int j0 = (int)(e0 % 32) / 2;  // byte index
        const float s = f16_bits_to_f32(reinterpret_cast<const uint16_t*>(w.meta)[blk]);
        const uint8_t* q = w.qs + blk * 16 + j0;
        for (int t = 0; t < 4; t++) {
            v[2 * t] = __fmul_rn((float)((int)(q[t] & 0x0F) - 8), s);
            v[2 * t + 1] = __fmul_rn((float)((int)(q[t] >> 4) - 8), s);
        }
    } else if (w.type == SSD_TYPE_Q8_0) {
        const int64_t blk = e0 / 32;
        const float s = f16_bits_to_f32(reinterpret_cast<const uint16_t*>(w.meta)[blk]);
        const int8_t* q = reinterpret_cast<const int8_t*>(w.qs) + e0;
        for (int t = 0; t < 8; t++) v[t] = __fmul_rn((float)q[t], s);
    } else if (w.type == SSD_TYPE_Q5_K) {  // scale * q - min, compute.rs:863-892
        const int64_t sbk = e0 / 256;
        const int sb = (int)(e0 % 256) / 32;
        const uint8_t* m = w.meta + sbk * 16;
        const float d = f16_bits_to_f32((uint16_t)(m[0] | (m[1] << 8)));
        const float dmin = f16_bits_to_f32((uint16_t)(m[2] | (m[3] << 8)));
        const uint8_t* sc = m + 4;
        int s6, m6;
        if (sb < 4) {
            s6 = sc[sb] & 0x3F;
            m6 = sc[sb + 4] & 0x3F;
        } else {
            s6 = (sc[sb - 4] >> 6) | ((sc[sb + 4] & 0x0F) << 2);
            m6 = (sc[sb] >> 6) | ((sc[sb + 4] >> 4) << 2);
        }
        const float scale = __fmul_rn(d, (float)s6), mn = __fmul_rn(dmin, (float)m6);
        const uint8_t* q = w.qs + e0;
        for (int t = 0; t < 8; t++) v[t] = __fsub_rn(__fmul_rn(scale, (float)(q[t] ^ 0x80)), mn);
    } else if (w.type == SSD_TYPE_Q8_K) {  // d * q, compute.rs:985-987
        const float dd = reinterpret_cast<const float*>(w.meta)[e0 / 32];
        const int8_t* q = reinterpret_cast<const int8_t*>(w.qs) + e0;
        for (int t = 0; t < 8; t++) v[t] = __fmul_rn(dd, (float)q[t]);
    } else if (w.type == SSD_TYPE_Q6_K) {  // (d * scale) * q, compute.rs:768-785
        const int64_t c = e0 / 32;
        const uint32_t m = reinterpret_cast<const uint32_t*>(w.meta)[c];
        const int sc = (int)(int8_t)((m >> (((e0 % 32) >= 16) ? 8 : 0)) & 0xFF);
        const float scale = __fmul_rn(f16_bits_to_f32((uint16_t)(m >> 16)), (float)sc);
        const int8_t* q = reinterpret_cast<const int8_t*>(w.qs) + e0;
        for (int t = 0; t < 8; t++) v[t] = __fmul_rn(scale, (float)q[t]);
    } else {  // Q4_K
        const int64_t sbk = e0 / 256;
        const int within = (int)(e0 % 256);
        const int sb = within / 32, j0 = (within % 32) / 2;
        const uint8_t* m = w.meta + sbk * 16;
        const float d = f16_bits_to_f32((uint16_t)(m[0] | (m[1] << 8)));
        const float dmin = f16_bits_to_f32((uint16_t)(m[2] | (m[3] << 8)));
        const uint8_t* sc = m + 4;
        int s6, m6;
        if (sb < 4) {
            s6 = sc[sb] & 0x3F;
            m6 = sc[sb + 4] & 0x3F;
        } else {
            s6 = (sc[sb - 4] >> 6) | ((sc[sb + 4] & 0x0F) << 2);
            m6 = (sc[sb] >> 6) | ((sc[sb + 4] >> 4) << 2);
        }
        const float scale = __fmul_rn(d, (float)s6), mn = __fmul_rn(dmin, (float)m6);
        const uint8_t* q = w.qs + sbk * 128 + sb * 16 + j0;
        for (int t = 0; t < 4; t++) {
            v[2 * t] = __fsub_rn(__fmul_rn(scale, (float)(q[t] & 0x0F)), mn);
            v[2 * t + 1] = __fsub_rn(__fmul_rn(scale, (float)(q[t] >> 4)), mn);
        }
    }
}

// RoPE angle of pair i at `pos` (src/metal/compute.rs:494-503): freq = 1 / theta^(2i/d),
// angle = pos * freq, rotation by (cos, sin). powf / sin / cos are evaluated in double
// and rounded once to float. Computed once per CTA for the head_dim/2 pairs.
__device__ __forceinline__ float2 rope_cs(int i, int head_dim, float theta, int pos) {
    const float e = __fdiv_rn(__fmul_rn(2.0f, (float)i), (float)head_dim);
    const float p = (float)pow((double)theta, (double)e);
    const float freq = __fdiv_rn(1.0f, p);
    const float ang = __fmul_rn((float)pos, freq);
    double sd, cd;
    sincos((double)ang, &sd, &cd);
    return make_float2((float)cd, (float)sd);
}
// ------------------------------------------------------------- TMA / mbarrier
// Device-side status word (one int per context, ssd_ctx::dev_status): a bounded wait
// that gives up records SSD_ERR_TIMEOUT there (read and cleared by
// ssd_ctx_device_status) and the kernel skips the work that depended on it.

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Waits for phase `parity` of the barrier with an iteration limit (about a second).
// Returns false, after recording SSD_ERR_TIMEOUT in *status, if the limit is reached.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
    const uint32_t addr = smem_u32(bar);
    for (uint32_t it = 0; it < (1u << 20); it++) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    if (status) atomicExch(status, SSD_ERR_TIMEOUT);
    return false;
}
// 2-D tiled TMA load (no multicast) of box {c0, c1} into shared memory, completing on bar.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// 3-D tiled TMA load (no multicast) of box {c0, c1, c2} into shared memory.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum of v over a CTA of NT threads (red: NT / 32 floats of shared memory); every
// thread gets the total, the warps' sums added in warp order.
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < NT / 32; w++) t += red[w];
    return t;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ------------------------------------------------------------ host side
// The low-bit formats kept in the reference's block layout (lowbit.cuh).
__host__ __device__ constexpr bool is_lowbit(int t) {
    return t == SSD_TYPE_Q2_K || t == SSD_TYPE_Q3_K || t == SSD_TYPE_IQ4_NL ||
           t == SSD_TYPE_IQ4_XS || t == SSD_TYPE_IQ3_XXS || t == SSD_TYPE_IQ3_S ||
           t == SSD_TYPE_IQ2_XXS || t == SSD_TYPE_IQ2_XS;
}
__host__ __device__ constexpr int type_block(int type) {
    switch (type) {
        case SSD_TYPE_Q4_0:
        case SSD_TYPE_Q8_0: return 32;
        case SSD_TYPE_Q4_K:
        case SSD_TYPE_Q5_K:
        case SSD_TYPE_Q6_K:
        case SSD_TYPE_Q8_K: return 256;
        case SSD_TYPE_F32:
        case SSD_TYPE_F16:
        case SSD_TYPE_BF16: return 1;
        case SSD_TYPE_IQ4_NL: return 32;
        case SSD_TYPE_Q2_K:
        case SSD_TYPE_Q3_K:
        case SSD_TYPE_IQ4_XS:
        case SSD_TYPE_IQ3_XXS:
        case SSD_TYPE_IQ3_S:
        case SSD_TYPE_IQ2_XXS:
        case SSD_TYPE_IQ2_XS: return 256;
        default: return 0;
    }
}
__host__ __device__ constexpr int type_block_bytes(int type) {
    switch (type) {
        case SSD_TYPE_Q4_0: return 18;
        case SSD_TYPE_Q8_0: return 34;
        case SSD_TYPE_Q4_K: return 144;
        case SSD_TYPE_Q5_K: return 176;
        case SSD_TYPE_Q6_K: return 210;
        case SSD_TYPE_Q8_K: return 292;
        case SSD_TYPE_F32: return 4;
        case SSD_TYPE_F16:
        case SSD_TYPE_BF16: return 2;
        case SSD_TYPE_Q2_K: return 84;
        case SSD_TYPE_Q3_K: return 110;
        case SSD_TYPE_IQ4_NL: return 18;
        case SSD_TYPE_IQ4_XS: return 148;
        case SSD_TYPE_IQ3_XXS: return 98;
        case SSD_TYPE_IQ3_S: return 110;
        case SSD_TYPE_IQ2_XXS: return 66;
        case SSD_TYPE_IQ2_XS: return 74;
        default: return 0;
    }
}

// A NULL stream argument is CUDA's default stream (it orders with torch's default
// stream and every other legacy-stream user); the context's own stream is only used
// when passed explicitly (ssd_ctx_stream) and by the synchronous host-slice calls.
inline cudaStream_t pick_stream(ssd_ctx* ctx, void* s) {
    (void)ctx;
    return (cudaStream_t)s;
}

int check_ctx(ssd_ctx* ctx);
// Zeroes `bytes` at device pointer p and waits until it is done. The context's stream is
// non-blocking, so a plain cudaMemset (legacy default stream, asynchronous for device
// memory) would not be ordered before kernels the caller launches next on that stream;
// every one-time initialisation of device state goes through this.
int zero_device(ssd_ctx* ctx, void* p, size_t bytes);
// Encodes a 2-D fp32 tensor map over a vector of n floats viewed as rows of 32 floats
// (128 B), box = 32 rows, 128-byte swizzle: chunk c's 16-byte unit u lands at unit
// u ^ (c & 7) of its row, so the 8 units a lane reads are bank-conflict free across a
// quarter warp. n must be a multiple of 32 and ptr 16-byte aligned.
int encode_vec_map(CUtensorMap* map, const float* ptr, int n);
// 2-D byte tensor map over `rows` rows of row_bytes (16-byte multiple, >= 128) at ptr
// (16-byte aligned): box = 128 bytes x box_rows rows, 128-byte swizzle (16-byte unit u
// of box row r lands at unit u ^ (r & 7)); out-of-range rows and bytes read as zero.
int encode_rows_map(CUtensorMap* map, const void* ptr, uint64_t row_bytes, uint64_t rows,
                    uint32_t box_rows);
// 3-D view of the same rows as 128-byte blocks: box = box_blocks blocks x box_rows rows,
// landing in shared memory as [block][row][128 B] with the 128-byte swizzle (unit u of
// shared row r at u ^ (r & 7) when box_rows is 8). row_bytes must be a multiple of 128.
int encode_blocks_map(CUtensorMap* map, const void* ptr, uint64_t row_bytes, uint64_t rows,
                      uint32_t box_rows, uint32_t box_blocks);
// 2-D byte tensor map over `rows` rows of row_bytes at ptr: box = box_bytes x box_rows,
// the 128-byte swizzle (box_bytes 128) or none; out-of-range rows read as zero.
int encode_bytes_map(CUtensorMap* map, const void* ptr, uint64_t row_bytes, uint64_t rows,
                     uint32_t box_bytes, uint32_t box_rows, bool swizzle128);
constexpr int kVecBoxRows = 32;
// Largest grid of the tensor-core matvec (matvec_i8.cu); sizes the split-K scratch of a weight.
constexpr int kI8MaxGrid = 160;
// Device layout of one weight (library layout, see ssd_weight): the payload, the scales,
// and the tensor-core kernel's split-K counters and partial rows, each 256-byte aligned.
struct WeightLayout {
    size_t qs_pad = 0, meta_bytes = 0, meta_pad = 0, counter_bytes = 0, partial_bytes = 0;
    size_t total = 0;  // bytes from the weight's base (256-byte aligned)
    bool fix = false;  // carries split-K scratch (the counters must start at zero)
};
int weight_layout(int type, int rows, int cols, WeightLayout* out);
// Points *w (caller-owned; base left null, so ssd_weight_free does not free it) at the
// regions of `L` from p (256-byte aligned device memory of L.total bytes).
void carve_weight(ssd_ctx* ctx, int type, int rows, int cols, const WeightLayout& L, uint8_t* p,
                  ssd_weight* w);
// The reference's raw bytes (already on the device) into w's layout on stream s: dense and
// low-bit types as they are, the others through the repack kernel.
int upload_raw(ssd_weight* w, const void* raw_dev, cudaStream_t s);
int alloc_weight(ssd_ctx* ctx, int type, int rows, int cols, ssd_weight** out);
int ensure_scratch(ssd_ctx* ctx, size_t bytes);

// Launch with the programmatic-stream-serialization attribute (PDL) so that the
// kernel's pre-wait prologue (weight prefetch) overlaps the previous kernel's tail.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace ssd
