// ctx.cu — context, errors, HBM-resident weights, (de)quantization and synthetic inputs.
//
// Replaces MetalCompute::new / MetalGpu::new (src/metal/compute.rs:47-72,
// src/metal/gpu.rs:73-160) and the streamer's dequantize_to_f32
// (src/ssd/streamer.rs:93-180).
#include <stdarg.h>
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "lowbit.cuh"

namespace ssd {

static thread_local char g_err[1024];


// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int tensor_map_fn(EncodeTiledFn* out) {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        SSD_CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q));
        SSD_REQ(f != nullptr && q == cudaDriverEntryPointSuccess, SSD_ERR_CUDA,
                "cuTensorMapEncodeTiled unavailable");
        fn = (EncodeTiledFn)f;
    }
    *out = fn;
    return SSD_OK;
}

int encode_vec_map(CUtensorMap* map, const float* ptr, int n) {
    EncodeTiledFn fn;
    SSD_TRY(tensor_map_fn(&fn));
    SSD_REQ(ptr && ((uintptr_t)ptr & 15u) == 0 && n > 0 && n % 32 == 0, SSD_ERR_ARG,
            "tensor map: vector must be 16-byte aligned with a multiple of 32 floats");
    cuuint64_t dims[2] = {32, (cuuint64_t)(n / 32)};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {32, (cuuint32_t)kVecBoxRows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)ptr, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    SSD_REQ(r == CUDA_SUCCESS, SSD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SSD_OK;
}

int encode_rows_map(CUtensorMap* map, const void* ptr, uint64_t row_bytes, uint64_t rows,
                    uint32_t box_rows) {
    EncodeTiledFn fn;
    SSD_TRY(tensor_map_fn(&fn));
    SSD_REQ(ptr && ((uintptr_t)ptr & 15u) == 0 && row_bytes % 16 == 0 && row_bytes >= 128 &&
                rows >= box_rows && box_rows >= 1 && box_rows <= 256,
            SSD_ERR_ARG, "tensor map: rows of %llu bytes x %llu not tileable",
            (unsigned long long)row_bytes, (unsigned long long)rows);
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)ptr, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    SSD_REQ(r == CUDA_SUCCESS, SSD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SSD_OK;
}

int encode_blocks_map(CUtensorMap* map, const void* ptr, uint64_t row_bytes, uint64_t rows,
                      uint32_t box_rows, uint32_t box_blocks) {
    EncodeTiledFn fn;
    SSD_TRY(tensor_map_fn(&fn));
    SSD_REQ(ptr && ((uintptr_t)ptr & 15u) == 0 && row_bytes % 128 == 0 && row_bytes >= 128 &&
                rows >= box_rows && box_rows >= 1 && box_rows <= 256 && box_blocks >= 1 &&
                box_blocks <= 256,
            SSD_ERR_ARG, "tensor map: rows of %llu bytes x %llu not tileable in 128-byte blocks",
            (unsigned long long)row_bytes, (unsigned long long)rows);
    // dims: byte within a 128-byte block, row, block; the box lands as [block][row][128 B]
    cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)(row_bytes / 128)};
    cuuint64_t strides[2] = {(cuuint64_t)row_bytes, 128};
    cuuint32_t box[3] = {128, box_rows, box_blocks};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, (void*)ptr, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    SSD_REQ(r == CUDA_SUCCESS, SSD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SSD_OK;
}

int encode_bytes_map(CUtensorMap* map, const void* ptr, uint64_t row_bytes, uint64_t rows,
                     uint32_t box_bytes, uint32_t box_rows, bool swizzle128) {
    EncodeTiledFn fn;
    SSD_TRY(tensor_map_fn(&fn));
    SSD_REQ(ptr && ((uintptr_t)ptr & 15u) == 0 && row_bytes % 16 == 0 && rows >= 1 &&
                box_bytes % 16 == 0 && box_bytes >= 16 && box_bytes <= (swizzle128 ? 128u : 256u) &&
                box_rows >= 1 && box_rows <= 256,
            SSD_ERR_ARG, "tensor map: rows of %llu bytes (box %u x %u) not tileable",
            (unsigned long long)row_bytes, box_bytes, box_rows);
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {box_bytes, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)ptr, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    SSD_REQ(r == CUDA_SUCCESS, SSD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SSD_OK;
}

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int check_ctx(ssd_ctx* ctx) {
    SSD_REQ(ctx != nullptr, SSD_ERR_ARG, "null context");
    SSD_CK(cudaSetDevice(ctx->device));
    return SSD_OK;
}

int zero_device(ssd_ctx* ctx, void* p, size_t bytes) {
    if (!bytes) return SSD_OK;
    SSD_CK(cudaMemsetAsync(p, 0, bytes, ctx->stream));
    SSD_CK(cudaStreamSynchronize(ctx->stream));
    return SSD_OK;
}

int ensure_scratch(ssd_ctx* ctx, size_t bytes) {
    if (ctx->scratch_bytes >= bytes) return SSD_OK;
    if (ctx->scratch) {  // callers may have work in flight on any stream
        SSD_CK(cudaDeviceSynchronize());
        SSD_CK(cudaFree(ctx->scratch));
        ctx->scratch = nullptr;
        ctx->scratch_bytes = 0;
    }
    size_t b = bytes < (1u << 20) ? (1u << 20) : bytes;
    if (cudaMalloc(&ctx->scratch, b) != cudaSuccess) {
        cudaGetLastError();
        set_error("scratch allocation of %zu bytes failed", b);
        return SSD_ERR_NOMEM;
    }
    ctx->scratch_bytes = b;
    return SSD_OK;
}

// ----------------------------------------------------- layout kernels

// Reference layout (AoS blocks) -> library layout (SoA). One thread per block.
__global__ void k_repack(const uint8_t* __restrict__ raw, int type, int64_t nblocks,
                         uint8_t* __restrict__ qs, uint8_t* __restrict__ meta) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    if (type == SSD_TYPE_Q4_0) {
        const uint8_t* s = raw + i * 18;
        uint8_t* d = qs + i * 16;
#pragma unroll
        for (int j = 0; j < 16; j++) d[j] = s[2 + j];
        meta[2 * i] = s[0];
        meta[2 * i + 1] = s[1];
    } else if (type == SSD_TYPE_Q8_0) {
        const uint8_t* s = raw + i * 34;
        uint8_t* d = qs + i * 32;
#pragma unroll
        for (int j = 0; j < 32; j++) d[j] = s[2 + j];
        meta[2 * i] = s[0];
        meta[2 * i + 1] = s[1];
    } else if (type == SSD_TYPE_Q8_K) {  // bytes as they are, d per 32, sums aside
        const uint8_t* s = raw + i * 292;
        for (int j = 0; j < 256; j++) qs[i * 256 + j] = s[4 + j];
        for (int c = 0; c < 8; c++)
            for (int j = 0; j < 4; j++) meta[(i * 8 + c) * 4 + j] = s[j];
        uint8_t* sums = meta + nblocks * 32;
        for (int j = 0; j < 32; j++) sums[i * 32 + j] = s[260 + j];
    } else if (type == SSD_TYPE_Q5_K) {  // one byte per weight (q ^ 0x80) + the header
        const uint8_t* s = raw + i * 176;
        uint8_t* d = qs + i * 256;
        for (int idx = 0; idx < 256; idx++) {  // compute.rs:877-890
            const uint8_t b = s[48 + (idx / 32) * 16 + (idx % 32) / 2];
            const int low4 = (idx & 1) ? (b >> 4) & 0x0F : b & 0x0F;
            const int hbit = (s[16 + idx / 8] >> (idx % 8)) & 1;
            d[idx] = (uint8_t)((low4 | (hbit << 4)) ^ 0x80);
        }
#pragma unroll
        for (int j = 0; j < 16; j++) meta[i * 16 + j] = s[j];
    } else if (type == SSD_TYPE_Q6_K) {  // one signed byte per weight + a word per 32
        const uint8_t* s = raw + i * 210;
        int8_t* d = reinterpret_cast<int8_t*>(qs) + i * 256;
        for (int idx = 0; idx < 256; idx++) {  // compute.rs:771-780
            const uint8_t qlb = s[idx / 2];
            const int low4 = (idx & 1) ? (qlb >> 4) & 0x0F : qlb & 0x0F;
            const int high2 = (s[128 + idx / 4] >> ((idx % 4) * 2)) & 0x03;
            d[idx] = (int8_t)(((high2 << 4) | low4) - 32);
        }
        for (int c = 0; c < 8; c++) {
            uint8_t* m = meta + (i * 8 + c) * 4;
            m[0] = s[192 + 2 * c];
            m[1] = s[192 + 2 * c + 1];
            m[2] = s[208];
            m[3] = s[209];
        }
    } else {  // Q4_K
        const uint8_t* s = raw + i * 144;
        uint8_t* d = qs + i * 128;
#pragma unroll 8
        for (int j = 0; j < 128; j++) d[j] = s[16 + j];
#pragma unroll
        for (int j = 0; j < 16; j++) meta[i * 16 + j] = s[j];
    }
}

__global__ void k_unpack(const uint8_t* __restrict__ qs, const uint8_t* __restrict__ meta, int type,
                         int64_t nblocks, uint8_t* __restrict__ raw) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    if (type == SSD_TYPE_Q4_0) {
        uint8_t* d = raw + i * 18;
        d[0] = meta[2 * i];
        d[1] = meta[2 * i + 1];
        for (int j = 0; j < 16; j++) d[2 + j] = qs[i * 16 + j];
    } else if (type == SSD_TYPE_Q8_0) {
        uint8_t* d = raw + i * 34;
        d[0] = meta[2 * i];
        d[1] = meta[2 * i + 1];
        for (int j = 0; j < 32; j++) d[2 + j] = qs[i * 32 + j];
    } else if (type == SSD_TYPE_Q8_K) {  // exact inverse of k_repack
        uint8_t* d = raw + i * 292;
        for (int j = 0; j < 4; j++) d[j] = meta[i * 32 + j];
        for (int j = 0; j < 256; j++) d[4 + j] = qs[i * 256 + j];
        for (int j = 0; j < 32; j++) d[260 + j] = meta[nblocks * 32 + i * 32 + j];
    } else if (type == SSD_TYPE_Q5_K) {  // exact inverse of k_repack
        uint8_t* d = raw + i * 176;
        for (int j = 0; j < 16; j++) d[j] = meta[i * 16 + j];
        for (int j = 16; j < 176; j++) d[j] = 0;
        for (int idx = 0; idx < 256; idx++) {
            const int v = qs[i * 256 + idx] ^ 0x80;
            d[48 + (idx / 32) * 16 + (idx % 32) / 2] |= (uint8_t)((v & 0x0F) << (4 * (idx & 1)));
            d[16 + idx / 8] |= (uint8_t)(((v >> 4) & 1) << (idx % 8));
        }
    } else if (type == SSD_TYPE_Q6_K) {  // exact inverse of k_repack
        uint8_t* d = raw + i * 210;
        for (int j = 0; j < 192; j++) d[j] = 0;
        const int8_t* q = reinterpret_cast<const int8_t*>(qs) + i * 256;
        for (int idx = 0; idx < 256; idx++) {
            const int v = q[idx] + 32;
            d[idx / 2] |= (uint8_t)((v & 0x0F) << (4 * (idx & 1)));
            d[128 + idx / 4] |= (uint8_t)(((v >> 4) & 0x03) << (2 * (idx % 4)));
        }
        for (int c = 0; c < 8; c++) {
            d[192 + 2 * c] = meta[(i * 8 + c) * 4];
            d[192 + 2 * c + 1] = meta[(i * 8 + c) * 4 + 1];
        }
        d[208] = meta[i * 32 + 2];
        d[209] = meta[i * 32 + 3];
    } else {
        uint8_t* d = raw + i * 144;
        for (int j = 0; j < 16; j++) d[j] = meta[i * 16 + j];
        for (int j = 0; j < 128; j++) d[16 + j] = qs[i * 128 + j];
    }
}

// ------------------------------------------------------- quantizers
// Builder's quantizers (the reference has none for these formats), exact inverses
// of the reference decoders. Every float operation is an explicit round-to-nearest
// intrinsic so the device result is bit-identical to the host restatement.

__device__ void quant_block_q4_0(const float* x, uint8_t* nib16, uint16_t* d_out) {
    float amax = 0.0f, m = 0.0f;
    for (int j = 0; j < 32; j++) {
        float a = fabsf(x[j]);
        if (a > amax) {
            amax = a;
            m = x[j];
        }
    }
    float d = __fdiv_rn(m, -8.0f);
    float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    *d_out = __half_as_ushort(__float2half_rn(d));
    for (int j = 0; j < 16; j++) {
        int q0 = (int)floorf(__fadd_rn(__fmul_rn(x[2 * j], id), 8.5f));
        int q1 = (int)floorf(__fadd_rn(__fmul_rn(x[2 * j + 1], id), 8.5f));
        q0 = min(15, max(0, q0));
        q1 = min(15, max(0, q1));
        nib16[j] = (uint8_t)(q0 | (q1 << 4));
    }
}

__device__ void quant_block_q8_0(const float* x, int8_t* q32, uint16_t* d_out) {
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
    float d = __fdiv_rn(amax, 127.0f);
    float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    *d_out = __half_as_ushort(__float2half_rn(d));
    for (int j = 0; j < 32; j++) {
        int q = (int)roundf(__fmul_rn(x[j], id));
        q32[j] = (int8_t)min(127, max(-127, q));
    }
}

// Q4_K super-block: meta16 = f16 d, f16 dmin, 12 bytes of 6-bit (scale, min);
// qs128 = 16 nibble bytes per 32-wide sub-block (element 2j = low nibble of byte j).
__device__ void quant_block_q4_k(const float* x, uint8_t* meta16, uint8_t* qs128) {
    float scale[8], mins[8], max_scale = 0.0f, max_min = 0.0f;
    for (int s = 0; s < 8; s++) {
        float lo = 0.0f, hi = 0.0f;
        for (int j = 0; j < 32; j++) {
            float v = x[s * 32 + j];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        scale[s] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
        mins[s] = -lo;
        if (scale[s] > max_scale) max_scale = scale[s];
        if (mins[s] > max_min) max_min = mins[s];
    }
    __half dh = __float2half_rn(__fdiv_rn(max_scale, 63.0f));
    __half mh = __float2half_rn(__fdiv_rn(max_min, 63.0f));
    float d = __half2float(dh), dmin = __half2float(mh);
    // f16 d and dmin, little-endian: aligned 16-bit stores (meta16 is 2-byte aligned)
    reinterpret_cast<uint16_t*>(meta16)[0] = __half_as_ushort(dh);
    reinterpret_cast<uint16_t*>(meta16)[1] = __half_as_ushort(mh);
    uint8_t sc6[8], m6[8];
    for (int s = 0; s < 8; s++) {
        sc6[s] = (uint8_t)(d > 0.0f ? min(63, max(0, (int)roundf(__fdiv_rn(scale[s], d)))) : 0);
        m6[s] = (uint8_t)(dmin > 0.0f ? min(63, max(0, (int)roundf(__fdiv_rn(mins[s], dmin)))) : 0);
    }
    uint8_t* sc = meta16 + 4;
    for (int s = 0; s < 4; s++) {
        sc[s] = (uint8_t)((sc6[s] & 0x3F) | ((sc6[s + 4] & 0x3) << 6));
        sc[s + 4] = (uint8_t)((m6[s] & 0x3F) | ((m6[s + 4] & 0x3) << 6));
        sc[s + 8] = (uint8_t)((sc6[s + 4] >> 2) | ((m6[s + 4] >> 2) << 4));
    }
    for (int s = 0; s < 8; s++) {
        float es = __fmul_rn(d, (float)sc6[s]);
        float em = __fmul_rn(dmin, (float)m6[s]);
        for (int j = 0; j < 16; j++) {
            int q0 = 0, q1 = 0;
            if (es > 0.0f) {
                q0 = min(15, max(0, (int)roundf(__fdiv_rn(__fadd_rn(x[s * 32 + 2 * j], em), es))));
                q1 = min(15, max(0, (int)roundf(__fdiv_rn(__fadd_rn(x[s * 32 + 2 * j + 1], em), es))));
            }
            qs128[s * 16 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

// f32 rows -> reference block layout.
__global__ void k_quantize_raw(const float* __restrict__ x, int type, int64_t nblocks,
                               uint8_t* __restrict__ raw) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    if (type == SSD_TYPE_Q4_0) {
        uint8_t* o = raw + i * 18;
        uint16_t d;
        uint8_t nib[16];
        quant_block_q4_0(x + i * 32, nib, &d);
        *reinterpret_cast<uint16_t*>(o) = d;  // 18-byte blocks: 2-byte aligned
        for (int j = 0; j < 16; j++) o[2 + j] = nib[j];
    } else if (type == SSD_TYPE_Q8_0) {
        uint8_t* o = raw + i * 34;
        uint16_t d;
        int8_t q[32];
        quant_block_q8_0(x + i * 32, q, &d);
        *reinterpret_cast<uint16_t*>(o) = d;  // 34-byte blocks: 2-byte aligned
        for (int j = 0; j < 32; j++) o[2 + j] = (uint8_t)q[j];
    } else {
        uint8_t* o = raw + i * 144;
        quant_block_q4_k(x + i * 256, o, o + 16);
    }
}

// Synthetic N(0, std^2) weights, generated and quantized straight into the
// library layout. Block i of the window -> global (row, col) -> hashed normals.
__global__ void k_synth_weight(int type, uint64_t seed, uint32_t tid, float std_dev,
                               int64_t total_cols, int row0, int rows, int col0, int cols,
                               uint8_t* __restrict__ qs, uint8_t* __restrict__ meta) {
    int bs = (type == SSD_TYPE_Q4_K) ? 256 : 32;
    int64_t bpr = cols / bs;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * bpr) return;
    int64_t r = i / bpr, b = i % bpr;
    uint64_t base = (uint64_t)(row0 + r) * (uint64_t)total_cols + (uint64_t)(col0 + b * bs);
    float x[256];
    for (int j = 0; j < bs; j++) x[j] = __fmul_rn(synth_normal(seed, tid, base + j), std_dev);
    if (type == SSD_TYPE_Q4_0) {
        uint16_t d;
        uint8_t nib[16];
        quant_block_q4_0(x, nib, &d);
        uint4 v;
        memcpy(&v, nib, 16);
        reinterpret_cast<uint4*>(qs)[i] = v;
        reinterpret_cast<uint16_t*>(meta)[i] = d;
    } else if (type == SSD_TYPE_Q8_0) {
        uint16_t d;
        int8_t q[32];
        quant_block_q8_0(x, q, &d);
        uint4 v[2];
        memcpy(v, q, 32);
        reinterpret_cast<uint4*>(qs)[2 * i] = v[0];
        reinterpret_cast<uint4*>(qs)[2 * i + 1] = v[1];
        reinterpret_cast<uint16_t*>(meta)[i] = d;
    } else {
        quant_block_q4_k(x, meta + i * 16, qs + i * 128);
    }
}

__global__ void k_synth_f32(uint64_t seed, uint32_t tid, float mean, float std_dev,
                            int64_t total_cols, int row0, int rows, int col0, int cols,
                            float* __restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * cols) return;
    int64_t r = i / cols, c = i % cols;
    uint64_t idx = (uint64_t)(row0 + r) * (uint64_t)total_cols + (uint64_t)(col0 + c);
    out[i] = __fadd_rn(__fmul_rn(synth_normal(seed, tid, idx), std_dev), mean);
}

// ----------------------------------------------------------- dequant
// Bit-exact with src/ssd/streamer.rs:128-180 (q as f32 * scale, one rounding) and
// the Q4_K element formula src/metal/compute.rs:735-741 (two roundings, no FMA).
__global__ void k_dequant(const ssd_weight w, float* __restrict__ out) {
    int64_t n = (int64_t)w.rows * w.cols;
    int64_t e0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;  // 8 elements
    if (e0 >= n) return;
    if (is_lowbit(w.type)) {  // decode the 32-element group holding e0 .. e0 + 7
        const int64_t r = e0 / w.cols;
        const int c = (int)(e0 % w.cols), bs = type_block(w.type);
        const uint8_t* blk = w.qs + (size_t)r * (w.cols / bs) * type_block_bytes(w.type) +
                             (size_t)(c / bs) * type_block_bytes(w.type);
        float g[32];
        lowbit_group_any(w.type, blk, (c % bs) / 32, g);
        for (int t = 0; t < 8; t++) out[e0 + t] = g[c % 32 + t];
        return;
    }
    float v[8];
    dequant8(w, e0, v);
    for (int t = 0; t < 8; t++) out[e0 + t] = v[t];
}

static std::mutex g_ctx_mu;
static ssd_ctx* g_ctx_cache[64] = {nullptr};

}  // namespace ssd

using namespace ssd;

// =============================================================== C ABI

extern "C" int ssd_abi_version(void) { return SSD_ABI_VERSION; }

extern "C" const char* ssd_status_str(int s) {
    switch (s) {
        case SSD_OK: return "ok";
        case SSD_ERR_ARG: return "invalid argument";
        case SSD_ERR_TYPE: return "unsupported ggml type";
        case SSD_ERR_SHAPE: return "shape mismatch";
        case SSD_ERR_CUDA: return "CUDA error";
        case SSD_ERR_TIMEOUT: return "device wait timed out";
        case SSD_ERR_NCCL: return "NCCL error";
        case SSD_ERR_NOMEM: return "out of device memory";
        case SSD_ERR_STATE: return "invalid state";
        default: return "unknown status";
    }
}

extern "C" const char* ssd_last_error(void) { return g_err; }

extern "C" int ssd_ctx_create(int device, ssd_ctx** out) {
    SSD_REQ(out != nullptr, SSD_ERR_ARG, "null out");
    int n = 0;
    SSD_CK(cudaGetDeviceCount(&n));
    SSD_REQ(device >= 0 && device < n, SSD_ERR_ARG, "device %d out of range (%d)", device, n);
    SSD_CK(cudaSetDevice(device));
    cudaDeviceProp p;
    SSD_CK(cudaGetDeviceProperties(&p, device));
    SSD_REQ(p.major >= 10, SSD_ERR_ARG, "device %d is sm_%d%d; this library is built for sm_100a",
            device, p.major, p.minor);
    ssd_ctx* c = new ssd_ctx();
    c->device = device;
    c->num_sms = p.multiProcessorCount;
    c->smem_optin = p.sharedMemPerBlockOptin;
    c->smem_per_sm = p.sharedMemPerMultiprocessor;
    snprintf(c->name, sizeof(c->name), "%s", p.name);
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&c->argmax_key, 64) != cudaSuccess ||
        cudaMemsetAsync(c->argmax_key, 0, 64, c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess) {
        set_error("context setup failed: %s", cudaGetErrorString(cudaGetLastError()));
        delete c;
        return SSD_ERR_CUDA;
    }
    c->dev_status = reinterpret_cast<int*>(c->argmax_key + 4);  // same 64-byte allocation
    *out = c;
    return SSD_OK;
}

extern "C" int ssd_ctx_get(int device, ssd_ctx** out) {
    SSD_REQ(out != nullptr && device >= 0 && device < 64, SSD_ERR_ARG, "bad device/out");
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    if (!g_ctx_cache[device]) {
        ssd_ctx* c = nullptr;
        SSD_TRY(ssd_ctx_create(device, &c));
        c->cached = true;
        g_ctx_cache[device] = c;
    }
    *out = g_ctx_cache[device];
    return SSD_OK;
}

extern "C" int ssd_ctx_destroy(ssd_ctx* ctx) {
    if (!ctx || ctx->cached) return SSD_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->argmax_key) cudaFree(ctx->argmax_key);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return SSD_OK;
}

extern "C" int ssd_ctx_stream(ssd_ctx* ctx, void** s) {
    SSD_REQ(ctx && s, SSD_ERR_ARG, "null arg");
    *s = (void*)ctx->stream;
    return SSD_OK;
}

extern "C" int ssd_ctx_sync(ssd_ctx* ctx) {
    SSD_TRY(check_ctx(ctx));
    SSD_CK(cudaStreamSynchronize(ctx->stream));
    return SSD_OK;
}

extern "C" int ssd_ctx_device_status(ssd_ctx* ctx, int* status) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(status != nullptr, SSD_ERR_ARG, "null status");
    SSD_CK(cudaDeviceSynchronize());
    SSD_CK(cudaMemcpy(status, ctx->dev_status, sizeof(int), cudaMemcpyDeviceToHost));
    return zero_device(ctx, ctx->dev_status, sizeof(int));
}

extern "C" int ssd_ctx_set_pdl(ssd_ctx* ctx, int on) {
    SSD_REQ(ctx != nullptr, SSD_ERR_ARG, "null ctx");
    ctx->pdl = on != 0;
    return SSD_OK;
}

extern "C" int ssd_ctx_info(ssd_ctx* ctx, int* num_sms, char* name, size_t name_len) {
    SSD_REQ(ctx != nullptr, SSD_ERR_ARG, "null ctx");
    if (num_sms) *num_sms = ctx->num_sms;
    if (name && name_len) snprintf(name, name_len, "%s", ctx->name);
    return SSD_OK;
}

extern "C" int ssd_copy_to_device(ssd_ctx* ctx, void* dst, const void* src, size_t bytes) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(dst && src, SSD_ERR_ARG, "null pointer");
    SSD_CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    SSD_CK(cudaStreamSynchronize(ctx->stream));
    return SSD_OK;
}

extern "C" int ssd_copy_to_host(ssd_ctx* ctx, void* dst, const void* src, size_t bytes) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(dst && src, SSD_ERR_ARG, "null pointer");
    SSD_CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    SSD_CK(cudaStreamSynchronize(ctx->stream));
    return SSD_OK;
}

extern "C" size_t ssd_row_bytes(int type, int64_t cols) {
    int bs = type_block(type);
    if (!bs || cols % bs) return 0;
    return (size_t)(cols / bs) * (size_t)type_block_bytes(type);
}

namespace ssd {
int weight_layout(int type, int rows, int cols, WeightLayout* out) {
    SSD_REQ(type == SSD_TYPE_Q4_0 || type == SSD_TYPE_Q8_0 || type == SSD_TYPE_Q4_K ||
                type == SSD_TYPE_Q5_K || type == SSD_TYPE_Q6_K || type == SSD_TYPE_Q8_K ||
                type == SSD_TYPE_F16 || type == SSD_TYPE_BF16 || type == SSD_TYPE_F32 ||
                is_lowbit(type),
            SSD_ERR_TYPE,
            "ggml type %d not supported (F32=0, F16=1, Q4_0=2, Q8_0=8, Q2_K=10, Q3_K=11, "
            "Q4_K=12, Q5_K=13, Q6_K=14, Q8_K=15, IQ2_XXS=16, IQ2_XS=17, IQ3_XXS=18, IQ4_NL=20, "
            "IQ3_S=21, IQ4_XS=23, BF16=30)",
            type);
    SSD_REQ(rows > 0 && cols > 0, SSD_ERR_SHAPE, "empty tensor %dx%d", rows, cols);
    int bs = type_block(type);
    SSD_REQ(cols % bs == 0, SSD_ERR_SHAPE, "cols %d not a multiple of block %d", cols, bs);
    int64_t nb = (int64_t)rows * (cols / bs);
    size_t qs_bytes, meta_bytes;
    if (type == SSD_TYPE_Q4_0) {
        qs_bytes = nb * 16;
        meta_bytes = nb * 2;
    } else if (type == SSD_TYPE_Q8_0) {
        qs_bytes = nb * 32;
        meta_bytes = nb * 2;
    } else if (type == SSD_TYPE_Q4_K) {
        qs_bytes = nb * 128;
        meta_bytes = nb * 16;
    } else if (type == SSD_TYPE_Q5_K) {
        qs_bytes = nb * 256;
        meta_bytes = nb * 16;
    } else if (type == SSD_TYPE_Q8_K) {
        qs_bytes = nb * 256;
        meta_bytes = nb * 64;
    } else if (type == SSD_TYPE_Q6_K) {
        qs_bytes = nb * 256;
        meta_bytes = nb * 32;
    } else if (is_lowbit(type)) {  // the reference's blocks as they are
        qs_bytes = (size_t)nb * type_block_bytes(type);
        meta_bytes = 0;
    } else {  // dense: F32, F16, BF16
        qs_bytes = (size_t)rows * cols * type_block_bytes(type);
        meta_bytes = 0;
    }
    WeightLayout L;
    L.qs_pad = (qs_bytes + 255) & ~(size_t)255;
    L.meta_bytes = meta_bytes;
    L.meta_pad = (meta_bytes + 255) & ~(size_t)255;
    // split-K scratch of the tensor-core matvec (quantized types): counters for up to
    // 2 * ceil(rows / 64) + 16 row tiles (a fused QKV or gate/up launch uses the first
    // weight's), partial rows for kI8MaxGrid CTAs
    L.fix = type_block(type) > 1 && !is_lowbit(type);
    const size_t n_counters = L.fix ? 2 * (((size_t)rows + 63) / 64) + 16 : 0;
    L.counter_bytes = (n_counters * 4 + 255) & ~(size_t)255;
    L.partial_bytes = L.fix ? (size_t)2 * kI8MaxGrid * 128 * 4 : 0;
    L.total = L.qs_pad + L.meta_pad + L.counter_bytes + L.partial_bytes + 256;
    *out = L;
    return SSD_OK;
}

void carve_weight(ssd_ctx* ctx, int type, int rows, int cols, const WeightLayout& L, uint8_t* p,
                  ssd_weight* w) {
    *w = ssd_weight();
    w->ctx = ctx;
    w->type = type;
    w->rows = rows;
    w->cols = cols;
    w->alloc_bytes = L.total;
    w->qs = p;
    w->meta = L.meta_bytes ? p + L.qs_pad : nullptr;
    if (L.fix) {
        uint8_t* f = p + L.qs_pad + L.meta_pad;
        w->fix_counter = reinterpret_cast<unsigned int*>(f);
        w->fix_partial = reinterpret_cast<float*>(f + L.counter_bytes);
    }
}

int upload_raw(ssd_weight* w, const void* raw_dev, cudaStream_t s) {
    const size_t bytes = ssd_row_bytes(w->type, w->cols) * (size_t)w->rows;
    if (type_block(w->type) == 1 || is_lowbit(w->type)) {  // dense / low-bit: the bytes as they are
        SSD_CK(cudaMemcpyAsync(w->qs, raw_dev, bytes, cudaMemcpyDeviceToDevice, s));
    } else {
        int64_t nb = (int64_t)w->rows * (w->cols / type_block(w->type));
        k_repack<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>((const uint8_t*)raw_dev, w->type,
                                                              nb, w->qs, w->meta);
        SSD_REQ(cudaGetLastError() == cudaSuccess, SSD_ERR_CUDA, "repack launch failed");
    }
    return SSD_OK;
}

int alloc_weight(ssd_ctx* ctx, int type, int rows, int cols, ssd_weight** out) {
    SSD_REQ(out != nullptr, SSD_ERR_ARG, "null out");
    WeightLayout L;
    SSD_TRY(weight_layout(type, rows, cols, &L));
    void* p = nullptr;
    if (cudaMalloc(&p, L.total) != cudaSuccess) {
        cudaGetLastError();
        set_error("weight allocation of %zu bytes failed", L.total);
        return SSD_ERR_NOMEM;
    }
    ssd_weight* w = new ssd_weight();
    carve_weight(ctx, type, rows, cols, L, (uint8_t*)p, w);
    w->base = p;
    if (L.fix && zero_device(ctx, w->fix_counter, L.counter_bytes) != SSD_OK) {
        cudaGetLastError();
        cudaFree(p);
        delete w;
        set_error("weight scratch initialisation failed");
        return SSD_ERR_CUDA;
    }
    *out = w;
    return SSD_OK;
}
}  // namespace ssd

extern "C" int ssd_weight_upload_device(ssd_ctx* ctx, const void* raw_dev, size_t bytes, int type,
                                        int rows, int cols, ssd_weight** out, void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(raw_dev != nullptr, SSD_ERR_ARG, "null raw pointer");
    size_t need = ssd_row_bytes(type, cols) * (size_t)rows;
    SSD_REQ(type_block(type) != 0, SSD_ERR_TYPE, "ggml type %d not supported", type);
    SSD_REQ(need != 0 && bytes == need, SSD_ERR_SHAPE,
            "got %zu bytes, %dx%d of type %d needs %zu", bytes, rows, cols, type, need);
    ssd_weight* w = nullptr;
    SSD_TRY(alloc_weight(ctx, type, rows, cols, &w));
    const int st = upload_raw(w, raw_dev, pick_stream(ctx, stream));
    if (st != SSD_OK) {
        ssd_weight_free(w);
        return st;
    }
    *out = w;
    return SSD_OK;
}

extern "C" int ssd_weight_upload(ssd_ctx* ctx, const void* host_raw, size_t bytes, int type,
                                 int rows, int cols, ssd_weight** out) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(host_raw != nullptr && out != nullptr, SSD_ERR_ARG, "null argument");
    size_t need = ssd_row_bytes(type, cols) * (size_t)rows;
    SSD_REQ(type_block(type) != 0, SSD_ERR_TYPE, "ggml type %d not supported", type);
    SSD_REQ(need != 0 && bytes == need, SSD_ERR_SHAPE,
            "got %zu bytes, %dx%d of type %d needs %zu", bytes, rows, cols, type, need);
    void* staging = nullptr;
    if (cudaMalloc(&staging, bytes) != cudaSuccess) {
        cudaGetLastError();
        set_error("staging allocation of %zu bytes failed", bytes);
        return SSD_ERR_NOMEM;
    }
    int st = SSD_OK;
    if (cudaMemcpyAsync(staging, host_raw, bytes, cudaMemcpyHostToDevice, ctx->stream) !=
        cudaSuccess) {
        set_error("upload copy failed: %s", cudaGetErrorString(cudaGetLastError()));
        st = SSD_ERR_CUDA;
    }
    if (st == SSD_OK) st = ssd_weight_upload_device(ctx, staging, bytes, type, rows, cols, out,
                                            (void*)ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(staging);
    return st;
}

extern "C" int ssd_weight_download(ssd_ctx* ctx, const ssd_weight* w, void* host_raw,
                                   size_t bytes) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(w && host_raw, SSD_ERR_ARG, "null argument");
    size_t need = ssd_row_bytes(w->type, w->cols) * (size_t)w->rows;
    SSD_REQ(bytes == need, SSD_ERR_SHAPE, "need %zu bytes, got %zu", need, bytes);
    if (type_block(w->type) == 1 || is_lowbit(w->type)) {
        SSD_CK(cudaMemcpyAsync(host_raw, w->qs, bytes, cudaMemcpyDeviceToHost, ctx->stream));
        SSD_CK(cudaStreamSynchronize(ctx->stream));
        return SSD_OK;
    }
    void* staging = nullptr;
    SSD_CK(cudaMalloc(&staging, bytes));
    int64_t nb = (int64_t)w->rows * (w->cols / type_block(w->type));
    k_unpack<<<(unsigned)((nb + 255) / 256), 256, 0, ctx->stream>>>(w->qs, w->meta, w->type, nb,
                                                                    (uint8_t*)staging);
    cudaError_t e = cudaMemcpyAsync(host_raw, staging, bytes, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(staging);
    SSD_CK(e);
    return SSD_OK;
}

extern "C" int ssd_weight_free(ssd_weight* w) {
    if (!w) return SSD_OK;
    if (w->base) {
        cudaSetDevice(w->ctx->device);
        cudaFree(w->base);
    }
    delete w;
    return SSD_OK;
}

extern "C" int ssd_weight_info(const ssd_weight* w, int* type, int* rows, int* cols,
                               size_t* raw_bytes) {
    SSD_REQ(w != nullptr, SSD_ERR_ARG, "null weight");
    if (type) *type = w->type;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (raw_bytes) *raw_bytes = ssd_row_bytes(w->type, w->cols) * (size_t)w->rows;
    return SSD_OK;
}

extern "C" int ssd_weight_synth(ssd_ctx* ctx, int type, uint64_t seed, uint32_t tensor_id,
                                float std_dev, int64_t total_cols, int row0, int rows, int col0,
                                int cols, ssd_weight** out, void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(type == SSD_TYPE_Q4_0 || type == SSD_TYPE_Q8_0 || type == SSD_TYPE_Q4_K, SSD_ERR_TYPE,
            "synthetic weights support Q4_0/Q8_0/Q4_K, not %d", type);
    int bs = type_block(type);
    SSD_REQ(col0 % bs == 0 && cols % bs == 0 && col0 + cols <= total_cols && row0 >= 0,
            SSD_ERR_SHAPE, "window not block aligned");
    ssd_weight* w = nullptr;
    SSD_TRY(alloc_weight(ctx, type, rows, cols, &w));
    int64_t nb = (int64_t)rows * (cols / bs);
    cudaStream_t s = pick_stream(ctx, stream);
    int threads = type == SSD_TYPE_Q4_K ? 64 : 128;
    k_synth_weight<<<(unsigned)((nb + threads - 1) / threads), threads, 0, s>>>(
        type, seed, tensor_id, std_dev, total_cols, row0, rows, col0, cols, w->qs, w->meta);
    if (cudaGetLastError() != cudaSuccess) {
        ssd_weight_free(w);
        set_error("synth launch failed");
        return SSD_ERR_CUDA;
    }
    *out = w;
    return SSD_OK;
}

extern "C" int ssd_synth_f32(ssd_ctx* ctx, uint64_t seed, uint32_t tensor_id, float mean,
                             float std_dev, int64_t total_cols, int row0, int rows, int col0,
                             int cols, float* out_dev, void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(out_dev && rows > 0 && cols > 0, SSD_ERR_ARG, "bad arguments");
    int64_t n = (int64_t)rows * cols;
    k_synth_f32<<<(unsigned)((n + 255) / 256), 256, 0, pick_stream(ctx, stream)>>>(
        seed, tensor_id, mean, std_dev, total_cols, row0, rows, col0, cols, out_dev);
    SSD_CK_LAUNCH();
    return SSD_OK;
}

extern "C" int ssd_quantize(ssd_ctx* ctx, const float* x_dev, int rows, int cols, int type,
                            void* raw_out_dev, void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(x_dev && raw_out_dev, SSD_ERR_ARG, "null pointer");
    SSD_REQ(type == SSD_TYPE_Q4_0 || type == SSD_TYPE_Q8_0 || type == SSD_TYPE_Q4_K, SSD_ERR_TYPE,
            "quantize supports Q4_0/Q8_0/Q4_K, not %d", type);
    int bs = type_block(type);
    SSD_REQ(rows > 0 && cols > 0 && cols % bs == 0, SSD_ERR_SHAPE, "cols %d not a multiple of %d",
            cols, bs);
    int64_t nb = (int64_t)rows * (cols / bs);
    k_quantize_raw<<<(unsigned)((nb + 127) / 128), 128, 0, pick_stream(ctx, stream)>>>(
        x_dev, type, nb, (uint8_t*)raw_out_dev);
    SSD_CK_LAUNCH();
    return SSD_OK;
}

extern "C" int ssd_dequantize(ssd_ctx* ctx, const ssd_weight* w, float* out_dev, void* stream) {
    SSD_TRY(check_ctx(ctx));
    SSD_REQ(w && out_dev, SSD_ERR_ARG, "null pointer");
    int64_t n = (int64_t)w->rows * w->cols;
    SSD_REQ(n % 8 == 0, SSD_ERR_SHAPE, "element count must be a multiple of 8");
    int64_t threads = n / 8;
    k_dequant<<<(unsigned)((threads + 255) / 256), 256, 0, pick_stream(ctx, stream)>>>(*w, out_dev);
    SSD_CK_LAUNCH();
    return SSD_OK;
}
