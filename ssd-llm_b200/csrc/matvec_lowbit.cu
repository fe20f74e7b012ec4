// matvec_lowbit.cu — matvec over the reference's low-bit formats (Q3_K, Q2_K, IQ4_NL, IQ4_XS,
// IQ3_XXS, IQ3_S, IQ2_XXS, IQ2_XS; matvec_*_cpu, src/metal/compute.rs:793-1075, 1964-2240),
// read in their own block layouts.
//
// One warp per output row (rows strided over the grid's warps): lane l decodes the 32-weight
// groups l, l + 32, ... of the row (lowbit_group: the reference's element values), dots
// each with its 32 x values (float4 loads, L1-resident across the CTA's rows), and the warp
// sums the lane partials (butterfly, then lane 0 stores; + base with EPI_RESID). The 32
// lanes of a warp read 4 consecutive 256-weight blocks per group step, so a warp's loads
// cover contiguous block bytes. These formats carry 2.1-4.6 bits per weight; the decode
// (grid lookups from L1, per-element sign and scale products) sets the rate, not HBM.
#include "lowbit.cuh"
#include "matvec.cuh"
#include "matvec_dev.cuh"

namespace ssd {

constexpr int kLbThreads = 256;

template <int T, int EPI>
__global__ void __launch_bounds__(kLbThreads) k_matvec_lowbit(const MvArgs a) {
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (kLbThreads / 32);
    const int bs = T == SSD_TYPE_IQ4_NL ? 32 : 256;
    const int gpb = bs / 32;  // groups per block
    const size_t bb = (size_t)type_block_bytes(T);
    const int ngroups = a.cols / 32;
    const size_t row_bytes = (size_t)(a.cols / bs) * bb;
    for (int row = blockIdx.x * (kLbThreads / 32) + (threadIdx.x >> 5); row < a.rows; row += warps) {
        const uint8_t* r = a.qs[0] + (size_t)row * row_bytes;
        float acc = 0.0f;
        for (int g = lane; g < ngroups; g += 32) {
            float w[32];
            lowbit_group<T>(r + (size_t)(g / gpb) * bb, g % gpb, w);
            const float4* x4 = reinterpret_cast<const float4*>(a.x + (size_t)g * 32);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float4 xv = __ldg(x4 + i);
                acc = fmaf(w[4 * i], xv.x, acc);
                acc = fmaf(w[4 * i + 1], xv.y, acc);
                acc = fmaf(w[4 * i + 2], xv.z, acc);
                acc = fmaf(w[4 * i + 3], xv.w, acc);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) a.y[row] = EPI == EPI_RESID ? __fadd_rn(a.base[row], acc) : acc;
    }
}

template <int T>
static int launch_lb(ssd_ctx* ctx, int epi, const MvArgs& a, cudaStream_t s, bool pdl) {
    const int want = (a.rows + kLbThreads / 32 - 1) / (kLbThreads / 32);
    const int cap = ctx->num_sms * 8;
    const int grid = want < cap ? want : cap;
    if (epi == EPI_RESID)
        SSD_CK(launch_pdl(k_matvec_lowbit<T, EPI_RESID>, dim3(grid), dim3(kLbThreads), 0, s, pdl, a));
    else
        SSD_CK(launch_pdl(k_matvec_lowbit<T, EPI_STORE>, dim3(grid), dim3(kLbThreads), 0, s, pdl, a));
    return SSD_OK;
}

int launch_matvec_lowbit(ssd_ctx* ctx, int type, int epi, const MvArgs& a, cudaStream_t s,
                         bool pdl) {
    SSD_REQ(a.rows > 0 && a.cols > 0 && a.cols % type_block(type) == 0, SSD_ERR_SHAPE,
            "cols %d not a multiple of the %d-weight block", a.cols, type_block(type));
    SSD_REQ(a.x && a.y && ((uintptr_t)a.x & 15) == 0, SSD_ERR_ARG,
            "x and y must be non-null, x 16-byte aligned");
    SSD_REQ(((epi == EPI_STORE) || (epi == EPI_RESID && a.base)) && a.map == MAP_PLAIN &&
                !a.x_add && !a.norm_w && a.ar_in_n == 0,
            SSD_ERR_ARG, "low-bit formats: plain or residual matvec only");
    switch (type) {
        case SSD_TYPE_Q3_K: return launch_lb<SSD_TYPE_Q3_K>(ctx, epi, a, s, pdl);
        case SSD_TYPE_Q2_K: return launch_lb<SSD_TYPE_Q2_K>(ctx, epi, a, s, pdl);
        case SSD_TYPE_IQ4_NL: return launch_lb<SSD_TYPE_IQ4_NL>(ctx, epi, a, s, pdl);
        case SSD_TYPE_IQ4_XS: return launch_lb<SSD_TYPE_IQ4_XS>(ctx, epi, a, s, pdl);
        case SSD_TYPE_IQ3_XXS: return launch_lb<SSD_TYPE_IQ3_XXS>(ctx, epi, a, s, pdl);
        case SSD_TYPE_IQ3_S: return launch_lb<SSD_TYPE_IQ3_S>(ctx, epi, a, s, pdl);
        case SSD_TYPE_IQ2_XXS: return launch_lb<SSD_TYPE_IQ2_XXS>(ctx, epi, a, s, pdl);
        case SSD_TYPE_IQ2_XS: return launch_lb<SSD_TYPE_IQ2_XS>(ctx, epi, a, s, pdl);
        default: set_error("not a low-bit type: %d", type); return SSD_ERR_TYPE;
    }
}

}  // namespace ssd
