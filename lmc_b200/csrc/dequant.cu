// dequant.cu - K1: bit-exact block dequantization (LMc src/quant.c:178-521).
//
// One thread decodes 8 consecutive weights and writes them as two float4
// stores, so a warp writes 1 KB contiguous; the kernel is bound by the fp32
// writes (4 bytes per weight against 0.33-1.06 bytes read).  Grid-stride
// loop over 8-weight groups, launched at a multiple of the SM count.
#include "lmc_blocks.cuh"
#include "lmc_common.cuh"
#include "lmc_internal.h"

#include <algorithm>

template <int T>
__global__ void __launch_bounds__(256) k_dequant(const uint8_t *__restrict__ src, float *__restrict__ dst,
                                                 size_t n_groups) {
    using F = lmcq::Fmt<T>;
    constexpr int GPB = F::BE / 8;  // 8-weight groups per block
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < n_groups;
         g += (size_t)gridDim.x * blockDim.x) {
        const size_t blk = g / GPB;
        const int j = (int)(g % GPB) * 8;
        float y[8];
        lmcq::decode8<T>(src + blk * F::BB, j, y);
        float4 *o = reinterpret_cast<float4 *>(dst + g * 8);
        o[0] = make_float4(y[0], y[1], y[2], y[3]);
        o[1] = make_float4(y[4], y[5], y[6], y[7]);
    }
}

// Scalar tail for F32/F16 tensors whose length is not a multiple of 8.
__global__ void k_dequant_tail(uint32_t type, const uint8_t *__restrict__ src, float *__restrict__ dst,
                               size_t first, size_t n) {
    size_t i = first + blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (type == LMC_TYPE_F32) dst[i] = __ldg(reinterpret_cast<const float *>(src) + i);
    else dst[i] = lmcq::h2f(lmcq::ld16(src + 2 * i));
}

static int g_sm_count = 0;
extern "C" int lmc_sm_count(void) {
    if (!g_sm_count) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (g_sm_count <= 0) g_sm_count = 148;
    }
    return g_sm_count;
}

extern "C" int lmc_dequant(uint32_t type, const void *d_blocks, size_t n, float *d_out, void *stream) {
    int be, bb;
    if (lmc_block_geometry(type, &be, &bb)) return lmc_set_error(LMC_ERR_UNSUPPORTED, "dequant: type %u", type);
    if (!d_blocks || !d_out) return lmc_set_error(LMC_ERR_INVALID, "dequant: null pointer");
    if (n % (size_t)be) return lmc_set_error(LMC_ERR_INVALID, "dequant: %zu not a multiple of %d", n, be);
    if (((uintptr_t)d_out & 15) || ((uintptr_t)d_blocks & 1))
        return lmc_set_error(LMC_ERR_INVALID, "dequant: output must be 16-byte aligned, blocks 2-byte aligned");
    if ((type == LMC_TYPE_F32) && ((uintptr_t)d_blocks & 15))
        return lmc_set_error(LMC_ERR_INVALID, "dequant: F32 input must be 16-byte aligned");
    if (n == 0) return LMC_OK;
    cudaStream_t s = lmc_stream(stream);
    const size_t groups = n / 8;  // block formats: n is a multiple of 32
    const unsigned grid = (unsigned)std::min<size_t>(lmc_cdiv(groups, 256), (size_t)lmc_sm_count() * 8);
    switch (type) {
#define CASE(T)                                                                                   \
    case T:                                                                                       \
        if (groups) k_dequant<T><<<grid ? grid : 1, 256, 0, s>>>((const uint8_t *)d_blocks, d_out, groups); \
        break;
        LMC_FOR_EACH_TYPE(CASE)
#undef CASE
    default:
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "dequant: type %u", type);
    }
    LMC_LAUNCH_CHECK("dequant");
    if ((type == LMC_TYPE_F32 || type == LMC_TYPE_F16) && groups * 8 < n) {
        k_dequant_tail<<<1, 32, 0, s>>>(type, (const uint8_t *)d_blocks, d_out, groups * 8, n);
        LMC_LAUNCH_CHECK("dequant tail");
    }
    return LMC_OK;
}
