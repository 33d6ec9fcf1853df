// gemv_generic.cu - K2 (generic): fused dequant + matrix-vector product on
// CUDA cores for every block format and any shape (LMc matmul_vec,
// src/ops.c:69-97, applied to the dequant_* result).
//
// One warp per output row.  The row is the flat element range [m*K, m*K+K)
// of the block stream; the warp walks it in 8-weight groups aligned to the
// flat index (a group never crosses a block), decodes each group with the
// bit-exact decoders and accumulates in fp32.  Handles rows that start or end
// inside a block (K not a multiple of the block size), as LMc does.  This is
// the path for formats and shapes without a tensor-core kernel.
#include "lmc_blocks.cuh"
#include "lmc_common.cuh"

#include <algorithm>

#define GEN_WARPS 8
#define GEN_MAXB 8

template <int T>
__global__ void __launch_bounds__(GEN_WARPS * 32)
k_gemv_generic(const uint8_t *__restrict__ W, int M, int K, const float *__restrict__ x, int ldx,
               const float *__restrict__ bias, float *__restrict__ y, int ldy, int nb, int epi) {
    using F = lmcq::Fmt<T>;
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int m = blockIdx.x * GEN_WARPS + (threadIdx.x >> 5);
    if (m >= M) return;
    const size_t r0 = (size_t)m * K, r1 = r0 + K;
    const size_t g0 = r0 >> 3, g1 = (r1 + 7) >> 3;
    float acc[GEN_MAXB];
#pragma unroll
    for (int b = 0; b < GEN_MAXB; b++) acc[b] = 0.0f;
    for (size_t g = g0 + lane; g < g1; g += 32) {
        const size_t e = g << 3;
        float w[8];
        lmcq::decode8<T>(W + (e / F::BE) * F::BB, (int)(e % F::BE), w);
        const bool full = e >= r0 && e + 8 <= r1;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const long long k = (long long)(e + i) - (long long)r0;
            if (full || (k >= 0 && k < K)) {
#pragma unroll
                for (int b = 0; b < GEN_MAXB; b++)
                    if (b < nb) acc[b] = fmaf(w[i], __ldg(x + (size_t)b * ldx + k), acc[b]);
            }
        }
    }
#pragma unroll
    for (int b = 0; b < GEN_MAXB; b++) {
        if (b >= nb) break;
        float v = warp_sum(acc[b]);
        if (lane == 0) {
            if (bias) v += bias[m];
            if (epi & LMC_EPI_GELU) v = lmc_gelu_f(v);
            float *o = y + (size_t)b * ldy + m;
            *o = (epi & LMC_EPI_ACCUM) ? *o + v : v;
        }
    }
}

// Rows made of whole 8-weight groups (K % 8 == 0) with 16-byte aligned
// activation rows: the batch width is a template parameter (no per-weight
// predicates) and each group's 8 activations come as two float4 loads.
template <int T, int NB>
__global__ void __launch_bounds__(GEN_WARPS * 32)
k_gemv_generic_g8(const uint8_t *__restrict__ W, int M, int K, const float *__restrict__ x, int ldx,
                  const float *__restrict__ bias, float *__restrict__ y, int ldy, int nb, int epi) {
    using F = lmcq::Fmt<T>;
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int m = blockIdx.x * GEN_WARPS + (threadIdx.x >> 5);
    if (m >= M) return;
    const int ng = K >> 3;
    const size_t g0 = (size_t)m * ng;
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b] = 0.0f;
    for (int gi = lane; gi < ng; gi += 32) {
        const size_t e = (g0 + gi) << 3;
        float w[8];
        lmcq::decode8<T>(W + (e / F::BE) * F::BB, (int)(e % F::BE), w);
        const float *xk = x + (gi << 3);
#pragma unroll
        for (int b = 0; b < NB; b++) {
            if (b < nb) {  // uniform across the warp
                const float4 u = __ldg(reinterpret_cast<const float4 *>(xk + (size_t)b * ldx));
                const float4 v = __ldg(reinterpret_cast<const float4 *>(xk + (size_t)b * ldx + 4));
                float a = acc[b];
                a = fmaf(w[0], u.x, a);
                a = fmaf(w[1], u.y, a);
                a = fmaf(w[2], u.z, a);
                a = fmaf(w[3], u.w, a);
                a = fmaf(w[4], v.x, a);
                a = fmaf(w[5], v.y, a);
                a = fmaf(w[6], v.z, a);
                a = fmaf(w[7], v.w, a);
                acc[b] = a;
            }
        }
    }
#pragma unroll
    for (int b = 0; b < NB; b++) {
        if (b >= nb) break;
        float v = warp_sum(acc[b]);
        if (lane == 0) {
            if (bias) v += bias[m];
            if (epi & LMC_EPI_GELU) v = lmc_gelu_f(v);
            float *o = y + (size_t)b * ldy + m;
            *o = (epi & LMC_EPI_ACCUM) ? *o + v : v;
        }
    }
}

extern "C" int lmc_gemv_generic_launch(uint32_t type, const void *d_blocks, int M, int K, const float *d_x,
                                       int ldx, const float *d_bias, float *d_y, int ldy, int batch, int epi,
                                       cudaStream_t s) {
    const unsigned grid = lmc_cdiv((size_t)M, GEN_WARPS);
    const bool g8 = K % 8 == 0 && ldx % 4 == 0 && ((uintptr_t)d_x & 15) == 0;
    for (int b0 = 0; b0 < batch; b0 += GEN_MAXB) {
        const int nb = std::min(GEN_MAXB, batch - b0);
        const float *xb = d_x + (size_t)b0 * ldx;
        float *yb = d_y + (size_t)b0 * ldy;
        if (g8) {
            switch (type) {
#define CASE(T)                                                                                                  \
    case T:                                                                                                      \
        if (nb == 1)                                                                                             \
            LMC_LAUNCH("gemv_generic", (k_gemv_generic_g8<T, 1>), grid, GEN_WARPS * 32, 0, s,                    \
                       (const uint8_t *)d_blocks, M, K, xb, ldx, d_bias, yb, ldy, nb, epi);                      \
        else if (nb == 2)                                                                                        \
            LMC_LAUNCH("gemv_generic", (k_gemv_generic_g8<T, 2>), grid, GEN_WARPS * 32, 0, s,                    \
                       (const uint8_t *)d_blocks, M, K, xb, ldx, d_bias, yb, ldy, nb, epi);                      \
        else if (nb <= 4)                                                                                        \
            LMC_LAUNCH("gemv_generic", (k_gemv_generic_g8<T, 4>), grid, GEN_WARPS * 32, 0, s,                    \
                       (const uint8_t *)d_blocks, M, K, xb, ldx, d_bias, yb, ldy, nb, epi);                      \
        else                                                                                                     \
            LMC_LAUNCH("gemv_generic", (k_gemv_generic_g8<T, 8>), grid, GEN_WARPS * 32, 0, s,                    \
                       (const uint8_t *)d_blocks, M, K, xb, ldx, d_bias, yb, ldy, nb, epi);                      \
        break;
                LMC_FOR_EACH_TYPE(CASE)
#undef CASE
            default:
                return lmc_set_error(LMC_ERR_UNSUPPORTED, "matmul: type %u", type);
            }
            continue;
        }
        switch (type) {
#define CASE(T)                                                                                       \
    case T:                                                                                           \
        LMC_LAUNCH("gemv_generic", k_gemv_generic<T>, grid, GEN_WARPS * 32, 0, s, (const uint8_t *)d_blocks, M, K, \
                   xb, ldx, d_bias, yb, ldy, nb, epi);                                                \
        break;
            LMC_FOR_EACH_TYPE(CASE)
#undef CASE
        default:
            return lmc_set_error(LMC_ERR_UNSUPPORTED, "matmul: type %u", type);
        }
    }
    return LMC_OK;
}
