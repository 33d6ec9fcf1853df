// lmc_common.cuh - shared helpers for the CUDA side of liblmc_b200.so.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/lmc_cuda.h"

// Records a formatted message for lmc_last_error() and returns `code`.
extern "C" int lmc_set_error(int code, const char *fmt, ...);

#define LMC_CUDA_TRY(expr)                                                        \
    do {                                                                          \
        cudaError_t _e = (expr);                                                  \
        if (_e != cudaSuccess)                                                    \
            return lmc_set_error(LMC_ERR_CUDA, "%s: %s (%s:%d)", #expr,           \
                                 cudaGetErrorString(_e), __FILE__, __LINE__);     \
    } while (0)

// After a kernel launch: report launch-configuration errors.
#define LMC_LAUNCH_CHECK(name)                                                    \
    do {                                                                          \
        cudaError_t _e = cudaGetLastError();                                      \
        if (_e != cudaSuccess)                                                    \
            return lmc_set_error(LMC_ERR_CUDA, "%s launch: %s", name,             \
                                 cudaGetErrorString(_e));                         \
    } while (0)

static inline cudaStream_t lmc_stream(void *s) { return (cudaStream_t)s; }

static inline unsigned lmc_cdiv(size_t a, size_t b) { return (unsigned)((a + b - 1) / b); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum; `red` must hold blockDim.x/32 floats.  All threads get it.
__device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.0f;
    return warp_sum(t);
}

__device__ __forceinline__ float block_max(float v, float *red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : -INFINITY;
    return warp_max(t);
}

// Greedy-pick key (src/lmc.c:45-47: largest value, first index on ties):
// high word = the float's bits mapped to an order-preserving unsigned,
// low word = ~index, so the unsigned 64-bit maximum is the first maximum.
__device__ __forceinline__ unsigned long long lmc_argmax_key(float v, int idx) {
    const unsigned int f = __float_as_uint(v);
    const unsigned int o = (f & 0x80000000u) ? ~f : (f | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned int)idx);
}
__device__ __forceinline__ int lmc_key_index(unsigned long long k) { return (int)(0xFFFFFFFFu - (unsigned int)(k & 0xFFFFFFFFu)); }

// LMc activations (src/ops.c:20-29), same expression and operation order.
__device__ __forceinline__ float lmc_gelu_f(float x) { return x * (1.0f / (1.0f + expf(-1.702f * x))); }
__device__ __forceinline__ float lmc_silu_f(float x) { return x * (1.0f / (1.0f + expf(-x))); }

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL).  Kernels of a decode step are launched
// with the programmatic-serialization attribute, so kernel N+1 is scheduled
// while kernel N drains; every kernel calls pdl_launch_dependents() early and
// pdl_wait() before it touches memory written by earlier kernels.  Work that
// only reads weights (loads, L2 prefetch) is issued before pdl_wait() and so
// overlaps the previous kernel.  Every kernel calls pdl_wait(), so completion
// stays transitive along the chain.  Without the attribute both are no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

extern "C" int lmc_pdl_enabled(void);

template <typename... KArgs, typename... Args>
static inline cudaError_t lmc_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                     Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = lmc_pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

#define LMC_LAUNCH(name, kern, grid, block, smem, stream, ...)                                        \
    do {                                                                                              \
        cudaError_t _e = lmc_launch(kern, dim3(grid), dim3(block), (size_t)(smem), stream, __VA_ARGS__); \
        if (_e != cudaSuccess) return lmc_set_error(LMC_ERR_CUDA, "%s launch: %s", name, cudaGetErrorString(_e)); \
    } while (0)
