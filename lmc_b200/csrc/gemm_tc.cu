// gemm_tc.cu - K3: batched dequant-GEMM on the 5th-generation tensor cores.
//   Y[n][m] = epilogue( sum_k X[n][k] * W[m][k] ),  n < N (tokens / sequences),
// W a GGUF block-quantized matrix (any of the 15 formats), for batch widths
// above the GEMV's 8 rows (prefill, many concurrent sequences).  Replaces LMc
// matmul_vec (src/ops.c:69-97) applied once per token row, over dequant_*
// (src/quant.c).
//
// Per CTA: one 128-row tile of W x one BN-token tile of X (BN = 64/128/256),
// K in 64-wide k-blocks through two shared-memory stages.
//   * A (W): the CTA's 128 threads decode their row's 64 weights with the
//     bit-exact LMc decoders (lmc_blocks.cuh), scale by a per-tensor power of
//     two (so every weight is a normal fp16) and store fp16 into the
//     128-byte-swizzled K-major layout the tensor core reads.
//   * B (X): fp16 hi and lo parts of the (prologue-transformed, per-row
//     power-of-two scaled) activations, prepared once per launch by
//     k_gemm_prep_x; hi + lo carries x to ~22 bits.
//   * One thread issues tcgen05.mma (kind::f16, M=128, N=BN, K=16) for hi and
//     lo into an fp32 accumulator in tensor memory and commits to the stage's
//     mbarrier; the threads decode the next k-block meanwhile.
//   * Split-K over a cluster of CL CTAs (same output tile): partial
//     accumulators are added into the leader's shared memory through
//     distributed shared memory; the leader applies the epilogue (per-row /
//     per-tensor scales, bias, GELU, residual, greedy-pick key).
// Precision: the fp16 weight has a relative rounding error <= 2^-11, the
// hi+lo activation ~2^-22, accumulation fp32: relative error of Y ~3e-4 rms.
#include <cuda_fp16.h>

#include "lmc_blocks.cuh"
#include "lmc_common.cuh"
#include "lmc_internal.h"

#include <algorithm>
#include <math.h>
#include <string.h>

namespace {

constexpr int BM = 128, BK = 64, GTHR = 128;

struct GArgs {
    const uint8_t *w;     // raw blocks
    int M, K, N;
    const __half *xh, *xl;  // [N][K]
    const float *xinv;      // [N] inverse activation scales
    float wscale, winv;     // weight prescale and its inverse (powers of two)
    const float *bias;
    float *y;
    int ldy, epi;
    unsigned long long *keys;
    int BN, MT, CL, nkb;
};

__device__ int g_gemm_timeout;

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(65536u)
        : "memory");
    return ok != 0;
}
// bounded: about one second, then the flag is set and the caller goes on
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t t = 0; t < (1u << 14); t++)
        if (bar_try(bar, parity)) return true;
    atomicExch(&g_gemm_timeout, 1);
    return false;
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (start address in 16-byte units in bits 0-13, leading
// offset 1, stride offset 64 at bit 32, descriptor version 1 at bit 46,
// layout type 2 = 128-byte swizzle at bit 61).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator (bit 4), A and B fp16,
// both K-major, N/8 at bit 17, M/16 at bit 24.
__device__ __forceinline__ uint32_t idesc(int n) { return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24); }

__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem),
        "l"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ uint32_t ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t clusterid() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cl_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cl_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
__device__ __forceinline__ void red_remote(uint32_t local, uint32_t rank, float v) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    asm volatile("red.shared::cluster.add.f32 [%0], %1;" ::"r"(r), "f"(v) : "memory");
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ void epi_store(const GArgs &a, int n, int m, float v) {
    if (a.bias) v += a.bias[m];
    if (a.epi & LMC_EPI_GELU) v = lmc_gelu_f(v);
    float *o = a.y + (size_t)n * a.ldy + m;
    *o = (a.epi & LMC_EPI_ACCUM) ? *o + v : v;
    if (a.keys) atomicMax(a.keys + n, lmc_argmax_key(v, m));
}

// smem: [stage 0: A 16 KB | Bh BN*128 | Bl BN*128] [stage 1: same] [2 mbarriers] [tmem slot]
template <int T>
__global__ void __launch_bounds__(GTHR, 1) k_gemm_tc(GArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    constexpr int BE = lmcq::Fmt<T>::BE, BB = lmcq::Fmt<T>::BB;
    const int BN = a.BN, stage_bytes = BM * 128 + 2 * BN * 128;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 2 * stage_bytes);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int rank = a.CL > 1 ? (int)ctarank() : 0;
    const int tile = a.CL > 1 ? (int)clusterid() : (int)blockIdx.x;
    const int m0 = (tile % a.MT) * BM, n0 = (tile / a.MT) * BN;
    const int kb0 = (int)((long long)rank * a.nkb / a.CL), kb1 = (int)((long long)(rank + 1) * a.nkb / a.CL);
    const int nit = kb1 - kb0;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tslot)), "r"(BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&bars[0])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&bars[1])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_launch_dependents();
    pdl_wait();  // X (prepared by the previous kernel), bias and Y are ready
    const uint32_t id = idesc(BN);
    const int m = m0 + tid;
    bool ok = true;
    for (int it = 0; it < nit; it++) {
        const int s = it & 1, kb = kb0 + it;
        uint8_t *A = smem + s * stage_bytes, *Bh = A + BM * 128, *Bl = Bh + BN * 128;
        if (it >= 2 && ok) ok = bar_wait(su32(&bars[s]), (uint32_t)(((it - 2) >> 1) & 1));  // stage free
        // A: this thread's row, 64 weights -> 8 swizzled 16-byte chunks
#pragma unroll 2
        for (int c = 0; c < 8; c++) {
            float v[8];
            if (m < a.M) {
                const size_t e = (size_t)m * a.K + (size_t)kb * BK + 8 * c;
                lmcq::decode8<T>(a.w + (e / BE) * BB, (int)(e % BE), v);
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = 0.0f;
            }
            uint4 q;
            q.x = pack_h2(v[0] * a.wscale, v[1] * a.wscale);
            q.y = pack_h2(v[2] * a.wscale, v[3] * a.wscale);
            q.z = pack_h2(v[4] * a.wscale, v[5] * a.wscale);
            q.w = pack_h2(v[6] * a.wscale, v[7] * a.wscale);
            *reinterpret_cast<uint4 *>(A + tid * 128 + ((c ^ (tid & 7)) << 4)) = q;
        }
        // B: BN token rows x 8 chunks, hi and lo
        for (int i = tid; i < BN * 8; i += GTHR) {
            const int r = i >> 3, c = i & 7, n = n0 + r;
            uint4 h = make_uint4(0u, 0u, 0u, 0u), l = h;
            if (n < a.N) {
                const size_t off = (size_t)n * a.K + (size_t)kb * BK + 8 * c;
                h = __ldg(reinterpret_cast<const uint4 *>(a.xh + off));
                l = __ldg(reinterpret_cast<const uint4 *>(a.xl + off));
            }
            const int o = r * 128 + ((c ^ (r & 7)) << 4);
            *reinterpret_cast<uint4 *>(Bh + o) = h;
            *reinterpret_cast<uint4 *>(Bl + o) = l;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int j = 0; j < BK / 16; j++) {  // 16 fp16 = 32 bytes per K step
                const uint64_t ad = sdesc(su32(A) + 32 * j);
                mma_f16(tmem, ad, sdesc(su32(Bh) + 32 * j), id, (it > 0 || j > 0) ? 1u : 0u);
                mma_f16(tmem, ad, sdesc(su32(Bl) + 32 * j), id, 1u);
            }
            mma_commit(su32(&bars[s]));
        }
    }
    if (nit > 0 && ok) ok = bar_wait(su32(&bars[(nit - 1) & 1]), (uint32_t)(((nit - 1) >> 1) & 1));
    tc_fence_after();
    const float wi = a.winv;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    if (a.CL == 1) {
        for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
            if (nit > 0) tmem_ld16(trow + c0, v);
            else
#pragma unroll
                for (int i = 0; i < 16; i++) v[i] = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const int n = n0 + c0 + i;
                if (n < a.N && m < a.M) epi_store(a, n, m, v[i] * (wi * a.xinv[n]));
            }
        }
    } else {
        // leader tile [BN][128] fp32 over the (now idle) stage memory
        float *red = reinterpret_cast<float *>(smem);
        if (rank == 0)
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float v[16];
                if (nit > 0) tmem_ld16(trow + c0, v);
                else
#pragma unroll
                    for (int i = 0; i < 16; i++) v[i] = 0.0f;
#pragma unroll
                for (int i = 0; i < 16; i++) red[(c0 + i) * BM + tid] = v[i];
            }
        cl_arrive();
        cl_wait();  // the leader's tile holds its partial
        if (rank != 0 && nit > 0)
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float v[16];
                tmem_ld16(trow + c0, v);
#pragma unroll
                for (int i = 0; i < 16; i++) red_remote(su32(&red[(c0 + i) * BM + tid]), 0u, v[i]);
            }
        cl_arrive();
        cl_wait();  // every partial added
        if (rank == 0)
            for (int c = 0; c < BN; c++) {
                const int n = n0 + c;
                if (n < a.N && m < a.M) epi_store(a, n, m, red[c * BM + tid] * (wi * a.xinv[n]));
            }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
}

// Activation prep: one CTA per token row n.  v = prologue(x[n]) (as the
// GEMV), scale 2^(14-e) with max|v| < 2^e, hi = fp16(v s), lo = fp16(v s - hi).
__global__ void __launch_bounds__(256) k_gemm_prep_x(const float *__restrict__ x, int ldx, int K, int pro,
                                                     const float *__restrict__ pw, const float *__restrict__ pb,
                                                     const float *__restrict__ x2, float eps, __half *xh, __half *xl,
                                                     float *xinv) {
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const int n = blockIdx.x, tid = threadIdx.x;
    const float *xr = x + (size_t)n * ldx;
    float mu = 0.0f, rs = 1.0f;
    if (pro == LMC_PRO_LAYERNORM || pro == LMC_PRO_RMSNORM) {
        float s1 = 0.0f;
        for (int k = tid; k < K; k += blockDim.x) s1 += pro == LMC_PRO_RMSNORM ? xr[k] * xr[k] : xr[k];
        s1 = block_sum(s1, red);
        if (pro == LMC_PRO_RMSNORM) {
            rs = 1.0f / sqrtf(s1 / (float)K + eps);
        } else {  // two-pass variance, as src/ops.c:52-54
            mu = s1 / (float)K;
            float s2 = 0.0f;
            for (int k = tid; k < K; k += blockDim.x) s2 += (xr[k] - mu) * (xr[k] - mu);
            s2 = block_sum(s2, red);
            rs = 1.0f / sqrtf(s2 / (float)K + 1e-5f);
        }
    }
    auto val = [&](int k) -> float {
        const float v = xr[k];
        switch (pro) {
        case LMC_PRO_LAYERNORM: return (v - mu) * rs * pw[k] + pb[k];
        case LMC_PRO_RMSNORM: return pw[k] * rs * v;
        case LMC_PRO_SWIGLU: return lmc_silu_f(v) * x2[(size_t)n * ldx + k];
        default: return v;
        }
    };
    float mx = 0.0f;
    for (int k = tid; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(val(k)));
    mx = block_max(mx, red);
    const int e = max((int)((__float_as_uint(mx) >> 23) & 0xFF) - 126, -100);
    const float s = mx > 0.0f ? __uint_as_float((uint32_t)(127 + 14 - e) << 23) : 1.0f;
    if (tid == 0) xinv[n] = mx > 0.0f ? __uint_as_float((uint32_t)(127 - 14 + e) << 23) : 0.0f;
    for (int k = tid; k < K; k += blockDim.x) {
        const float v = val(k) * s;
        const __half h = __float2half_rn(v);
        xh[(size_t)n * K + k] = h;
        xl[(size_t)n * K + k] = __float2half_rn(v - __half2float(h));
    }
}

// max |w| over a tensor (bit pattern of a non-negative float, atomicMax)
template <int T>
__global__ void k_absmax(const uint8_t *__restrict__ w, size_t n_groups, unsigned int *out) {
    constexpr int BE = lmcq::Fmt<T>::BE, BB = lmcq::Fmt<T>::BB;
    float mx = 0.0f;
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < n_groups; g += (size_t)gridDim.x * blockDim.x) {
        const size_t e = g * 8;
        float v[8];
        lmcq::decode8<T>(w + (e / BE) * BB, (int)(e % BE), v);
#pragma unroll
        for (int i = 0; i < 8; i++) mx = fmaxf(mx, fabsf(v[i]));  // NaN weights are ignored
    }
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(mx));
}

}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static __half *g_xh = NULL, *g_xl = NULL;
static float *g_xinv = NULL;
static size_t g_x_cap = 0;  // elements of xh / xl
static int g_xinv_cap = 0;

extern "C" int lmc_gemm_reserve(int N, int K, cudaStream_t s) {
    const size_t need = (size_t)N * K;
    if (need <= g_x_cap && N <= g_xinv_cap) return LMC_OK;
    cudaStreamCaptureStatus cs;
    if (cudaStreamIsCapturing(s, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
        return lmc_set_error(LMC_ERR_INVALID, "gemm: workspace must be reserved before stream capture");
    if (g_xh) cudaFree(g_xh);
    if (g_xl) cudaFree(g_xl);
    if (g_xinv) cudaFree(g_xinv);
    g_xh = g_xl = NULL;
    g_xinv = NULL;
    g_x_cap = 0;
    g_xinv_cap = 0;
    LMC_CUDA_TRY(cudaMalloc(&g_xh, need * sizeof(__half)));
    LMC_CUDA_TRY(cudaMalloc(&g_xl, need * sizeof(__half)));
    LMC_CUDA_TRY(cudaMalloc(&g_xinv, (size_t)N * sizeof(float)));
    g_x_cap = need;
    g_xinv_cap = N;
    return LMC_OK;
}

extern "C" int lmc_gemm_status(void) {
    int v = 0;
    LMC_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_gemm_timeout, sizeof(int)));
    if (!v) return LMC_OK;
    const int zero = 0;
    LMC_CUDA_TRY(cudaMemcpyToSymbol(g_gemm_timeout, &zero, sizeof(int)));
    return LMC_ERR_TIMEOUT;
}

// Power-of-two prescale for a tensor's fp16 weights: 2^(14-e), max|w| < 2^e.
extern "C" int lmc_gemm_prepare(lmc_qtensor *t) {
    t->gemm_wscale = 0.0f;
    if (t->cols % BK) return LMC_OK;
    unsigned int *d = NULL;
    LMC_CUDA_TRY(cudaMalloc(&d, sizeof(unsigned int)));
    cudaError_t e = cudaMemset(d, 0, sizeof(unsigned int));
    const size_t groups = (size_t)t->rows * t->cols / 8;
    const int grid = (int)std::min<size_t>((groups + 255) / 256, 4096);
    switch (t->type) {
#define LMC_ABSMAX_CASE(TY) \
    case TY: k_absmax<TY><<<grid, 256>>>((const uint8_t *)t->blocks, groups, d); break;
        LMC_FOR_EACH_TYPE(LMC_ABSMAX_CASE)
#undef LMC_ABSMAX_CASE
    default: break;
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    unsigned int bits = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&bits, d, sizeof(bits), cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (e != cudaSuccess) return lmc_set_error(LMC_ERR_CUDA, "gemm prepare: %s", cudaGetErrorString(e));
    float mx;
    memcpy(&mx, &bits, sizeof(mx));
    int ex = 0;
    if (mx > 0.0f && isfinite(mx)) frexpf(mx, &ex);
    ex = std::max(-100, std::min(ex, 100));
    t->gemm_wscale = ldexpf(1.0f, 14 - ex);
    return LMC_OK;
}

static int clusters_for(int cl, size_t smem, const void *fn) {
    if (cl == 1) return lmc_sm_count();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl);
    cfg.blockDim = dim3(GTHR);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cl;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) n = 0;
    (void)cudaGetLastError();
    return n;
}

extern "C" int lmc_gemm_launch(const lmc_qtensor *t, const float *d_x, int ldx, const float *d_bias, float *d_y,
                               int ldy, int N, int epi, const lmc_gemv_extra *ex, cudaStream_t s) {
    if (t->cols % BK || t->gemm_wscale <= 0.0f)
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "gemm: needs cols %% 64 == 0 and a prepared tensor");
    const int M = t->rows, K = t->cols;
    int rc = lmc_gemm_reserve(N, K, s);
    if (rc) return rc;
    // activations -> fp16 hi/lo (with the prologue op)
    LMC_LAUNCH("gemm prep", k_gemm_prep_x, N, 256, 0, s, d_x, ldx, K, ex ? ex->pro : LMC_PRO_NONE,
               ex ? ex->w : (const float *)NULL, ex ? ex->b : (const float *)NULL, ex ? ex->x2 : (const float *)NULL,
               ex ? ex->eps : 0.0f, g_xh, g_xl, g_xinv);
    GArgs a;
    a.w = (const uint8_t *)t->blocks;
    a.M = M;
    a.K = K;
    a.N = N;
    a.xh = g_xh;
    a.xl = g_xl;
    a.xinv = g_xinv;
    a.wscale = t->gemm_wscale;
    a.winv = 1.0f / t->gemm_wscale;
    a.bias = d_bias;
    a.y = d_y;
    a.ldy = ldy;
    a.epi = epi;
    a.keys = ex ? ex->keys : NULL;
    a.BN = N <= 64 ? 64 : N <= 128 ? 128 : 256;
    a.MT = (M + BM - 1) / BM;
    a.nkb = K / BK;
    const int NTL = (N + a.BN - 1) / a.BN, tiles = a.MT * NTL;
    const size_t smem = 2 * (size_t)(BM * 128 + 2 * a.BN * 128) + 64 + 1024;
    const void *fn = NULL;
    switch (t->type) {
#define LMC_GEMM_FN(TY) \
    case TY: fn = (const void *)k_gemm_tc<TY>; break;
        LMC_FOR_EACH_TYPE(LMC_GEMM_FN)
#undef LMC_GEMM_FN
    default: return lmc_set_error(LMC_ERR_UNSUPPORTED, "gemm: type %u", t->type);
    }
    LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    // split K over a cluster until the tiles cover the SMs (each CTA keeps >= 2 k-blocks)
    int cl = 1;
    while (cl < 8 && tiles * cl * 2 <= lmc_sm_count() && a.nkb >= 4 * cl) cl *= 2;
    while (cl > 1 && clusters_for(cl, smem, fn) < 1) cl /= 2;
    a.CL = cl;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles * cl);
    cfg.blockDim = dim3(GTHR);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    int n = 0;
    if (lmc_pdl_enabled()) {
        at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[n].val.programmaticStreamSerializationAllowed = 1;
        n++;
    }
    if (cl > 1) {
        at[n].id = cudaLaunchAttributeClusterDimension;
        at[n].val.clusterDim.x = cl;
        at[n].val.clusterDim.y = 1;
        at[n].val.clusterDim.z = 1;
        n++;
    }
    cfg.attrs = at;
    cfg.numAttrs = n;
    void *args[1] = {&a};
    cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return lmc_set_error(LMC_ERR_CUDA, "gemm launch: %s", cudaGetErrorString(e));
    return LMC_OK;
}
