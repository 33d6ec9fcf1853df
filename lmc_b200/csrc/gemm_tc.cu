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

constexpr int BM = 128, BK = 64, GTHR = 256;
constexpr uint32_t LO4C = 0x0F0F0F0Fu;

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
    int key_base;  // global index of row 0 in the keys
    int BN, MT, CL, nkb;
    const uint8_t *wt;  // tiled copy (16-row x 256-column units), or NULL
    int RT, KBU;        // row tiles and unit columns of the tiled copy
    const uint8_t *xs;  // Q4_K fast path: 32-column sums of the scaled x (x 2^-5) as MMA tiles, see k_gemm_prep_x
    int Npad;  // fast path: x tiles are [K/64][Npad][64], pre-swizzled
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
// Limit of every bounded wait below (nanoseconds of %globaltimer).
__device__ long long g_gemm_wait_ns = 1000000000ll;
// bounded: about one second (g_gemm_wait_ns), then the flag is set and the caller goes on
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
    if (bar_try(bar, parity)) return true;
    long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
        if (bar_try(bar, parity)) return true;
        long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > g_gemm_wait_ns) break;
    }
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

// D (+)= A B.  The accumulate flag is an immediate in one of two forms: a
// predicate set per MMA made the issue loop about three times slower than
// the MMA itself.
__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    if (acc)
        asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 1;" ::"r"(tmem), "l"(a), "l"(b), "r"(id));
    else
        asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 0;" ::"r"(tmem), "l"(a), "l"(b), "r"(id));
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
// 32 lanes x 16 columns of 32-bit TMEM words; the caller waits (tcgen05.wait::ld)
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
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

// Stores output (token n, row m) and returns its greedy-pick key.
__device__ __forceinline__ unsigned long long epi_store(const GArgs &a, int n, int m, float v) {
    if (a.bias) v += a.bias[m];
    if (a.epi & LMC_EPI_GELU) v = lmc_gelu_f(v);
    float *o = a.y + (size_t)n * a.ldy + m;
    *o = (a.epi & LMC_EPI_ACCUM) ? *o + v : v;
    return lmc_argmax_key(v, m + a.key_base);
}
// Warp-collective epilogue of NC consecutive columns nc0.. (warp-uniform)
// for row m (per lane), v[c] the unscaled sums: every load (activation
// scales, bias, old Y) is issued before the first store.
template <int NC>
__device__ __forceinline__ void epi_cols(const GArgs &a, int nc0, int m, const float (&v)[NC]) {
    const bool mok = m < a.M;
    const float bm = (a.bias && mok) ? __ldg(a.bias + m) : 0.0f;
    float xi[NC], old[NC];
#pragma unroll
    for (int c = 0; c < NC; c++) {
        const int n = nc0 + c;
        xi[c] = n < a.N ? __ldg(a.xinv + n) : 0.0f;
        old[c] = (a.epi & LMC_EPI_ACCUM) && n < a.N && mok ? a.y[(size_t)n * a.ldy + m] : 0.0f;
    }
#pragma unroll
    for (int c = 0; c < NC; c++) {
        const int n = nc0 + c;
        float r = v[c] * xi[c] + bm;
        if (a.epi & LMC_EPI_GELU) r = lmc_gelu_f(r);
        if (n < a.N && mok) a.y[(size_t)n * a.ldy + m] = (a.epi & LMC_EPI_ACCUM) ? old[c] + r : r;
        if (a.keys && n < a.N) {
            const unsigned long long k = n < a.N && mok ? lmc_argmax_key(r, m + a.key_base) : 0ull;
            const unsigned hi = (unsigned)(k >> 32), lo = (unsigned)k;
            const unsigned mh = __reduce_max_sync(0xffffffffu, hi);
            const unsigned ml = __reduce_max_sync(0xffffffffu, hi == mh ? lo : 0u);
            if ((threadIdx.x & 31) == 0 && (mh | ml)) atomicMax(a.keys + n, ((unsigned long long)mh << 32) | ml);
        }
    }
}
// Same for the columns nc0 + 4 k, 4 k < lim, k < 8.
__device__ __forceinline__ void epi_strided(const GArgs &a, int nc0, int lim, int m, const float (&v)[8]) {
    const bool mok = m < a.M;
    const float bm = (a.bias && mok) ? __ldg(a.bias + m) : 0.0f;
    float xi[8], old[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int n = nc0 + 4 * k;
        const bool nok = 4 * k < lim && n < a.N;
        xi[k] = nok ? __ldg(a.xinv + n) : 0.0f;
        old[k] = (a.epi & LMC_EPI_ACCUM) && nok && mok ? a.y[(size_t)n * a.ldy + m] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
        if (4 * k >= lim) break;
        const int n = nc0 + 4 * k;
        float r = v[k] * xi[k] + bm;
        if (a.epi & LMC_EPI_GELU) r = lmc_gelu_f(r);
        if (n < a.N && mok) a.y[(size_t)n * a.ldy + m] = (a.epi & LMC_EPI_ACCUM) ? old[k] + r : r;
        if (a.keys && n < a.N) {
            const unsigned long long kk = mok ? lmc_argmax_key(r, m + a.key_base) : 0ull;
            const unsigned hi = (unsigned)(kk >> 32), lo = (unsigned)kk;
            const unsigned mh = __reduce_max_sync(0xffffffffu, hi);
            const unsigned ml = __reduce_max_sync(0xffffffffu, hi == mh ? lo : 0u);
            if ((threadIdx.x & 31) == 0 && (mh | ml)) atomicMax(a.keys + n, ((unsigned long long)mh << 32) | ml);
        }
    }
}
// Warp-collective epilogue of column n (warp-uniform) for row m (per lane):
// store, then one atomic per warp for the greedy key of the column (the
// 64-bit maximum as two 32-bit warp reductions).
__device__ __forceinline__ void epi_col(const GArgs &a, int n, int m, float v) {
    unsigned long long k = 0ull;
    if (n < a.N && m < a.M) k = epi_store(a, n, m, v);
    if (a.keys && n < a.N) {
        const unsigned hi = (unsigned)(k >> 32), lo = (unsigned)k;
        const unsigned mh = __reduce_max_sync(0xffffffffu, hi);
        const unsigned ml = __reduce_max_sync(0xffffffffu, hi == mh ? lo : 0u);
        if ((threadIdx.x & 31) == 0 && (mh | ml)) atomicMax(a.keys + n, ((unsigned long long)mh << 32) | ml);
    }
}

// Accumulator (TMEM lanes = tile rows, columns = tokens) -> Y.  Warp w reads
// TMEM lanes 32 (w % 4) .. +31; with 8 warps, warps 4-7 take the second half
// of the columns.  With a cluster split of K, partials are added into the
// leader's shared memory ([BN][128] fp32 over its idle stages) first.
template <int NW>
__device__ __forceinline__ void gemm_epilogue(const GArgs &a, uint32_t tmem, int m0, int n0, bool has_acc, int rank,
                                              uint8_t *smem) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, BN = a.BN;
    const int q = warp & 3, cbeg = NW == 8 ? (warp >> 2) * (BN / 2) : 0, cend = NW == 8 ? cbeg + BN / 2 : BN;
    const int row = 32 * q + lane, m = m0 + row;
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
    const float wi = a.winv;
    if (a.CL == 1) {
        for (int c0 = cbeg; c0 < cend; c0 += 16) {
            float v[16];
            if (has_acc) tmem_ld16(trow + c0, v);
            else
#pragma unroll
                for (int i = 0; i < 16; i++) v[i] = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const int n = n0 + c0 + i;
                epi_col(a, n, m, v[i] * (wi * (n < a.N ? a.xinv[n] : 0.0f)));
            }
        }
        return;
    }
    float *red = reinterpret_cast<float *>(smem);
    if (rank == 0)
        for (int c0 = cbeg; c0 < cend; c0 += 16) {
            float v[16];
            if (has_acc) tmem_ld16(trow + c0, v);
            else
#pragma unroll
                for (int i = 0; i < 16; i++) v[i] = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; i++) red[(c0 + i) * BM + row] = v[i];
        }
    cl_arrive();
    cl_wait();  // the leader's tile holds its partial
    if (rank != 0 && has_acc)
        for (int c0 = cbeg; c0 < cend; c0 += 16) {
            float v[16];
            tmem_ld16(trow + c0, v);
#pragma unroll
            for (int i = 0; i < 16; i++) red_remote(su32(&red[(c0 + i) * BM + row]), 0u, v[i]);
        }
    cl_arrive();
    cl_wait();  // every partial added
    if (rank == 0)
        for (int c = cbeg; c < cend; c++) {
            const int n = n0 + c;
            epi_col(a, n, m, red[c * BM + row] * (wi * (n < a.N ? a.xinv[n] : 0.0f)));
        }
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
    bool ok = true;
    for (int it = 0; it < nit; it++) {
        const int s = it & 1, kb = kb0 + it;
        uint8_t *A = smem + s * stage_bytes, *Bh = A + BM * 128, *Bl = Bh + BN * 128;
        if (it >= 2 && ok) ok = bar_wait(su32(&bars[s]), (uint32_t)(((it - 2) >> 1) & 1));  // stage free
        // A: 128 rows x 8 groups of 8 weights -> swizzled 16-byte chunks; the 8
        // lanes of a row take its 8 consecutive groups (neighbouring bytes)
#pragma unroll 2
        for (int q0 = 0; q0 < BM * 8 / GTHR; q0++) {
            const int idx = tid + q0 * GTHR, r = idx >> 3, c = idx & 7, m = m0 + r;
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
            *reinterpret_cast<uint4 *>(A + r * 128 + ((c ^ (r & 7)) << 4)) = q;
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
            // 16 fp16 = 32 bytes per K step = 2 in the descriptors' address field
            const uint64_t ad = sdesc(su32(A)), bh = sdesc(su32(Bh)), bl = sdesc(su32(Bl));
            mma_f16(tmem, ad, bh, id, it > 0 ? 1u : 0u);
            mma_f16(tmem, ad, bl, id, 1u);
#pragma unroll
            for (int j = 1; j < BK / 16; j++) {
                mma_f16(tmem, ad + 2 * j, bh + 2 * j, id, 1u);
                mma_f16(tmem, ad + 2 * j, bl + 2 * j, id, 1u);
            }
            mma_commit(su32(&bars[s]));
        }
    }
    if (nit > 0 && ok) ok = bar_wait(su32(&bars[(nit - 1) & 1]), (uint32_t)(((nit - 1) >> 1) & 1));
    tc_fence_after();
    gemm_epilogue<GTHR / 32>(a, tmem, m0, n0, nit > 0, rank, smem);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
}

// ---------------------------------------------------------------------------
// Fast path for the formats with a tiled copy (Q4_K, Q6_K, Q8_0): the CTA's
// 8 units (16 rows x 256 columns each, 16-byte aligned, contiguous) of a unit
// column arrive by 8 bulk async copies into one of two raw stages; warp u turns
// unit u into fp16 for each 64-column k-block.  Codes become fp16 with the
// 1024 trick: (code | 0x6400) is the fp16 1024 + code, one LOP3 gives two, one
// HSUB2 removes the 1024 (exact) and one HFMA2 applies scale and min.  A
// lane's code word holds columns 4c..4c+3 and 16+4c..16+4c+3 of its 32-column
// group in the order the extraction yields, so the activations are stored
// with the same column permutation (see perm_pos) and no shuffles are needed.
// ---------------------------------------------------------------------------
__host__ __device__ constexpr int tunit_bytes(int qt) { return qt == 4 ? 2304 : qt == 6 ? 3360 : 4352; }

__device__ __forceinline__ __half2 u2h(uint32_t v) { return *reinterpret_cast<const __half2 *>(&v); }
__device__ __forceinline__ uint32_t h2u(__half2 v) { return *reinterpret_cast<const uint32_t *>(&v); }
__device__ __forceinline__ int tcode_word(int n, int t) { return ((n >> 2) * 32 + t) * 4 + (n & 3); }

// Nibble order of the converted codes: 8 nibble codes (bytes 0-3, low and
// high nibbles) give the fp16 values in the order (b0.lo, b2.lo, b1.lo,
// b3.lo, b0.hi, b2.hi, b1.hi, b3.hi)
// 4 byte codes -> 4 fp16 (q - OFF) * s, order (b0, b2, b1, b3); OFF = 32 for
// Q6_K codes 0..63, 128 for int8 codes stored with the sign bit flipped
template <int OFF> __device__ __forceinline__ uint2 cvt_byte(uint32_t q, __half2 s) {
    const __half2 k = __float2half2_rn(1024.0f + OFF);
    uint2 r;
    r.x = h2u(__hmul2(__hsub2(u2h((q & 0x00FF00FFu) | 0x64006400u), k), s));
    r.y = h2u(__hmul2(__hsub2(u2h(((q >> 8) & 0x00FF00FFu) | 0x64006400u), k), s));
    return r;
}
__device__ __forceinline__ void put_chunk(uint8_t *A, int row, int chunk, uint4 v) {
    *reinterpret_cast<uint4 *>(A + row * 128 + ((chunk ^ (row & 7)) << 4)) = v;
}
// 16-column K-major tile without swizzle: 8-row x 16-byte core matrices,
// column chunk kc at +128 bytes, 8-row group rg at +256 bytes.
__device__ __forceinline__ void put_core(uint8_t *T, int row, int kc, uint4 v) {
    *reinterpret_cast<uint4 *>(T + (row >> 3) * 256 + kc * 128 + (row & 7) * 16) = v;
}
__device__ __forceinline__ uint64_t sdesc_plain(uint32_t addr) {  // layout type 0, LBO 128 B, SBO 256 B
    return (uint64_t)((addr >> 4) & 0x3FFFu) | (8ull << 16) | (16ull << 32) | (1ull << 46);
}

// Q4_K 6-bit scale / min of sub-block j (src/quant.c:44-53) from the header words
__device__ __forceinline__ void q4k_scale(const uint4 &H, int j, int &sc, int &mn) {
    if (j < 4) {
        sc = (H.y >> (8 * j)) & 63;
        mn = (H.z >> (8 * j)) & 63;
    } else {
        const int i = 8 * (j - 4);
        sc = ((H.w >> i) & 0x0F) | (((H.y >> i) >> 6 & 3) << 4);
        mn = ((H.w >> i) >> 4 & 0x0F) | (((H.z >> i) >> 6 & 3) << 4);
    }
}

// 8 nibble codes -> 8 fp16 q * sc (order above), one fused multiply-add per
// pair: (1024 + q) sc - 1024 sc is exact (the result q sc <= 945 and
// 1024 sc <= 64512 are fp16 integers, the product is not rounded).
__device__ __forceinline__ uint4 cvt_nib_fma(uint32_t P, __half2 sc, __half2 nsc) {
    uint4 r;
    r.x = h2u(__hfma2(u2h((P & 0x000F000Fu) | 0x64006400u), sc, nsc));
    r.y = h2u(__hfma2(u2h(((P >> 8) & 0x000F000Fu) | 0x64006400u), sc, nsc));
    r.z = h2u(__hfma2(u2h(((P >> 4) & 0x000F000Fu) | 0x64006400u), sc, nsc));
    r.w = h2u(__hfma2(u2h(((P >> 12) & 0x000F000Fu) | 0x64006400u), sc, nsc));
    return r;
}

// Per unit column state of one converter warp of the warp-specialised
// kernel: the 16-byte headers of its rows r0 = 16u + g and r1 = r0 + 8
// (Q4_K d, dmin, scales; Q6_K the 16 int8 scales; Q8_0 the 8 fp16 block
// scales) and, for Q4_K, the scale multipliers of its four k-blocks.
struct ConvUnit {
    uint4 H0, H1;
    uint32_t s0, s1;  // Q4_K: byte h = the 6-bit scale of sub-block 2 h + part, rows r0 / r1
};
template <int QT>
__device__ __forceinline__ void conv_unit(ConvUnit &cu, const uint8_t *U, int part, int lane) {
    const int g = lane >> 2;
    cu.H0 = *reinterpret_cast<const uint4 *>(U + 16 * g);
    cu.H1 = *reinterpret_cast<const uint4 *>(U + 16 * g + 128);
    if (QT == 4) {
        cu.s0 = cu.s1 = 0u;
#pragma unroll
        for (int h = 0; h < 4; h++) {
            int sc0, m0, sc1, m1;
            q4k_scale(cu.H0, 2 * h + part, sc0, m0);
            q4k_scale(cu.H1, 2 * h + part, sc1, m1);
            cu.s0 |= (uint32_t)sc0 << (8 * h);
            cu.s1 |= (uint32_t)sc1 << (8 * h);
        }
    }
}
// Block scales (and the Q4_K mins rows) of the unit column: part-0 warps.
template <int QT>
__device__ __forceinline__ void conv_unit_side(const ConvUnit &cu, const uint8_t *U, int u, int lane, float ws, float2 *dsc,
                                               uint8_t *Mt) {
    const int g = lane >> 2, c = lane & 3, r0 = 16 * u + g, r1 = r0 + 8;
    if (QT == 4) {
        if (c < 2) {  // lanes c = 0 / 1: the mins rows of r0 / r1
            const uint4 H = c == 0 ? cu.H0 : cu.H1;
            const int r = c == 0 ? r0 : r1;
            int sc, mn[8];
#pragma unroll
            for (int j = 0; j < 8; j++) q4k_scale(H, j, sc, mn[j]);
            uint4 v;
            v.x = h2u(__floats2half2_rn((float)mn[0], (float)mn[1]));
            v.y = h2u(__floats2half2_rn((float)mn[2], (float)mn[3]));
            v.z = h2u(__floats2half2_rn((float)mn[4], (float)mn[5]));
            v.w = h2u(__floats2half2_rn((float)mn[6], (float)mn[7]));
            put_core(Mt, r, 0, v);
            put_core(Mt, r, 1, make_uint4(0u, 0u, 0u, 0u));
            dsc[r] = __half22float2(u2h(H.x));  // (d, dmin)
        }
    } else if (QT == 6) {
        if (c == 0) {
            dsc[r0] = make_float2(__half2float(*reinterpret_cast<const __half *>(U + 256 + 2 * g)), 0.0f);
            dsc[r1] = make_float2(__half2float(*reinterpret_cast<const __half *>(U + 256 + 2 * g + 16)), 0.0f);
        }
    } else if (c == 0) {
        dsc[r0] = dsc[r1] = make_float2(1.0f / ws, 0.0f);
    }
}
// k-block H of the unit column, K half `part`, rows r0 / r1 of the A tile:
//   Q4_K: A = q * sc (exact); Q6_K: A = sc * (q - 32) (exact up to 2048 in
//   magnitude, nearest-even above); Q8_0: A = fp16(q * d * ws) (one rounding).
// The block scales enter at readout (dsc): Q4_K d * sum(q sc x) - dmin *
// sum_j m_j X_j, Q6_K d, Q8_0 1 / ws.
__device__ __forceinline__ uint32_t pick4r(const uint4 &v, int j) { return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w; }
template <int QT>
__device__ __forceinline__ void conv_step(uint8_t *A, const uint8_t *U, const ConvUnit &cu, int u, int part, int lane, float ws,
                                          int H) {
    const int g = lane >> 2, c = lane & 3, r0 = 16 * u + g, r1 = r0 + 8;
    if (QT == 4) {
        const uint32_t *cw = reinterpret_cast<const uint32_t *>(U + 256);
        const int j = 2 * H + part;
        const uint32_t P = cw[tcode_word(2 * j, lane)], Q = cw[tcode_word(2 * j + 1, lane)];
        const __half2 m1024 = __float2half2_rn(-1024.0f);
        const __half2 s0 = __float2half2_rn((float)((cu.s0 >> (8 * H)) & 0xFFu)), s1 = __float2half2_rn((float)((cu.s1 >> (8 * H)) & 0xFFu));
        put_chunk(A, r0, 4 * part + c, cvt_nib_fma(P, s0, __hmul2(s0, m1024)));
        put_chunk(A, r1, 4 * part + c, cvt_nib_fma(Q, s1, __hmul2(s1, m1024)));
    } else if (QT == 6) {
        const uint32_t *lw = reinterpret_cast<const uint32_t *>(U + 288), *hw = reinterpret_cast<const uint32_t *>(U + 288 + 2048);
        const uint32_t w0 = pick4r(cu.H0, H), w1 = pick4r(cu.H1, H);  // scales of chunks 4H..4H+3
        const int j = 4 * H + 2 * part;                                   // even chunk; j + 1 odd
        const uint32_t P0 = lw[tcode_word(j, lane)], P1 = lw[tcode_word(j + 1, lane)];
        const uint32_t Hb = hw[tcode_word(j >> 1, lane)];
        const uint32_t a0 = (P0 & LO4C) | ((Hb << 4) & 0x30303030u), a1 = (P1 & LO4C) | (Hb & 0x30303030u);
        const uint32_t b0 = ((P0 >> 4) & LO4C) | ((Hb << 2) & 0x30303030u), b1 = ((P1 >> 4) & LO4C) | ((Hb >> 2) & 0x30303030u);
        const int e0 = 2 * part, e1 = e0 + 1;
        const __half2 sg0 = __float2half2_rn((float)(int8_t)((w0 >> (8 * e0)) & 0xFF));
        const __half2 sg1 = __float2half2_rn((float)(int8_t)((w0 >> (8 * e1)) & 0xFF));
        const __half2 sh0 = __float2half2_rn((float)(int8_t)((w1 >> (8 * e0)) & 0xFF));
        const __half2 sh1 = __float2half2_rn((float)(int8_t)((w1 >> (8 * e1)) & 0xFF));
        const uint2 x0 = cvt_byte<32>(a0, sg0), x1 = cvt_byte<32>(a1, sg1);
        const uint2 y0 = cvt_byte<32>(b0, sh0), y1 = cvt_byte<32>(b1, sh1);
        put_chunk(A, r0, 4 * part + c, make_uint4(x0.x, x0.y, x1.x, x1.y));
        put_chunk(A, r1, 4 * part + c, make_uint4(y0.x, y0.y, y1.x, y1.y));
    } else {
        const uint4 *cw = reinterpret_cast<const uint4 *>(U + 256);
        const int j = 2 * H + part;  // block j of each row; its scale is half (j & 1) of header word H
        const uint4 Aw = cw[j * 32 + lane];
        const float2 f0 = __half22float2(u2h(pick4r(cu.H0, H))), f1 = __half22float2(u2h(pick4r(cu.H1, H)));
        const __half2 s0 = __float2half2_rn((part ? f0.y : f0.x) * ws);
        const __half2 s1 = __float2half2_rn((part ? f1.y : f1.x) * ws);
        const uint2 x0 = cvt_byte<128>(Aw.x ^ 0x80808080u, s0), x1 = cvt_byte<128>(Aw.z ^ 0x80808080u, s0);
        const uint2 y0 = cvt_byte<128>(Aw.y ^ 0x80808080u, s1), y1 = cvt_byte<128>(Aw.w ^ 0x80808080u, s1);
        put_chunk(A, r0, 4 * part + c, make_uint4(x0.x, x0.y, x1.x, x1.y));
        put_chunk(A, r1, 4 * part + c, make_uint4(y0.x, y0.y, y1.x, y1.y));
    }
}

__device__ __forceinline__ void bulk_copy(uint32_t bar, void *dst, const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     su32(dst)),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Accumulators of one unit column -> registers, NC columns (multiple of 8)
// of one TMEM lane quarter in steps of 8: acc[c] += d * main - 32 dmin * mins.
// The MMAs run with N = 2 BN (hi rows then lo rows of x), so main and mins
// are column c plus column c + BN; the sums of x enter the mins MMA x 2^-5.
template <int QT, int BN, int NC>
__device__ __forceinline__ void block_readout_n(float (&acc)[NC], uint32_t tmain, uint32_t tmins, float2 dd) {
    static_assert(NC == 16, "one x16 load per accumulator part");
    uint32_t v[16], vl[16], mv[16], ml[16];
    tmem_ld16_nowait(tmain, v);  // every load in flight, one wait
    tmem_ld16_nowait(tmain + BN, vl);
    if (QT == 4) {
        tmem_ld16_nowait(tmins, mv);
        tmem_ld16_nowait(tmins + BN, ml);
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const float main = __uint_as_float(v[i]) + __uint_as_float(vl[i]);
        if (QT == 4)
            acc[i] += dd.x * main - (32.0f * dd.y) * (__uint_as_float(mv[i]) + __uint_as_float(ml[i]));
        else
            acc[i] += dd.x * main;
    }
}

// Fast path for the tiled Q4_K / Q6_K / Q8_0 copies: one CTA per 128-row x
// 64-token output tile (and K range of its cluster rank), warp-specialised,
// every hand-off an mbarrier:
//   warp 16 (producer, one lane): bulk copies of the weight units (8 per unit
//           column: 128 rows x 256 K) into R raw stages, of the activation
//           tiles (hi | lo, 64 K) into SB stages and, for Q4_K, of the
//           32-column sums tile with each unit column; L2 prefetch one unit
//           column further ahead.  Weights go out before the wait on the
//           previous kernel (they do not depend on it).
//   warp 17 (MMA, one lane): per 64-K step four tcgen05.mma (M 128, N 128 =
//           hi rows then lo rows, K 16) into the unit column's accumulator
//           (two in TMEM, alternating), plus the Q4_K mins MMA on the first
//           step; commits free the A and activation stages (and, with the
//           mins MMA, the raw stage) and mark the accumulator full.
//   warps 0-15: warp w converts rows 16u..16u+15 (u = w % 8), K half w / 8,
//           of each 64-K step into the A stage (exact integer * scale fp16,
//           conv_step), then, one step into the next unit column, reads its
//           16 columns (w / 4) of TMEM lane quarter w % 4 out of the previous
//           accumulator with the per-row block scales and frees it.
// After the last unit column: epilogue (direct, or a reduce-scatter over the
// cluster when K is split).
constexpr int WS_CONV = 16, WS_THREADS = 32 * (WS_CONV + 2);
template <int QT> struct WsCfg {
    static constexpr int R = QT == 8 ? 2 : 3, SA = 4, SB = 4;
    static constexpr int UNIT = tunit_bytes(QT), RAWB = 8 * UNIT;
    static constexpr int ABYTES = BM * 128, BBYTES = 2 * 64 * 128, MBYTES = QT == 4 ? 8192 : 0;
    static constexpr int A_OFF = 0, B_OFF = A_OFF + SA * ABYTES, R_OFF = B_OFF + SB * BBYTES;
    static constexpr int M_OFF = R_OFF + R * RAWB, D_OFF = M_OFF + R * MBYTES, BAR_OFF = D_OFF + 4 * BM * 8;
    static_assert(SA == SB && SA == 4, "hand-offs by pairs of stages (128 K): two pair slots");
    static constexpr int PS = SA / 2;
    static constexpr int NBARS = 2 * R + 2 * PS + 5;
    static constexpr int SLOT_OFF = BAR_OFF + NBARS * 8, TOTAL = SLOT_OFF + 16;
};
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void l2_prefetch(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void converters_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * WS_CONV) : "memory"); }

template <int QT>
__global__ void __launch_bounds__(WS_THREADS, 1) k_gemm_ws(GArgs a) {
    static_assert(BM * 4 == 32 * WS_CONV, "the reduce-scatter tail maps 4 columns x 128 rows onto the converters");
    using C = WsCfg<QT>;
    constexpr int BN = 64, R = C::R, UNIT = C::UNIT;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *As = smem + C::A_OFF, *Bs = smem + C::B_OFF, *raw = smem + C::R_OFF, *mins = smem + C::M_OFF;
    float2 *dsc = reinterpret_cast<float2 *>(smem + C::D_OFF);  // [4][BM] (d, dmin) per unit column
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    // Hand-offs are by pairs of 64-K steps (128 K, stages 2 ps and 2 ps + 1 of
    // pair slot ps): full[ps] = the converter warps' A tiles and the producer's
    // activation tiles (its expect-tx arrival) of the pair; empty[ps] = the
    // pair's MMAs are done (one commit), all four tiles may be refilled.
    constexpr int PS = C::PS;
    uint64_t *raw_full = bars, *raw_empty = bars + R, *full = bars + 2 * R, *empty = full + PS;
    uint64_t *acc_full = empty + PS, *acc_empty = acc_full + 2;
    uint64_t *mma_done = acc_empty + 2;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + C::SLOT_OFF);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rank = a.CL > 1 ? (int)ctarank() : 0;
    const int tile = a.CL > 1 ? (int)clusterid() : (int)blockIdx.x;
    const int m0 = (tile % a.MT) * BM, n0 = (tile / a.MT) * BN, rt0 = m0 / 16;
    const int kb0 = (int)((long long)rank * a.nkb / a.CL), kb1 = (int)((long long)(rank + 1) * a.nkb / a.CL);
    const int nu = kb1 - kb0;            // unit columns of this CTA
    const int nut = min(8, a.RT - rt0);  // unit rows present in this tile
    const int nq = 2 * nu;               // 128-K hand-offs (pairs of 64-K steps)
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tslot)), "r"(8 * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 32) {
        for (int s = 0; s < R; s++) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], WS_CONV + (QT == 4 ? 1 : 0));  // converter warps (+ the mins MMA's commit)
        }
        for (int s = 0; s < PS; s++) {
            mbar_init(&full[s], WS_CONV + 1);
            mbar_init(&empty[s], 1);
        }
        for (int p = 0; p < 2; p++) {
            mbar_init(&acc_full[p], 1);
            mbar_init(&acc_empty[p], WS_CONV);
        }
        mbar_init(mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_launch_dependents();
    constexpr int NC = BN / 4;  // accumulator columns per converter warp
    const int q = warp & 3, cb = (warp >> 2) * NC, row = 32 * q + lane;
    float acc[NC];
#pragma unroll
    for (int i = 0; i < NC; i++) acc[i] = 0.0f;
    bool ok = true;
    if (warp == WS_CONV) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const size_t xs_tile = ((size_t)(a.Npad / 64)) * 4096;  // bytes per unit column of the sums tiles
            auto weights = [&](int i) {  // unit column i: expect its bytes, copy its 8 weight units
                uint64_t *bar = &raw_full[i % R];
                mbar_expect(bar, (uint32_t)(nut * UNIT + (QT == 4 ? 4096 : 0)));
                for (int u = 0; u < nut; u++)
                    bulk_copy(su32(bar), raw + (i % R) * C::RAWB + u * UNIT,
                              a.wt + ((size_t)(rt0 + u) * a.KBU + kb0 + i) * UNIT, UNIT);
                if (i + R < nu)
                    for (int u = 0; u < nut; u++)
                        l2_prefetch(a.wt + ((size_t)(rt0 + u) * a.KBU + kb0 + i + R) * UNIT, UNIT);
            };
            auto sums = [&](int i) {  // Q4_K: the unit column's sums tile (hi | lo rows of this token tile)
                if (QT == 4)
                    bulk_copy(su32(&raw_full[i % R]), mins + (i % R) * C::MBYTES + 4096,
                              a.xs + (size_t)(kb0 + i) * xs_tile + (size_t)(n0 / 64) * 4096, 4096);
            };
            auto acts = [&](int q) {  // pair q: activation tiles (hi then lo) of steps 2 q, 2 q + 1
                uint64_t *bar = &full[q % PS];
                mbar_expect(bar, (uint32_t)(2 * C::BBYTES));
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    uint8_t *dst = Bs + (2 * (q % PS) + e) * C::BBYTES;
                    const size_t off = ((size_t)(4 * kb0 + 2 * q + e) * a.Npad + n0) * BK;
                    bulk_copy(su32(bar), dst, a.xh + off, BN * 128);
                    bulk_copy(su32(bar), dst + BN * 128, a.xl + off, BN * 128);
                }
            };
            const int npre = min(R, nu);
            for (int i = 0; i < npre; i++) weights(i);
            pdl_wait();  // activations and sums are written by the previous kernel
            for (int i = 0; i < npre; i++) sums(i);
            int nq_issued = min(PS, nq), nu_issued = npre;
            for (int q = 0; q < nq_issued; q++) acts(q);
            for (int q = 0; q < nq && ok; q++) {
                if (q + PS < nq) {  // the pair slot of q is free once its MMAs are done
                    ok = bar_wait(su32(&empty[q % PS]), (uint32_t)((q / PS) & 1));
                    if (!ok) break;
                    acts(q + PS);
                    nq_issued = q + PS + 1;
                }
                if ((q & 1) == 1 && (q >> 1) + R < nu) {  // unit column q / 2 consumed: refill its stage
                    const int i = q >> 1;
                    ok = bar_wait(su32(&raw_empty[i % R]), (uint32_t)((i / R) & 1));
                    if (!ok) break;
                    weights(i + R);
                    sums(i + R);
                    nu_issued = i + R + 1;
                }
            }
            // every copy issued has landed before the CTA can exit (bounded;
            // immediate when the consumers saw them)
            for (int i = max(0, nu_issued - R); i < nu_issued; i++)
                (void)bar_wait(su32(&raw_full[i % R]), (uint32_t)((i / R) & 1));
            for (int q = max(0, nq_issued - PS); q < nq_issued; q++)
                (void)bar_wait(su32(&full[q % PS]), (uint32_t)((q / PS) & 1));
        }
        __syncwarp();
    } else if (warp == WS_CONV + 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t id = idesc(2 * BN);  // N = 2 BN: hi tile rows then lo tile rows
            // stage s: the base descriptors plus s stages in 16-byte units (the address field)
            const uint64_t adesc0 = sdesc(su32(As)), bdesc0 = sdesc(su32(Bs));
            for (int q = 0; q < nq; q++) {
                const int i = q >> 1, h2 = q & 1, p = i & 1;
                if (ok) ok = bar_wait(su32(&full[q % PS]), (uint32_t)((q / PS) & 1));
                if (ok && h2 == 0 && i >= 2) ok = bar_wait(su32(&acc_empty[p]), (uint32_t)(((i - 2) >> 1) & 1));
                if (!ok) break;
                tc_fence_after();
                const uint32_t tmain = tmem + 4 * BN * p;
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    // 16 fp16 = 32 bytes per K step = 2 in the descriptors' address field
                    const int st = 2 * (q % PS) + e;
                    const uint64_t ad = adesc0 + (uint64_t)(st * (C::ABYTES >> 4)), bd = bdesc0 + (uint64_t)(st * (C::BBYTES >> 4));
                    mma_f16(tmain, ad, bd, id, (h2 > 0 || e > 0) ? 1u : 0u);
#pragma unroll
                    for (int j = 1; j < BK / 16; j++) mma_f16(tmain, ad + 2 * j, bd + 2 * j, id, 1u);
                }
                if (QT == 4 && h2 == 0) {
                    const uint32_t Mt = su32(mins + (i % R) * C::MBYTES);
                    mma_f16(tmain + 2 * BN, sdesc_plain(Mt), sdesc_plain(Mt + 4096), id, 0u);
                }
                mma_commit(su32(&empty[q % PS]));
                if (QT == 4 && h2 == 0) mma_commit(su32(&raw_empty[i % R]));
                if (h2 == 1) mma_commit(su32(&acc_full[p]));
            }
            mma_commit(su32(mma_done));  // every MMA issued above is complete once this arrives
            (void)bar_wait(su32(mma_done), 0u);
        }
        __syncwarp();
    } else {
        // ---------------- converters / accumulator readout ----------------
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + cb;
        auto readout = [&](int iu) {
            converters_sync();  // the block scales of unit column iu (every warp's rows) are in dsc
            const int p = iu & 1;
            if (ok) ok = bar_wait(su32(&acc_full[p]), (uint32_t)((iu >> 1) & 1));
            tc_fence_after();
            if (ok) block_readout_n<QT, BN, NC>(acc, tq + 4 * BN * p, tq + 4 * BN * p + 2 * BN, dsc[(iu & 3) * BM + row]);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[p]);
        };
        const int u = warp & 7, part = warp >> 3;
        const bool has = u < nut;
        ConvUnit cu;
        for (int i = 0; i < nu; i++) {
            const int s = i % R;
            if (ok) ok = bar_wait(su32(&raw_full[s]), (uint32_t)((i / R) & 1));
            const uint8_t *U = raw + s * C::RAWB + u * UNIT;
            if (ok && has) conv_unit<QT>(cu, U, part, lane);
            // pair P of unit column i (hand-off q = 2 i + P: 64-K steps 2 P, 2 P + 1);
            // one copy of the loop body (the instruction cache is shared by 18 warps)
#pragma unroll 1
            for (int P = 0; P < 2; P++) {
                const int q = 2 * i + P;
                if (q >= PS && ok) ok = bar_wait(su32(&empty[q % PS]), (uint32_t)(((q - PS) / PS) & 1));
                if (ok && has) {
                    // the mins stage and the dsc slot are free: their last readers (the MMAs of
                    // unit column i - R, the readout of unit column i - 4) are done
                    if (P == 0 && part == 0)
                        conv_unit_side<QT>(cu, U, u, lane, a.wscale, dsc + (i & 3) * BM, mins + s * C::MBYTES);
#pragma unroll 1
                    for (int e = 0; e < 2; e++)
                        conv_step<QT>(As + (2 * (q % PS) + e) * C::ABYTES, U, cu, u, part, lane, a.wscale, 2 * P + e);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[q % PS]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[s]);
            // previous unit column: its MMAs are done (this unit column's second
            // pair waited for them) and the next unit column's MMAs need its
            // accumulator back
            if (i > 0) readout(i - 1);
        }
        if (nu > 0) readout(nu - 1);
    }
    tc_fence_before();
    __syncthreads();  // MMAs complete, TMEM read
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(8 * BN));
    pdl_wait();  // bias, Y and the activation scales are ready
    const int m = m0 + row;
    if (a.CL == 1) {
        if (warp < WS_CONV) epi_cols<NC>(a, n0 + cb, m, acc);
        return;
    }
    // reduce-scatter over the cluster: rank o finishes columns [o W, (o + 1) W),
    // W = BN / CL; every rank stores its partial of them into rank o's
    // buffer slot [source rank][column][row] (plain remote stores), then each
    // rank sums its CL slots
    const int W = BN / a.CL;
    float *buf = reinterpret_cast<float *>(smem);  // [CL][W][128] over the idle A stages
    cl_arrive();
    cl_wait();  // every rank is done with its stages
    if (warp < WS_CONV)
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const int col = cb + c, o = col / W;
            const uint32_t la = su32(&buf[((size_t)rank * W + (col - o * W)) * BM + row]);
            uint32_t ra;
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"((uint32_t)o));
            asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(acc[c]) : "memory");
        }
    cl_arrive();
    cl_wait();  // every slot written
    // this rank's W columns x 128 rows over the converter threads: row
    // tid % 128, columns tid / 128 + 4 k (warp-uniform), k < W / 4 <= 8
    if (warp < WS_CONV) {
        const int r = tid & (BM - 1), c0 = tid >> 7;
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            v[k] = 0.0f;
            if (c0 + 4 * k < W)
                for (int src = 0; src < a.CL; src++) v[k] += buf[((size_t)src * W + c0 + 4 * k) * BM + r];
        }
        epi_strided(a, n0 + rank * W + c0, W - c0, m0 + r, v);
    }
}

// Position of column src (within its 64-column block) in the fast path's
// order: the order cvt_nib_fma / cvt_byte produce (see conv_step).
__device__ __forceinline__ int perm_pos(int src) {
    const int w = src & 31, i = w & 3, slot = (w & 16 ? 4 : 0) + (i == 1 ? 2 : i == 2 ? 1 : i);
    return 8 * (4 * (src >> 5) + ((w & 15) >> 2)) + slot;
}

// Byte offset of the sum of 32-column chunk j of token row n in the Q4_K
// sums tiles: per unit column (256 K) and 64-token tile one 4 KB tile of
// 128 rows (hi sums of the 64 tokens, then lo) x 16 K, K-major without
// swizzle (8-row x 16-byte core matrices; K columns 8-15 stay zero), the
// B operand of the mins MMA.
__device__ __forceinline__ size_t sums_offset(int n, int j, int Npad) {
    const int r = n & 63, kb = j >> 3, sub = j & 7;
    return ((size_t)kb * (Npad / 64) + (n >> 6)) * 4096 + (r >> 3) * 256 + (r & 7) * 16 + sub * 2;
}

// Activation prep: one CTA per token row n.  The row (SwiGLU: silu(x) * x2)
// is staged in shared memory with every load in flight at once, then
// v = prologue(row) (as the GEMV), scale 2^(14-e) with max|v| < 2^e,
// hi = fp16(v s), lo = fp16(v s - hi).  Fast path: column k goes to position
// perm_pos(k) of its 64-column block, tiles [K/64][Npad][64] pre-swizzled,
// and the 32-column sums (x 2^-5, hi / lo) for the Q4_K mins MMA.
__global__ void __launch_bounds__(256) k_gemm_prep_x(const float *__restrict__ x, int ldx, int K, int pro,
                                                     const float *__restrict__ pw, const float *__restrict__ pb,
                                                     const float *__restrict__ x2, float eps, __half *xh, __half *xl,
                                                     float *xinv, int perm, uint8_t *xs, int N, int Npad) {
    extern __shared__ float row[];  // [K]
    __shared__ float red[32];
    pdl_launch_dependents();
    if (pw)  // norm weights and bias do not depend on the previous kernel: into L1 meanwhile
        for (int k = threadIdx.x * 32; k < K; k += blockDim.x * 32) {
            asm volatile("prefetch.global.L1 [%0];" ::"l"(pw + k));
            if (pb) asm volatile("prefetch.global.L1 [%0];" ::"l"(pb + k));
        }
    pdl_wait();
    const int n = blockIdx.x, tid = threadIdx.x;
    if (n >= N) {  // fast-path padding rows: zero tiles
        for (int k = tid; k < K; k += blockDim.x) {
            const size_t o = ((size_t)(k >> 6) * Npad + n) * 64 + (k & 63);
            xh[o] = __float2half_rn(0.0f);
            xl[o] = __float2half_rn(0.0f);
        }
        if (xs)
            for (int j = tid; j < K / 32; j += blockDim.x) {
                uint8_t *p = xs + sums_offset(n, j, Npad);
                *reinterpret_cast<__half *>(p) = __float2half_rn(0.0f);
                *reinterpret_cast<__half *>(p + 2048) = __float2half_rn(0.0f);
            }
        return;
    }
    const float *xr = x + (size_t)n * ldx, *x2r = pro == LMC_PRO_SWIGLU ? x2 + (size_t)n * ldx : nullptr;
    float s1 = 0.0f;
#pragma unroll 4
    for (int k = 4 * tid; k < K; k += 4 * blockDim.x) {
        float4 v = __ldg(reinterpret_cast<const float4 *>(xr + k));
        if (pro == LMC_PRO_SWIGLU) {
            const float4 u = __ldg(reinterpret_cast<const float4 *>(x2r + k));
            v = make_float4(lmc_silu_f(v.x) * u.x, lmc_silu_f(v.y) * u.y, lmc_silu_f(v.z) * u.z, lmc_silu_f(v.w) * u.w);
        }
        *reinterpret_cast<float4 *>(row + k) = v;
        s1 += pro == LMC_PRO_RMSNORM ? v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w : v.x + v.y + v.z + v.w;
    }
    __syncthreads();  // row[] staged (read below with a different thread mapping)
    float mu = 0.0f, rs = 1.0f;
    if (pro == LMC_PRO_LAYERNORM || pro == LMC_PRO_RMSNORM) {
        s1 = block_sum(s1, red);
        if (pro == LMC_PRO_RMSNORM) {
            rs = 1.0f / sqrtf(s1 / (float)K + eps);
        } else {  // two-pass variance, as src/ops.c:52-54
            mu = s1 / (float)K;
            float s2 = 0.0f;
            for (int k = tid; k < K; k += blockDim.x) s2 += (row[k] - mu) * (row[k] - mu);
            s2 = block_sum(s2, red);
            rs = 1.0f / sqrtf(s2 / (float)K + 1e-5f);
        }
    }
    float mx = 0.0f;
    for (int k = tid; k < K; k += blockDim.x) {
        float v = row[k];
        if (pro == LMC_PRO_LAYERNORM) v = (v - mu) * rs * __ldg(pw + k) + __ldg(pb + k);
        else if (pro == LMC_PRO_RMSNORM) v = __ldg(pw + k) * rs * v;
        row[k] = v;
        mx = fmaxf(mx, fabsf(v));
    }
    mx = block_max(mx, red);  // (its barriers also publish row[])
    const int e = max((int)((__float_as_uint(mx) >> 23) & 0xFF) - 126, -100);
    const float s = mx > 0.0f ? __uint_as_float((uint32_t)(127 + 14 - e) << 23) : 1.0f;
    if (tid == 0) xinv[n] = mx > 0.0f ? __uint_as_float((uint32_t)(127 - 14 + e) << 23) : 0.0f;
    // a warp holds 32 consecutive columns: their sum feeds the Q4_K mins MMA
    for (int k = tid; k < K; k += blockDim.x) {
        const float v = row[k] * s;
        const __half h = __float2half_rn(v);
        size_t o = (size_t)n * K + k;
        if (perm) {  // [K/64][Npad][64], 16-byte chunk c of row n at chunk c ^ (n & 7) (the 128-byte swizzle)
            const int p = perm_pos(k & 63);
            o = ((size_t)(k >> 6) * Npad + n) * 64 + ((((p >> 3) ^ (n & 7)) << 3) | (p & 7));
        }
        xh[o] = h;
        xl[o] = __float2half_rn(v - __half2float(h));
        if (xs) {
            const float t = warp_sum(v) * (1.0f / 32.0f);
            if ((tid & 31) == 0) {
                const __half th = __float2half_rn(t);
                uint8_t *p = xs + sums_offset(n, k >> 5, Npad);
                *reinterpret_cast<__half *>(p) = th;
                *reinterpret_cast<__half *>(p + 2048) = __float2half_rn(t - __half2float(th));
            }
        }
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
static uint8_t *g_xs = NULL;
static float *g_xinv = NULL;
static size_t g_x_cap = 0;  // elements of xh / xl
static int g_xinv_cap = 0;

extern "C" int lmc_gemm_reserve(int N, int K, cudaStream_t s) {
    N = (N + 63) / 64 * 64;  // the fast path pads the token rows to 64
    const size_t need = (size_t)N * K;
    if (need <= g_x_cap && N <= g_xinv_cap) return LMC_OK;
    cudaStreamCaptureStatus cs;
    if (cudaStreamIsCapturing(s, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
        return lmc_set_error(LMC_ERR_INVALID, "gemm: workspace must be reserved before stream capture");
    if (g_xh) cudaFree(g_xh);
    if (g_xl) cudaFree(g_xl);
    if (g_xs) cudaFree(g_xs);
    g_xs = NULL;
    if (g_xinv) cudaFree(g_xinv);
    g_xh = g_xl = NULL;
    g_xinv = NULL;
    g_x_cap = 0;
    g_xinv_cap = 0;
    LMC_CUDA_TRY(cudaMalloc(&g_xh, need * sizeof(__half)));
    LMC_CUDA_TRY(cudaMalloc(&g_xl, need * sizeof(__half)));
    // sums tiles: K N / 4 bytes; K columns 8-15 of every tile stay zero
    LMC_CUDA_TRY(cudaMalloc(&g_xs, need / 4 + 4096));
    LMC_CUDA_TRY(cudaMemset(g_xs, 0, need / 4 + 4096));
    LMC_CUDA_TRY(cudaMalloc(&g_xinv, (size_t)N * sizeof(float)));
    g_x_cap = need;
    g_xinv_cap = N;
    return LMC_OK;
}

extern "C" int lmc_gemm_set_wait_limit(long long ns) {
    const long long v = ns > 0 ? ns : 1000000000ll;
    LMC_CUDA_TRY(cudaMemcpyToSymbol(g_gemm_wait_ns, &v, sizeof v));
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

static int clusters_fit(int cl, size_t smem, const void *fn, int nthr);
static int clusters_for(int cl, size_t smem, const void *fn, int nthr) {
    if (cl == 1) return lmc_sm_count();
    static struct {
        const void *fn;
        size_t smem;
        int cl, n;
    } memo[64];
    static int n_memo = 0;
    for (int i = 0; i < n_memo; i++)
        if (memo[i].fn == fn && memo[i].smem == smem && memo[i].cl == cl) return memo[i].n;
    const int n = clusters_fit(cl, smem, fn, nthr);
    if (n_memo < 64) {
        memo[n_memo].fn = fn;
        memo[n_memo].smem = smem;
        memo[n_memo].cl = cl;
        memo[n_memo++].n = n;
    }
    return n;
}
// clusters of cl CTAs that fit on the GPU at once
static int clusters_fit(int cl, size_t smem, const void *fn, int nthr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl);
    cfg.blockDim = dim3(nthr);
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
    int rc;
    const bool fast = t->tiled && (t->type == LMC_TYPE_Q4_K || t->type == LMC_TYPE_Q6_K || t->type == LMC_TYPE_Q8_0);
    const int Npad = fast ? (N + 63) / 64 * 64 : N;
    if ((rc = lmc_gemm_reserve(Npad, K, s))) return rc;
    // activations -> fp16 hi/lo (with the prologue op; the fast path's column order and tiles)
    if ((size_t)K * 4 > 48 * 1024)
        LMC_CUDA_TRY(cudaFuncSetAttribute(k_gemm_prep_x, cudaFuncAttributeMaxDynamicSharedMemorySize, K * 4));
    LMC_LAUNCH("gemm prep", k_gemm_prep_x, Npad, 256, (size_t)K * 4, s, d_x, ldx, K, ex ? ex->pro : LMC_PRO_NONE,
               ex ? ex->w : (const float *)NULL, ex ? ex->b : (const float *)NULL, ex ? ex->x2 : (const float *)NULL,
               ex ? ex->eps : 0.0f, g_xh, g_xl, g_xinv, fast ? 1 : 0,
               fast && t->type == LMC_TYPE_Q4_K ? g_xs : (uint8_t *)NULL, N, Npad);
    GArgs a = {};
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
    a.key_base = ex ? ex->key_base : 0;
    a.MT = (M + BM - 1) / BM;
    a.wt = (const uint8_t *)t->tiled;
    a.RT = t->tiled_rows / 16;
    a.KBU = K / 256;
    a.xs = g_xs;
    a.Npad = Npad;
    const void *fn = NULL;
    size_t smem;
    int nthr, min_kb;
    if (fast) {
        const int qt = t->type == LMC_TYPE_Q4_K ? 4 : t->type == LMC_TYPE_Q6_K ? 6 : 8;
        a.BN = 64;
        a.nkb = K / 256;
        smem = (qt == 4 ? WsCfg<4>::TOTAL : qt == 6 ? WsCfg<6>::TOTAL : WsCfg<8>::TOTAL) + 1024;
        fn = qt == 4 ? (const void *)k_gemm_ws<4> : qt == 6 ? (const void *)k_gemm_ws<6> : (const void *)k_gemm_ws<8>;
        nthr = WS_THREADS;
        min_kb = 1;
    } else {
        a.BN = N <= 64 ? 64 : N <= 128 ? 128 : 256;
        a.nkb = K / BK;
        smem = 2 * (size_t)(BM * 128 + 2 * a.BN * 128) + 64 + 1024;
        switch (t->type) {
#define LMC_GEMM_FN(TY) \
    case TY: fn = (const void *)k_gemm_tc<TY>; break;
            LMC_FOR_EACH_TYPE(LMC_GEMM_FN)
#undef LMC_GEMM_FN
        default: return lmc_set_error(LMC_ERR_UNSUPPORTED, "gemm: type %u", t->type);
        }
        nthr = GTHR;
        min_kb = 2;
    }
    const int NTL = (N + a.BN - 1) / a.BN, tiles = a.MT * NTL;
    LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    // split K over a cluster of cl CTAs: the cl with the least estimated
    // time, waves x (k-blocks per CTA + one k-block for the cluster
    // reduction), where a wave is as many tiles as clusters of that size fit
    // on the GPU at once (each CTA keeps >= min_kb k-blocks)
    int cl = 1;
    long long best = -1;
    for (int c = 1; c <= 8; c *= 2) {
        if (c > 1 && a.nkb < min_kb * c) break;
        const int fit = clusters_for(c, smem, fn, nthr);
        if (fit < 1) break;
        const long long waves = (tiles + fit - 1) / fit, cost = waves * ((a.nkb + c - 1) / c + (c > 1 ? 1 : 0));
        if (best < 0 || cost < best) {
            best = cost;
            cl = c;
        }
    }
    a.CL = cl;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles * cl);
    cfg.blockDim = dim3(nthr);
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
