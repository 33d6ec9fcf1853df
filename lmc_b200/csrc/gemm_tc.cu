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
    const __half *xsh, *xsl;  // [N][K/32] 32-column sums of the scaled x, x 2^-5, hi / lo
    int K32;
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

// Stores output (token n, row m) and returns its greedy-pick key.
__device__ __forceinline__ unsigned long long epi_store(const GArgs &a, int n, int m, float v) {
    if (a.bias) v += a.bias[m];
    if (a.epi & LMC_EPI_GELU) v = lmc_gelu_f(v);
    float *o = a.y + (size_t)n * a.ldy + m;
    *o = (a.epi & LMC_EPI_ACCUM) ? *o + v : v;
    return lmc_argmax_key(v, m + a.key_base);
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
constexpr int TTHR = 256;
__host__ __device__ constexpr int tunit_bytes(int qt) { return qt == 4 ? 2304 : qt == 6 ? 3360 : 4352; }

__device__ __forceinline__ __half2 u2h(uint32_t v) { return *reinterpret_cast<const __half2 *>(&v); }
__device__ __forceinline__ uint32_t h2u(__half2 v) { return *reinterpret_cast<const uint32_t *>(&v); }
__device__ __forceinline__ int tcode_word(int n, int t) { return ((n >> 2) * 32 + t) * 4 + (n & 3); }

// 8 nibble codes (bytes 0-3: low and high nibbles) -> 8 fp16 integers q * sc
// (exact, <= 945), in the order (b0.lo, b2.lo, b1.lo, b3.lo, b0.hi, b2.hi,
// b1.hi, b3.hi)
__device__ __forceinline__ uint4 cvt_nib(uint32_t P, __half2 sc) {
    const __half2 k = __float2half2_rn(1024.0f);
    uint4 r;
    r.x = h2u(__hmul2(__hsub2(u2h((P & 0x000F000Fu) | 0x64006400u), k), sc));
    r.y = h2u(__hmul2(__hsub2(u2h(((P >> 8) & 0x000F000Fu) | 0x64006400u), k), sc));
    r.z = h2u(__hmul2(__hsub2(u2h(((P >> 4) & 0x000F000Fu) | 0x64006400u), k), sc));
    r.w = h2u(__hmul2(__hsub2(u2h(((P >> 12) & 0x000F000Fu) | 0x64006400u), k), sc));
    return r;
}
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

// Warp u: rows 16u + g and 16u + g + 8 of the A tile for k-block h of its unit.
//   Q4_K: A = q * sc (exact); on h == 0 also the row's 8 mins (exact) into the
//         mins tile and (d, dmin) into dsc: the block's value is
//         d * sum(q sc x) - dmin * sum_j m_j X_j.
//   Q6_K: A = sc * (q - 32) (exact up to 2048 in magnitude, nearest-even
//         above); dsc = (d, 0).
//   Q8_0: A = fp16(q * d * ws) (one rounding); dsc = (1/ws, 0).
template <int QT>
__device__ __forceinline__ void build_a(uint8_t *A, const uint8_t *U, int u, int h, int lane, float ws, float2 *dsc,
                                        uint8_t *Mt) {
    const int g = lane >> 2, c = lane & 3, r0 = 16 * u + g, r1 = r0 + 8;
    if (QT == 4) {
        const uint4 H0 = *reinterpret_cast<const uint4 *>(U + 16 * g);
        const uint4 H1 = *reinterpret_cast<const uint4 *>(U + 16 * g + 128);
        const uint32_t *cw = reinterpret_cast<const uint32_t *>(U + 256);
#pragma unroll
        for (int jj = 0; jj < 2; jj++) {
            const int j = 2 * h + jj;
            int sc0, m0, sc1, m1;
            q4k_scale(H0, j, sc0, m0);
            q4k_scale(H1, j, sc1, m1);
            const uint32_t P = cw[tcode_word(2 * j, lane)], Q = cw[tcode_word(2 * j + 1, lane)];
            put_chunk(A, r0, 4 * jj + c, cvt_nib(P, __float2half2_rn((float)sc0)));
            put_chunk(A, r1, 4 * jj + c, cvt_nib(Q, __float2half2_rn((float)sc1)));
        }
        if (h == 0 && c < 2) {  // lanes c = 0 / 1: the mins rows of r0 / r1
            const uint4 H = c == 0 ? H0 : H1;
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
        const uint4 S0 = *reinterpret_cast<const uint4 *>(U + 16 * g);
        const uint4 S1 = *reinterpret_cast<const uint4 *>(U + 16 * g + 128);
        const uint32_t *lw = reinterpret_cast<const uint32_t *>(U + 288), *hw = reinterpret_cast<const uint32_t *>(U + 288 + 2048);
        const uint32_t w0 = h == 0 ? S0.x : h == 1 ? S0.y : h == 2 ? S0.z : S0.w;  // scales of chunks 4h..4h+3
        const uint32_t w1 = h == 0 ? S1.x : h == 1 ? S1.y : h == 2 ? S1.z : S1.w;
#pragma unroll
        for (int jp2 = 0; jp2 < 2; jp2++) {
            const int j = 4 * h + 2 * jp2;  // even chunk; j + 1 odd
            const uint32_t P0 = lw[tcode_word(j, lane)], P1 = lw[tcode_word(j + 1, lane)];
            const uint32_t H = hw[tcode_word(j >> 1, lane)];
            const uint32_t a0 = (P0 & LO4C) | ((H << 4) & 0x30303030u), a1 = (P1 & LO4C) | (H & 0x30303030u);
            const uint32_t b0 = ((P0 >> 4) & LO4C) | ((H << 2) & 0x30303030u), b1 = ((P1 >> 4) & LO4C) | ((H >> 2) & 0x30303030u);
            const int e0 = 2 * jp2, e1 = e0 + 1;
            const __half2 sg0 = __float2half2_rn((float)(int8_t)((w0 >> (8 * e0)) & 0xFF));
            const __half2 sg1 = __float2half2_rn((float)(int8_t)((w0 >> (8 * e1)) & 0xFF));
            const __half2 sh0 = __float2half2_rn((float)(int8_t)((w1 >> (8 * e0)) & 0xFF));
            const __half2 sh1 = __float2half2_rn((float)(int8_t)((w1 >> (8 * e1)) & 0xFF));
            const uint2 x0 = cvt_byte<32>(a0, sg0), x1 = cvt_byte<32>(a1, sg1);
            const uint2 y0 = cvt_byte<32>(b0, sh0), y1 = cvt_byte<32>(b1, sh1);
            put_chunk(A, r0, 4 * jp2 + c, make_uint4(x0.x, x0.y, x1.x, x1.y));
            put_chunk(A, r1, 4 * jp2 + c, make_uint4(y0.x, y0.y, y1.x, y1.y));
        }
        if (h == 0 && c == 0) {
            dsc[r0] = make_float2(__half2float(*reinterpret_cast<const __half *>(U + 256 + 2 * g)), 0.0f);
            dsc[r1] = make_float2(__half2float(*reinterpret_cast<const __half *>(U + 256 + 2 * g + 16)), 0.0f);
        }
    } else {
        const uint4 H0 = *reinterpret_cast<const uint4 *>(U + 16 * g);
        const uint4 H1 = *reinterpret_cast<const uint4 *>(U + 16 * g + 128);
        const uint4 *cw = reinterpret_cast<const uint4 *>(U + 256);
#pragma unroll
        for (int jj = 0; jj < 2; jj++) {
            const int j = 2 * h + jj, jw = j >> 1;
            const uint4 Aw = cw[j * 32 + lane];
            const uint32_t hw0 = jw == 0 ? H0.x : jw == 1 ? H0.y : jw == 2 ? H0.z : H0.w;
            const uint32_t hw1 = jw == 0 ? H1.x : jw == 1 ? H1.y : jw == 2 ? H1.z : H1.w;
            const float2 f0 = __half22float2(u2h(hw0)), f1 = __half22float2(u2h(hw1));
            const __half2 s0 = __float2half2_rn(((j & 1) ? f0.y : f0.x) * ws);
            const __half2 s1 = __float2half2_rn(((j & 1) ? f1.y : f1.x) * ws);
            const uint2 x0 = cvt_byte<128>(Aw.x ^ 0x80808080u, s0), x1 = cvt_byte<128>(Aw.z ^ 0x80808080u, s0);
            const uint2 y0 = cvt_byte<128>(Aw.y ^ 0x80808080u, s1), y1 = cvt_byte<128>(Aw.w ^ 0x80808080u, s1);
            put_chunk(A, r0, 4 * jj + c, make_uint4(x0.x, x0.y, x1.x, x1.y));
            put_chunk(A, r1, 4 * jj + c, make_uint4(y0.x, y0.y, y1.x, y1.y));
        }
        if (h == 0 && c == 0) dsc[r0] = dsc[r1] = make_float2(1.0f / ws, 0.0f);
    }
}

__device__ __forceinline__ void bulk_copy(uint32_t bar, void *dst, const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     su32(dst)),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Block accumulators -> registers: acc[c] += d * main - 32 dmin * mins.  The
// MMAs run with N = 2 BN (hi rows then lo rows of x), so main and mins are
// column c plus column c + BN; the sums of x enter the mins MMA x 2^-5.
template <int QT, int BN>
__device__ __forceinline__ void block_readout(float (&acc)[BN / 2], uint32_t tmain, uint32_t tmins, float2 dd) {
#pragma unroll
    for (int c0 = 0; c0 < BN / 2; c0 += 16) {
        float v[16], vl[16];
        tmem_ld16(tmain + c0, v);
        tmem_ld16(tmain + BN + c0, vl);
        if (QT == 4) {
            float mv[16], ml[16];
            tmem_ld16(tmins + c0, mv);
            tmem_ld16(tmins + BN + c0, ml);
#pragma unroll
            for (int i = 0; i < 16; i++) acc[c0 + i] += dd.x * (v[i] + vl[i]) - (32.0f * dd.y) * (mv[i] + ml[i]);
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++) acc[c0 + i] += dd.x * (v[i] + vl[i]);
        }
    }
}

// smem: [2 A stages: 16 KB] [4 B stages: Bh BN*128 | Bl BN*128 (arrive pre-swizzled)]
//       [2 mins stages: M 4 KB | Sh BN*32 | Sl BN*32] (Q4_K)
//       [2 raw stages: 8 units] [dsc: 2 x 128 float2]
//       [bars: raw full 0,1; MMA done 0,1; B full 0..3] [tmem slot]
// TMEM: 8 BN columns: block parity p -> main (2 BN) at 4 BN p, mins (2 BN) at 4 BN p + 2 BN.
template <int QT, int BN>
__global__ void __launch_bounds__(TTHR, 1) k_gemm_tiled(GArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    constexpr int UNIT = tunit_bytes(QT), AST = BM * 128, BST = 2 * BN * 128;
    constexpr int NST = QT == 4 ? 4096 + 2 * BN * 32 : 0;
    uint8_t *Bring = smem + 2 * AST;
    uint8_t *mins = Bring + 4 * BST;
    uint8_t *raw = mins + 2 * NST;
    float2 *dsc = reinterpret_cast<float2 *>(raw + 2 * 8 * UNIT);
    uint64_t *bars = reinterpret_cast<uint64_t *>(dsc + 2 * BM);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 8);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rank = a.CL > 1 ? (int)ctarank() : 0;
    const int tile = a.CL > 1 ? (int)clusterid() : (int)blockIdx.x;
    const int m0 = (tile % a.MT) * BM, n0 = (tile / a.MT) * BN, rt0 = m0 / 16;
    const int kb0 = (int)((long long)rank * a.nkb / a.CL), kb1 = (int)((long long)(rank + 1) * a.nkb / a.CL);
    const int nu = kb1 - kb0;            // unit columns of this CTA
    const int nut = min(8, a.RT - rt0);  // unit rows present in this tile
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tslot)), "r"(8 * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        for (int i = 0; i < 8; i++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&bars[i])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_launch_dependents();
    const int nit = 4 * (kb1 - kb0);
    auto issue_b = [&](int j) {  // activation tile of iteration j (k-block 4 kb0 + j, this n-tile): hi and lo
        const uint32_t bar = su32(&bars[4 + (j & 3)]);
        uint8_t *dst = Bring + (j & 3) * BST;
        const size_t off = ((size_t)(4 * kb0 + j) * a.Npad + n0) * BK;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"((uint32_t)BST) : "memory");
        bulk_copy(bar, dst, a.xh + off, BN * 128);
        bulk_copy(bar, dst + BN * 128, a.xl + off, BN * 128);
    };
    auto issue_raw = [&](int i) {  // unit column kb0 + i into raw stage i & 1 (weights only)
        const uint32_t bar = su32(&bars[i & 1]);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"((uint32_t)(nut * UNIT))
                     : "memory");
        for (int u = 0; u < nut; u++)
            bulk_copy(bar, raw + (i & 1) * 8 * UNIT + u * UNIT,
                      a.wt + ((size_t)(rt0 + u) * a.KBU + kb0 + i) * UNIT, UNIT);
    };
    if (tid == 0)
        for (int i = 0; i < 2 && i < nu; i++) issue_raw(i);
    pdl_wait();  // X (prepared by the previous kernel), bias and Y are ready
    if (tid == 0)
        for (int j = 0; j < 2 && j < nit; j++) issue_b(j);
    const uint32_t id = idesc(2 * BN);  // N = 2 BN: the hi tile rows then the lo tile rows
    // readout geometry: TMEM lane quarter (warp % 4), column half (warp / 4)
    const int q = warp & 3, cb = (warp >> 2) * (BN / 2), row = 32 * q + lane;
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + cb;
    float acc[BN / 2];
#pragma unroll
    for (int i = 0; i < BN / 2; i++) acc[i] = 0.0f;
    bool ok = true;
    int it = 0;
    for (int i = 0; i < nu; i++) {
        const uint8_t *R = raw + (i & 1) * 8 * UNIT;
        const int p = i & 1;
        uint8_t *Mt = mins + p * NST, *Sh = Mt + 4096, *Sl = Sh + BN * 32;
        if (ok) ok = bar_wait(su32(&bars[i & 1]), (uint32_t)((i >> 1) & 1));
        for (int h = 0; h < 4; h++, it++) {
            const int s = it & 1;
            uint8_t *A = smem + s * AST, *Bh = Bring + (it & 3) * BST;
            if (it >= 2 && ok) ok = bar_wait(su32(&bars[2 + s]), (uint32_t)(((it - 2) >> 1) & 1));
            // B stage (it + 2) & 3 was last read by the MMAs of it - 2 (done): prefetch
            if (tid == 0 && it + 2 < nit) issue_b(it + 2);
            if (h == 1 && i > 0) {  // the previous block's MMAs are done (waited above): read it out
                const int pp = (i - 1) & 1;
                block_readout<QT, BN>(acc, tq + 4 * BN * pp, tq + 4 * BN * pp + 2 * BN, dsc[pp * BM + row]);
            }
            if (warp < nut) build_a<QT>(A, R + warp * UNIT, warp, h, lane, a.wscale, dsc + p * BM, Mt);
            if (QT == 4 && h == 0)  // sub-block sums of x (x 2^-5), hi and lo, K = 8 (+ 8 zero)
                for (int e = tid; e < BN * 2; e += TTHR) {
                    const int r = e >> 1, kc = e & 1, n = n0 + r;
                    uint4 hv = make_uint4(0u, 0u, 0u, 0u), lv = hv;
                    if (kc == 0 && n < a.N) {
                        const size_t off = (size_t)n * a.K32 + (size_t)(kb0 + i) * 8;
                        hv = __ldg(reinterpret_cast<const uint4 *>(a.xsh + off));
                        lv = __ldg(reinterpret_cast<const uint4 *>(a.xsl + off));
                    }
                    put_core(Sh, r, kc, hv);
                    put_core(Sl, r, kc, lv);
                }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                if (ok) ok = bar_wait(su32(&bars[4 + (it & 3)]), (uint32_t)((it >> 2) & 1));  // B tile landed
                tc_fence_after();
                const uint32_t tmain = tmem + 4 * BN * p;
#pragma unroll
                for (int j = 0; j < BK / 16; j++)  // Bh and Bl are one 2 BN-row tile
                    mma_f16(tmain, sdesc(su32(A) + 32 * j), sdesc(su32(Bh) + 32 * j), id, (h > 0 || j > 0) ? 1u : 0u);
                if (QT == 4 && h == 0)  // Sh and Sl are one 2 BN-row tile
                    mma_f16(tmain + 2 * BN, sdesc_plain(su32(Mt)), sdesc_plain(su32(Sh)), id, 0u);
                mma_commit(su32(&bars[2 + s]));
            }
        }
        // every warp has converted this raw stage (the barrier above): refill it
        if (tid == 0 && i + 2 < nu) issue_raw(i + 2);
    }
    if (it > 0 && ok) ok = bar_wait(su32(&bars[2 + ((it - 1) & 1)]), (uint32_t)(((it - 1) >> 1) & 1));
    if (!ok && tid == 0) {  // bounded drain of the copies still in flight
        for (int i = max(0, nu - 2); i < nu; i++) (void)bar_wait(su32(&bars[i & 1]), (uint32_t)((i >> 1) & 1));
        for (int j = max(0, nit - 4); j < nit; j++) (void)bar_wait(su32(&bars[4 + (j & 3)]), (uint32_t)((j >> 2) & 1));
    }
    tc_fence_after();
    if (nu > 0) {
        const int pp = (nu - 1) & 1;
        block_readout<QT, BN>(acc, tq + 4 * BN * pp, tq + 4 * BN * pp + 2 * BN, dsc[pp * BM + row]);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(8 * BN));
    // epilogue from registers (cluster split: partials added in the leader's shared memory)
    const int m = m0 + row;
    if (a.CL == 1) {
#pragma unroll
        for (int c = 0; c < BN / 2; c++) {
            const int n = n0 + cb + c;
            epi_col(a, n, m, acc[c] * (n < a.N ? a.xinv[n] : 0.0f));
        }
        return;
    }
    // reduce-scatter over the cluster: rank o finishes columns [o W, (o + 1) W),
    // W = BN / CL; every rank stores its partial of them into rank o's
    // buffer slot [source rank][column][row] (plain remote stores), then each
    // rank sums its CL slots
    const int W = BN / a.CL;
    float *buf = reinterpret_cast<float *>(smem);  // [CL][W][128] over the idle stages
    cl_arrive();
    cl_wait();  // every rank is done with its stages
#pragma unroll
    for (int c = 0; c < BN / 2; c++) {
        const int col = cb + c, o = col / W;
        const uint32_t la = su32(&buf[((size_t)rank * W + (col - o * W)) * BM + row]);
        uint32_t ra;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"((uint32_t)o));
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(acc[c]) : "memory");
    }
    cl_arrive();
    cl_wait();  // every slot written
    for (int e = tid; e < W * BM; e += TTHR) {
        const int cc = e / BM, r = e % BM, n = n0 + rank * W + cc, mm = m0 + r;  // cc is warp-uniform
        float v = 0.0f;
        for (int src = 0; src < a.CL; src++) v += buf[((size_t)src * W + cc) * BM + r];
        epi_col(a, n, mm, v * (n < a.N ? a.xinv[n] : 0.0f));
    }
}

// Position of column src (within its 64-column block) in the fast path's
// order: the order cvt_nib / cvt_byte produce (see build_a).
__device__ __forceinline__ int perm_pos(int src) {
    const int w = src & 31, i = w & 3, slot = (w & 16 ? 4 : 0) + (i == 1 ? 2 : i == 2 ? 1 : i);
    return 8 * (4 * (src >> 5) + ((w & 15) >> 2)) + slot;
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
                                                     float *xinv, int perm, __half *xsh, __half *xsl, int N, int Npad) {
    extern __shared__ float row[];  // [K]
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const int n = blockIdx.x, tid = threadIdx.x;
    if (n >= N) {  // fast-path padding rows: zero tiles
        for (int k = tid; k < K; k += blockDim.x) {
            const size_t o = ((size_t)(k >> 6) * Npad + n) * 64 + (k & 63);
            xh[o] = __float2half_rn(0.0f);
            xl[o] = __float2half_rn(0.0f);
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
        if (xsh) {
            const float t = warp_sum(v) * (1.0f / 32.0f);
            if ((tid & 31) == 0) {
                const __half th = __float2half_rn(t);
                xsh[(size_t)n * (K / 32) + k / 32] = th;
                xsl[(size_t)n * (K / 32) + k / 32] = __float2half_rn(t - __half2float(th));
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
static __half *g_xh = NULL, *g_xl = NULL, *g_xsh = NULL, *g_xsl = NULL;
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
    if (g_xsh) cudaFree(g_xsh);
    if (g_xsl) cudaFree(g_xsl);
    g_xsh = g_xsl = NULL;
    if (g_xinv) cudaFree(g_xinv);
    g_xh = g_xl = NULL;
    g_xinv = NULL;
    g_x_cap = 0;
    g_xinv_cap = 0;
    LMC_CUDA_TRY(cudaMalloc(&g_xh, need * sizeof(__half)));
    LMC_CUDA_TRY(cudaMalloc(&g_xl, need * sizeof(__half)));
    LMC_CUDA_TRY(cudaMalloc(&g_xsh, (need / 32 + 8) * sizeof(__half)));
    LMC_CUDA_TRY(cudaMalloc(&g_xsl, (need / 32 + 8) * sizeof(__half)));
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
               fast && t->type == LMC_TYPE_Q4_K ? g_xsh : (__half *)NULL,
               fast && t->type == LMC_TYPE_Q4_K ? g_xsl : (__half *)NULL, N, Npad);
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
    a.xsh = g_xsh;
    a.xsl = g_xsl;
    a.K32 = K / 32;
    a.Npad = Npad;
    const void *fn = NULL;
    size_t smem;
    int nthr, min_kb;
    if (fast) {
        const int qt = t->type == LMC_TYPE_Q4_K ? 4 : t->type == LMC_TYPE_Q6_K ? 6 : 8;
        a.BN = 64;
        a.nkb = K / 256;
        smem = 2 * (size_t)BM * 128 + 4 * (size_t)(2 * a.BN * 128) + (qt == 4 ? 2 * (size_t)(4096 + 2 * a.BN * 32) : 0) +
               2 * 8 * (size_t)tunit_bytes(qt) + 2 * BM * 8 + 128 + 1024;
        fn = qt == 4 ? (const void *)k_gemm_tiled<4, 64> : qt == 6 ? (const void *)k_gemm_tiled<6, 64>
                                                                 : (const void *)k_gemm_tiled<8, 64>;
        nthr = TTHR;
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
