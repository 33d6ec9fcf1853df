// tiled_gemv.cu - K2 (tensor-core): dequant-GEMV for Q4_K and Q6_K on a
// row-tiled copy of the GGUF blocks, with mma.sync m16n8k16 (f16 x f16 ->
// f32).  Replaces LMc matmul_vec (src/ops.c:69-97) over dequant_q4k /
// dequant_q6k (src/quant.c:275-303, :386-414) for the decode batch sizes.
//
// Why tensor cores for a GEMV: at HBM speed an SM receives ~23 bytes/clock,
// i.e. ~45 Q4_K weights/clock; unpacking each weight to fp32 and FMA-ing it
// costs 3-4 CUDA-core instructions, which caps a CUDA-core kernel below the
// HBM roofline.  Here the weight codes go into the A operand as exact small
// integers in fp16, the activations into B split into hi + lo fp16 halves
// (x = hi + lo to ~2^-22), and the products accumulate in fp32 - so the
// result carries fp32 accuracy while one MMA does 2 x 256 multiply-adds.
//
// Layout ("unit" = 16 rows x 256 columns, units stored row-tile major):
//   Q4_K unit (2304 B = 16 x 144):  [16 rows x 16 B header: d, dmin, 12 B
//     packed scales (verbatim from the block)] [32 lanes x 64 B codes]; lane
//     (g = lane/4, c = lane%4) holds, for each of the 16 k-chunks j, one u32
//     with the 8 nibbles of its A fragment: rows g and g+8, k = 16j + 2c,
//     2c+1, 2c+8, 2c+9, arranged so that (u & 0x000F000F), (u & 0x00F000F0),
//     (u>>8 & ...) drop straight into fp16 mantissas.
//   Q6_K unit (3360 B = 16 x 210):  [16 rows x 16 int8 scales] [16 rows x
//     fp16 d] [32 lanes x 64 B low nibbles, same arrangement as Q4_K]
//     [32 lanes x 32 B high 2-bit pairs: one u16 per chunk].
// The bytes are the GGUF bytes rearranged (same count per weight), so the
// algorithmic traffic is unchanged.  Needs cols % 256 == 0; other shapes and
// formats use the generic kernel.
#include <cuda_fp16.h>

#include "lmc_blocks.cuh"
#include "lmc_common.cuh"
#include "lmc_internal.h"

#include <algorithm>

namespace {

constexpr int MAX_WARPS = 16;
constexpr int PF_UNITS = 4;  // L2 prefetch distance, in units of the warp's own sequence
constexpr int Q4K_UNIT = 2304, Q6K_UNIT = 3360;
constexpr int SMEM_LIMIT = 200 * 1024;

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t m, uint32_t o) {
    uint32_t d;  // (a & m) | o
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(m), "r"(o));
    return d;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                    uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint4 ld_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}
// fp16 constants
constexpr uint32_t H1024 = 0x64006400u, HNEG1024 = 0xE400E400u, HSIXTEENTH = 0x2C002C00u, HNEG64 = 0xD400D400u;
constexpr uint32_t H1056 = 0x64206420u;  // 1024 + 32
constexpr uint32_t HNEG96 = 0xD600D600u;  // -96

// {v, v} as exact fp16 for a byte v < 256 (byte i of w): mantissa trick.
__device__ __forceinline__ uint32_t byte_pair_h2(uint32_t w, int i0, int i1) {
    return hsub2(__byte_perm(w, 0x64u, (uint32_t)(i0 | (4 << 4) | (i1 << 8) | (4 << 12))), H1024);
}

// ---------------------------------------------------------------------------
// repack kernels (upload time)
// ---------------------------------------------------------------------------
// nibble / 6-bit code of element k (0..255) of a Q4_K / Q6_K block
__device__ __forceinline__ uint32_t q4k_code(const uint8_t *blk, int k) {
    const int g = k >> 6, w = k & 63;
    const uint32_t b = blk[16 + 32 * g + (w & 31)];
    return (w & 32) ? (b >> 4) : (b & 15);
}
__device__ __forceinline__ uint32_t q6k_code(const uint8_t *blk, int k) {
    const int p = k >> 7, r = k & 127, kk = r >> 5, l = r & 31;
    const uint32_t lo = (blk[64 * p + ((kk & 1) ? 32 : 0) + l] >> ((kk >> 1) * 4)) & 15;
    const uint32_t hi = (blk[128 + 32 * p + l] >> (2 * kk)) & 3;
    return lo | (hi << 4);
}

// u32 of the 8 A-fragment codes for lane (g, c), chunk j: bit layout
// nib0 = (g, 2c), nib1 = (g+8, 2c), nib2 = (g, 2c+8), nib3 = (g+8, 2c+8),
// nib4..7 = the same with k+1.
template <typename CODE>
__device__ __forceinline__ void frag_codes(CODE code, const uint8_t *b_g, const uint8_t *b_g8, int j, int c,
                                           uint32_t *lo_u32, uint32_t *hi_u16) {
    const int k0 = 16 * j + 2 * c;
    const int ks[8] = {k0, k0, k0 + 8, k0 + 8, k0 + 1, k0 + 1, k0 + 9, k0 + 9};
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint8_t *b = (i & 1) ? b_g8 : b_g;
        const uint32_t v = b ? code(b, ks[i]) : 0u;
        lo |= (v & 15u) << (4 * i);
        hi |= ((v >> 4) & 3u) << (2 * i);
    }
    *lo_u32 = lo;
    if (hi_u16) *hi_u16 = hi;
}

__global__ void k_repack_q4k(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int M, int KB, int RT) {
    const int unit = blockIdx.x;  // rt * KB + kb
    const int rt = unit / KB, kb = unit % KB, t = threadIdx.x;
    uint8_t *u = dst + (size_t)unit * Q4K_UNIT;
    if (t < 16) {  // header of row t
        const int r = rt * 16 + t;
        for (int i = 0; i < 16; i++) u[16 * t + i] = r < M ? src[((size_t)r * KB + kb) * 144 + i] : 0;
    }
    if (t < 32) {
        const int g = t >> 2, c = t & 3;
        const int r0 = rt * 16 + g, r1 = r0 + 8;
        const uint8_t *b0 = r0 < M ? src + ((size_t)r0 * KB + kb) * 144 : nullptr;
        const uint8_t *b1 = r1 < M ? src + ((size_t)r1 * KB + kb) * 144 : nullptr;
        uint32_t *o = reinterpret_cast<uint32_t *>(u + 256 + 64 * t);
        for (int j = 0; j < 16; j++) {
            uint32_t lo;
            frag_codes(q4k_code, b0, b1, j, c, &lo, nullptr);
            o[j] = lo;
        }
    }
}

__global__ void k_repack_q6k(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int M, int KB, int RT) {
    const int unit = blockIdx.x;
    const int rt = unit / KB, kb = unit % KB, t = threadIdx.x;
    uint8_t *u = dst + (size_t)unit * Q6K_UNIT;
    if (t < 16) {  // header: 16 rows x 16 int8 scales, then 16 rows x fp16 d
        const int r = rt * 16 + t;
        const uint8_t *b = r < M ? src + ((size_t)r * KB + kb) * 210 : nullptr;
        for (int i = 0; i < 16; i++) u[16 * t + i] = b ? b[192 + i] : 0;
        u[256 + 2 * t] = b ? b[208] : 0;
        u[256 + 2 * t + 1] = b ? b[209] : 0;
    }
    if (t < 32) {
        const int g = t >> 2, c = t & 3;
        const int r0 = rt * 16 + g, r1 = r0 + 8;
        const uint8_t *b0 = r0 < M ? src + ((size_t)r0 * KB + kb) * 210 : nullptr;
        const uint8_t *b1 = r1 < M ? src + ((size_t)r1 * KB + kb) * 210 : nullptr;
        uint32_t *o = reinterpret_cast<uint32_t *>(u + 288 + 64 * t);
        uint16_t *oh = reinterpret_cast<uint16_t *>(u + 288 + 2048 + 32 * t);
        for (int j = 0; j < 16; j++) {
            uint32_t lo, hi;
            frag_codes(q6k_code, b0, b1, j, c, &lo, &hi);
            o[j] = lo;
            oh[j] = (uint16_t)hi;
        }
    }
}

// ---------------------------------------------------------------------------
// activation fragments (per CTA, in shared memory)
// ---------------------------------------------------------------------------
// xf[kb][j][nt][lane] = B fragment (2 x f16x2) of chunk j: column n = 8nt + g
// is the hi (n even) or lo (n odd) fp16 part of x[n/2]; rows k = 16j + 2c,
// +1 (reg 0) and +8, +9 (reg 1).
// xs[kb][nt][lane] = B fragment of the per-32 sums used by the Q4_K min term
// (rows = sub-block index 2c, 2c+1; rows 8..15 are zero).
__device__ __forceinline__ float hi_lo(float v, int part) {
    const float h = __half2float(__float2half_rn(v));
    return part ? (v - h) : h;
}

template <int NT>
__device__ void build_xfrags(uint2 *xf, uint32_t *xs, float *xsum_tmp, const float *__restrict__ x, int ldx, int nb,
                             int KB, bool want_sums) {
    const int n_entries = KB * 16 * NT * 32;
    for (int e = threadIdx.x; e < n_entries; e += blockDim.x) {
        const int lane = e & 31, nt = (e >> 5) % NT, j = (e / (32 * NT)) & 15, kb = e / (32 * NT * 16);
        const int g = lane >> 2, c = lane & 3, n = nt * 8 + g, b = n >> 1, part = n & 1;
        uint2 r = make_uint2(0u, 0u);
        if (b < nb) {
            const float2 *xb = reinterpret_cast<const float2 *>(x + (size_t)b * ldx + kb * 256 + 16 * j + 2 * c);
            const float2 p0 = xb[0], p1 = xb[4];
            r.x = pack_h2(hi_lo(p0.x, part), hi_lo(p0.y, part));
            r.y = pack_h2(hi_lo(p1.x, part), hi_lo(p1.y, part));
        }
        xf[e] = r;
    }
    if (!want_sums) return;
    // per-32 sums of x, one warp per (kb, sub, b): xsum_tmp[(kb*8 + sub)*nb + b]
    const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int e = threadIdx.x >> 5; e < KB * 8 * nb; e += nw) {
        const int b = e % nb, sub = (e / nb) & 7, kb = e / (nb * 8);
        const float v = warp_sum(x[(size_t)b * ldx + kb * 256 + 32 * sub + lane]);
        if (lane == 0) xsum_tmp[e] = v;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < KB * NT * 32; e += blockDim.x) {
        const int ln = e & 31, nt = (e >> 5) % NT, kb = e / (32 * NT);
        const int g = ln >> 2, c = ln & 3, n = nt * 8 + g, b = n >> 1, part = n & 1;
        uint32_t r = 0u;
        if (b < nb)
            r = pack_h2(hi_lo(xsum_tmp[(kb * 8 + 2 * c) * nb + b], part),
                        hi_lo(xsum_tmp[(kb * 8 + 2 * c + 1) * nb + b], part));
        xs[e] = r;
    }
}

// ---------------------------------------------------------------------------
// the GEMV kernels: persistent CTAs, each owning `rpc` row tiles at a time;
// the `ksplit` warps of a row tile take every ksplit-th 256-column unit and
// their partial sums meet in shared memory.
// ---------------------------------------------------------------------------
struct TArgs {
    const uint8_t *w;
    const float *x, *bias;
    float *y;
    int M, KB, RT, ldx, ldy, nb, epi, ksplit, rpc, ngroups;
};

// The sequence of units one warp processes: row-tile groups grp = blockIdx.x,
// blockIdx.x + gridDim.x, ...; inside a group, units kb = ks, ks + ksplit, ...
struct UnitIter {
    int grp, kb;
    __device__ __forceinline__ bool valid(const TArgs &a, int rt_local) const {
        return grp < a.ngroups && grp * a.rpc + rt_local < a.RT;
    }
    __device__ __forceinline__ void next(const TArgs &a, int ks) {
        kb += a.ksplit;
        if (kb >= a.KB) { kb = ks; grp += gridDim.x; }
    }
};

// Issue L2 prefetches for the first PF_UNITS units of this warp (one lane
// each) - used before pdl_wait(), so the weight stream of this kernel starts
// while the previous kernel of the step is still running.
__device__ __forceinline__ UnitIter prefetch_head(const TArgs &a, int rt_local, int ks, int lane, int unit_bytes) {
    UnitIter it{(int)blockIdx.x, ks};
    if (ks >= a.KB) { it.grp = a.ngroups; return it; }
    for (int i = 0; i < PF_UNITS && it.valid(a, rt_local); i++) {
        if (lane == i)
            prefetch_l2(a.w + ((size_t)(it.grp * a.rpc + rt_local) * a.KB + it.kb) * unit_bytes, unit_bytes);
        it.next(a, ks);
    }
    return it;
}

template <int NT>
__device__ __forceinline__ void finish(const TArgs &a, float (&tot)[NT][4], float *red, int rt, int ks, int lane) {
    const int wid = threadIdx.x >> 5;
    if (a.ksplit > 1) {
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) red[((wid * NT + nt) * 4 + i) * 32 + lane] = tot[nt][i];
    }
    __syncthreads();
    if (ks == 0 && rt < a.RT) {
        for (int s = 1; s < a.ksplit; s++) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int i = 0; i < 4; i++) tot[nt][i] += red[(((wid + s) * NT + nt) * 4 + i) * 32 + lane];
        }
        const int g = lane >> 2, c = lane & 3;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int b = nt * 4 + c;
            if (b >= a.nb) continue;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int row = rt * 16 + g + 8 * h;
                if (row >= a.M) continue;
                float v = tot[nt][2 * h] + tot[nt][2 * h + 1];  // hi + lo halves of x
                if (a.bias) v += a.bias[row];
                if (a.epi & LMC_EPI_GELU) v = lmc_gelu_f(v);
                float *o = a.y + (size_t)b * a.ldy + row;
                *o = (a.epi & LMC_EPI_ACCUM) ? *o + v : v;
            }
        }
    }
    __syncthreads();  // `red` is reused by the next row-tile group
}

// Q4_K (src/quant.c:275-303): y = sum_units d * sum_k (sc*q) x - dmin * sum_sub m * X_sub
template <int NT>
__global__ void __launch_bounds__(MAX_WARPS * 32) k_gemv_q4k(TArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint2 *xf = reinterpret_cast<uint2 *>(smem);
    uint32_t *xs = reinterpret_cast<uint32_t *>(xf + a.KB * 16 * NT * 32);
    float *tmp = reinterpret_cast<float *>(xs + a.KB * NT * 32);  // x sums, later the reduction area
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int rt_local = wid / a.ksplit, ks = wid % a.ksplit;
    const int g = lane >> 2, c = lane & 3;
    pdl_launch_dependents();
    UnitIter pf = prefetch_head(a, rt_local, ks, lane, Q4K_UNIT);  // weights only: before the wait
    pdl_wait();
    build_xfrags<NT>(xf, xs, tmp, a.x, a.ldx, a.nb, a.KB, true);
    __syncthreads();
    for (int grp = blockIdx.x; grp < a.ngroups; grp += gridDim.x) {
        const int rt = grp * a.rpc + rt_local;
        float tot[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) tot[nt][i] = 0.0f;
        if (rt < a.RT && ks < a.KB) {
            const uint8_t *base = a.w + (size_t)rt * a.KB * Q4K_UNIT;
            uint4 h0, h1, q0, q1, q2, q3;
            {
                const uint8_t *u = base + (size_t)ks * Q4K_UNIT;
                h0 = __ldg(reinterpret_cast<const uint4 *>(u + 16 * g));
                h1 = __ldg(reinterpret_cast<const uint4 *>(u + 16 * (g + 8)));
                const uint8_t *q = u + 256 + 64 * lane;
                q0 = ld_stream(q); q1 = ld_stream(q + 16); q2 = ld_stream(q + 32); q3 = ld_stream(q + 48);
            }
            for (int kb = ks; kb < a.KB; kb += a.ksplit) {
                if (pf.valid(a, rt_local)) {  // keep PF_UNITS units of this warp in flight to L2
                    if (lane == 0)
                        prefetch_l2(a.w + ((size_t)(pf.grp * a.rpc + rt_local) * a.KB + pf.kb) * Q4K_UNIT, Q4K_UNIT);
                    pf.next(a, ks);
                }
                const uint4 H0 = h0, H1 = h1;
                const uint32_t qs[16] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w,
                                         q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
                const int nk = kb + a.ksplit;
                if (nk < a.KB) {  // prefetch the next unit
                    const uint8_t *u = base + (size_t)nk * Q4K_UNIT;
                    h0 = __ldg(reinterpret_cast<const uint4 *>(u + 16 * g));
                    h1 = __ldg(reinterpret_cast<const uint4 *>(u + 16 * (g + 8)));
                    const uint8_t *q = u + 256 + 64 * lane;
                    q0 = ld_stream(q); q1 = ld_stream(q + 16); q2 = ld_stream(q + 32); q3 = ld_stream(q + 48);
                }
                // 6-bit scales / mins of rows g and g+8, four at a time (src/quant.c:44-53)
                const uint32_t sc0a = H0.y & 0x3F3F3F3Fu, sc0b = (H0.w & 0x0F0F0F0Fu) | ((H0.y >> 2) & 0x30303030u);
                const uint32_t sc1a = H1.y & 0x3F3F3F3Fu, sc1b = (H1.w & 0x0F0F0F0Fu) | ((H1.y >> 2) & 0x30303030u);
                const uint32_t m0a = H0.z & 0x3F3F3F3Fu, m0b = ((H0.w >> 4) & 0x0F0F0F0Fu) | ((H0.z >> 2) & 0x30303030u);
                const uint32_t m1a = H1.z & 0x3F3F3F3Fu, m1b = ((H1.w >> 4) & 0x0F0F0F0Fu) | ((H1.z >> 2) & 0x30303030u);
                float acc[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
#pragma unroll
                    for (int i = 0; i < 4; i++) acc[nt][i] = 0.0f;
                const uint2 *xk = xf + (size_t)(kb * 16) * NT * 32 + lane;
#pragma unroll
                for (int sb = 0; sb < 8; sb++) {
                    const uint32_t w0 = sb < 4 ? sc0a : sc0b, w1 = sb < 4 ? sc1a : sc1b;
                    const uint32_t s0 = byte_pair_h2(w0, sb & 3, sb & 3);  // {sc, sc} row g
                    const uint32_t s1 = byte_pair_h2(w1, sb & 3, sb & 3);  // {sc, sc} row g+8
                    const uint32_t b0 = s0, c0 = hmul2(s0, HNEG1024);
                    const uint32_t b1 = hmul2(s1, HSIXTEENTH), c1 = hmul2(s1, HNEG64);
#pragma unroll
                    for (int jj = 0; jj < 2; jj++) {
                        const int j = 2 * sb + jj;
                        const uint32_t u = qs[j], u8 = u >> 8;
                        // A = q * sc, exact: (1024 + q)*sc - 1024*sc, (1024 + 16q)*sc/16 - 64*sc
                        const uint32_t a0 = hfma2(lop_and_or(u, 0x000F000Fu, H1024), b0, c0);
                        const uint32_t a1 = hfma2(lop_and_or(u, 0x00F000F0u, H1024), b1, c1);
                        const uint32_t a2 = hfma2(lop_and_or(u8, 0x000F000Fu, H1024), b0, c0);
                        const uint32_t a3 = hfma2(lop_and_or(u8, 0x00F000F0u, H1024), b1, c1);
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            const uint2 bx = xk[(j * NT + nt) * 32];
                            mma(acc[nt], a0, a1, a2, a3, bx.x, bx.y);
                        }
                    }
                }
                // min term: rows g / g+8, sub-blocks 2c, 2c+1 (k rows 8..15 zero)
                const uint32_t mw0 = c < 2 ? m0a : m0b, mw1 = c < 2 ? m1a : m1b;
                const int i0 = (2 * c) & 3, i1 = (2 * c + 1) & 3;
                const uint32_t am0 = byte_pair_h2(mw0, i0, i1), am1 = byte_pair_h2(mw1, i0, i1);
                const float2 dd0 = __half22float2(*reinterpret_cast<const __half2 *>(&H0.x));
                const float2 dd1 = __half22float2(*reinterpret_cast<const __half2 *>(&H1.x));
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    float accm[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    mma(accm, am0, am1, 0u, 0u, xs[(kb * NT + nt) * 32 + lane], 0u);
                    tot[nt][0] += dd0.x * acc[nt][0] - dd0.y * accm[0];
                    tot[nt][1] += dd0.x * acc[nt][1] - dd0.y * accm[1];
                    tot[nt][2] += dd1.x * acc[nt][2] - dd1.y * accm[2];
                    tot[nt][3] += dd1.x * acc[nt][3] - dd1.y * accm[3];
                }
            }
        }
        finish<NT>(a, tot, tmp, rt, ks, lane);
    }
}

// int8 byte i of w as an exact float: (2^23 + 128 + b) - (2^23 + 128)
__device__ __forceinline__ float s8_to_f(uint32_t w, int i) {
    const uint32_t v = __byte_perm(w, 0x4Bu, (uint32_t)(i | (5 << 4) | (5 << 8) | (4 << 12))) ^ 0x80u;
    return __uint_as_float(v) - 8388736.0f;
}

// Q6_K (src/quant.c:386-414): y = sum_units sum_chunks (d*sc) * sum_16 (q-32) x
template <int NT>
__global__ void __launch_bounds__(MAX_WARPS * 32) k_gemv_q6k(TArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint2 *xf = reinterpret_cast<uint2 *>(smem);
    float *tmp = reinterpret_cast<float *>(xf + a.KB * 16 * NT * 32);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int rt_local = wid / a.ksplit, ks = wid % a.ksplit;
    const int g = lane >> 2;
    pdl_launch_dependents();
    UnitIter pf = prefetch_head(a, rt_local, ks, lane, Q6K_UNIT);  // weights only: before the wait
    pdl_wait();
    build_xfrags<NT>(xf, nullptr, nullptr, a.x, a.ldx, a.nb, a.KB, false);
    __syncthreads();
    for (int grp = blockIdx.x; grp < a.ngroups; grp += gridDim.x) {
        const int rt = grp * a.rpc + rt_local;
        float tot[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) tot[nt][i] = 0.0f;
        if (rt < a.RT && ks < a.KB) {
            const uint8_t *base = a.w + (size_t)rt * a.KB * Q6K_UNIT;
            uint4 s0v, s1v, q0, q1, q2, q3, hq0, hq1;
            uint32_t dw;
            auto load = [&](int kb) {
                const uint8_t *u = base + (size_t)kb * Q6K_UNIT;
                s0v = __ldg(reinterpret_cast<const uint4 *>(u + 16 * g));
                s1v = __ldg(reinterpret_cast<const uint4 *>(u + 16 * (g + 8)));
                dw = (uint32_t)__ldg(reinterpret_cast<const unsigned short *>(u + 256 + 2 * g)) |
                     ((uint32_t)__ldg(reinterpret_cast<const unsigned short *>(u + 256 + 2 * (g + 8))) << 16);
                const uint8_t *q = u + 288 + 64 * lane;
                q0 = ld_stream(q); q1 = ld_stream(q + 16); q2 = ld_stream(q + 32); q3 = ld_stream(q + 48);
                hq0 = ld_stream(u + 288 + 2048 + 32 * lane);
                hq1 = ld_stream(u + 288 + 2048 + 32 * lane + 16);
            };
            load(ks);
            for (int kb = ks; kb < a.KB; kb += a.ksplit) {
                if (pf.valid(a, rt_local)) {  // keep PF_UNITS units of this warp in flight to L2
                    if (lane == 0)
                        prefetch_l2(a.w + ((size_t)(pf.grp * a.rpc + rt_local) * a.KB + pf.kb) * Q6K_UNIT, Q6K_UNIT);
                    pf.next(a, ks);
                }
                const uint32_t qs[16] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w,
                                         q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
                const uint32_t hs[8] = {hq0.x, hq0.y, hq0.z, hq0.w, hq1.x, hq1.y, hq1.z, hq1.w};
                const uint32_t sw0[4] = {s0v.x, s0v.y, s0v.z, s0v.w}, sw1[4] = {s1v.x, s1v.y, s1v.z, s1v.w};
                const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&dw));
                if (kb + a.ksplit < a.KB) load(kb + a.ksplit);  // prefetch the next unit
                const uint2 *xk = xf + (size_t)(kb * 16) * NT * 32 + lane;
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float s0 = dd.x * s8_to_f(sw0[j >> 2], j & 3);  // d * sc, as LMc (quant.c:407)
                    const float s1 = dd.y * s8_to_f(sw1[j >> 2], j & 3);
                    const uint32_t u4 = qs[j], u8 = u4 >> 8;
                    const uint32_t hb = (hs[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
                    // high 2 bits of nibble i sit at bits 2i..2i+1 of hb; move them to
                    // mantissa bits 4-5 (plain fields) or 8-9 (x16 fields)
                    const uint32_t h_a0 = ((hb & 0x3u) << 4) | ((hb & 0x300u) << 12);
                    const uint32_t h_a1 = ((hb & 0xCu) << 6) | ((hb & 0xC00u) << 14);
                    const uint32_t h_a2 = (hb & 0x30u) | ((hb & 0x3000u) << 8);
                    const uint32_t h_a3 = ((hb & 0xC0u) << 2) | ((hb & 0xC000u) << 10);
                    const uint32_t v0 = lop_and_or(u4, 0x000F000Fu, H1024) | h_a0;  // 1024 + q
                    const uint32_t v1 = lop_and_or(u4, 0x00F000F0u, H1024) | h_a1;  // 1024 + 16q
                    const uint32_t v2 = lop_and_or(u8, 0x000F000Fu, H1024) | h_a2;
                    const uint32_t v3 = lop_and_or(u8, 0x00F000F0u, H1024) | h_a3;
                    const uint32_t a0 = hsub2(v0, H1056);              // q - 32
                    const uint32_t a1 = hfma2(v1, HSIXTEENTH, HNEG96);  // (1024+16q)/16 - 96 = q - 32
                    const uint32_t a2 = hsub2(v2, H1056);
                    const uint32_t a3 = hfma2(v3, HSIXTEENTH, HNEG96);
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
                        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        const uint2 bx = xk[(j * NT + nt) * 32];
                        mma(acc, a0, a1, a2, a3, bx.x, bx.y);
                        tot[nt][0] += s0 * acc[0];
                        tot[nt][1] += s0 * acc[1];
                        tot[nt][2] += s1 * acc[2];
                        tot[nt][3] += s1 * acc[3];
                    }
                }
            }
        }
        finish<NT>(a, tot, tmp, rt, ks, lane);
    }
}

size_t smem_bytes(uint32_t type, int KB, int NT, int warps) {
    size_t xf = (size_t)KB * 16 * NT * 32 * sizeof(uint2);
    size_t xs = type == LMC_TYPE_Q4_K ? (size_t)KB * NT * 32 * 4 : 0;
    size_t red = (size_t)warps * NT * 4 * 32 * 4;
    size_t sums = type == LMC_TYPE_Q4_K ? (size_t)KB * 8 * 4 * NT * 4 : 0;
    return xf + xs + std::max(red, sums);
}

void plan(int KB, int *ksplit, int *rpc) {
    *ksplit = std::min(KB, MAX_WARPS);
    *rpc = std::max(1, MAX_WARPS / *ksplit);
}

}  // namespace

extern "C" int lmc_tiled_build(lmc_qtensor *t) {
    t->tiled = NULL;
    if ((t->type != LMC_TYPE_Q4_K && t->type != LMC_TYPE_Q6_K) || t->cols % 256) return LMC_OK;
    const int KB = t->cols / 256, RT = (t->rows + 15) / 16;
    if (smem_bytes(t->type, KB, 1, MAX_WARPS) > SMEM_LIMIT) return LMC_OK;  // very long rows: generic path
    const size_t unit = t->type == LMC_TYPE_Q4_K ? Q4K_UNIT : Q6K_UNIT;
    const size_t bytes = (size_t)RT * KB * unit;
    LMC_CUDA_TRY(cudaMalloc(&t->tiled, bytes));
    if (t->type == LMC_TYPE_Q4_K)
        k_repack_q4k<<<RT * KB, 32>>>((const uint8_t *)t->blocks, (uint8_t *)t->tiled, t->rows, KB, RT);
    else
        k_repack_q6k<<<RT * KB, 32>>>((const uint8_t *)t->blocks, (uint8_t *)t->tiled, t->rows, KB, RT);
    LMC_LAUNCH_CHECK("repack");
    LMC_CUDA_TRY(cudaDeviceSynchronize());
    t->tiled_bytes = bytes;
    t->tiled_rows = RT * 16;
    return LMC_OK;
}

template <int NT>
static int launch_nt(const lmc_qtensor *t, TArgs a, cudaStream_t s) {
    const int threads = a.ksplit * a.rpc * 32;
    const size_t smem = smem_bytes(t->type, a.KB, NT, threads / 32);
    if (smem > SMEM_LIMIT) return LMC_ERR_UNSUPPORTED;
    const void *fn = t->type == LMC_TYPE_Q4_K ? (const void *)k_gemv_q4k<NT> : (const void *)k_gemv_q6k<NT>;
    LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    LMC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem));
    const int grid = std::max(1, std::min(a.ngroups, std::max(per_sm, 1) * lmc_sm_count()));
    if (t->type == LMC_TYPE_Q4_K)
        LMC_LAUNCH("tiled gemv q4k", k_gemv_q4k<NT>, grid, threads, smem, s, a);
    else
        LMC_LAUNCH("tiled gemv q6k", k_gemv_q6k<NT>, grid, threads, smem, s, a);
    return LMC_OK;
}

extern "C" int lmc_tiled_gemv_launch(const lmc_qtensor *t, const float *d_x, int ldx, const float *d_bias, float *d_y,
                                     int ldy, int batch, int epi, cudaStream_t s) {
    if (((uintptr_t)d_x & 7) || (ldx & 1))  // float2 fragment loads
        return lmc_gemv_generic_launch(t->type, t->blocks, t->rows, t->cols, d_x, ldx, d_bias, d_y, ldy, batch, epi, s);
    TArgs a;
    a.w = (const uint8_t *)t->tiled;
    a.bias = d_bias;
    a.M = t->rows;
    a.KB = t->cols / 256;
    a.RT = t->tiled_rows / 16;
    a.ldx = ldx;
    a.ldy = ldy;
    a.epi = epi;
    plan(a.KB, &a.ksplit, &a.rpc);
    a.ngroups = (a.RT + a.rpc - 1) / a.rpc;
    for (int b0 = 0; b0 < batch;) {
        const int nb = std::min(batch - b0, 8);
        a.x = d_x + (size_t)b0 * ldx;
        a.y = d_y + (size_t)b0 * ldy;
        int rc;
        a.nb = nb;
        if (nb <= 4) {
            rc = launch_nt<1>(t, a, s);
        } else {
            rc = launch_nt<2>(t, a, s);
            if (rc == LMC_ERR_UNSUPPORTED) {  // not enough shared memory for 2 n-tiles: two passes of 4
                a.nb = 4;
                rc = launch_nt<1>(t, a, s);
                if (!rc) {
                    TArgs a2 = a;
                    a2.x += (size_t)4 * ldx;
                    a2.y += (size_t)4 * ldy;
                    a2.nb = nb - 4;
                    rc = launch_nt<1>(t, a2, s);
                }
            }
        }
        if (rc == LMC_ERR_UNSUPPORTED)
            return lmc_set_error(rc, "tiled gemv: %d columns need too much shared memory", t->cols);
        if (rc) return rc;
        b0 += nb;
    }
    return LMC_OK;
}
