// tiled_gemv.cu - K2 (tensor-core): dequant-GEMV for Q4_K and Q6_K on a
// row-tiled copy of the GGUF blocks, on the integer tensor cores
// (mma.sync s8 x s8 -> s32).  Replaces LMc matmul_vec (src/ops.c:69-97) over
// dequant_q4k / dequant_q6k (src/quant.c:275-303, :386-414) at decode batch
// sizes.
//
// Why integer MMA for a GEMV: at HBM speed an SM receives ~23 bytes/clock
// (~45 Q4_K weights).  Unpacking each weight to fp32 and FMA-ing it costs 3-4
// CUDA-core instructions, and even an fp16 MMA path needs ~2 instructions per
// 8 weights to build fp16 operands.  Here a weight code is already the int8
// operand: one LOP3 turns 8 packed nibbles into 4 int8 lanes, and one
// mma.m16n8k32 does 512 multiply-adds.  The activations enter as three int8
// limbs of a 23-bit fixed-point copy (x ~= 2^-s (L0 + 2^8 L1 + 2^16 L2), one
// exponent s per vector, so the error is <= 2^-23 max|x|); products and sums
// are exact in int32 until the per-block scales are applied in fp32.
//
// Layout ("unit" = 16 rows x 256 columns, units stored row-tile major; the
// bytes are the GGUF bytes rearranged, so the traffic per weight is the
// GGUF traffic):
//   Q4_K unit 2304 B = [16 rows x 16 B block header: d, dmin, 12 B packed
//     scales, verbatim] [32 lanes x 64 B codes].  Lane (g = lane/4, c = lane%4)
//     holds, for each 32-column sub-block j, u32 P_j (row g) and Q_j (row g+8):
//     byte i = code(k = 32j + 4c + i) | code(k = 32j + 16 + 4c + i) << 4, so
//     P & 0x0F0F0F0F and (P >> 4) & 0x0F0F0F0F are the a0 / a2 registers of the
//     m16n8k32 A fragment.
//   Q6_K unit 3360 B = [16 rows x 16 int8 scales] [16 rows x fp16 d]
//     [32 lanes x 64 B low nibbles: per 16-column chunk j one u32, byte i =
//     lo(g, k) | lo(g+8, k) << 4, k = 16j + 4c + i] [32 lanes x 32 B high bits:
//     per chunk pair one u32, byte i = hi(g, k) | hi(g+8, k) << 2 | hi(g, k+16)
//     << 4 | hi(g+8, k+16) << 6].  The code q = lo | hi << 4 (0..63) is the int8
//     operand; the -32 offset is applied once per chunk through per-16 sums of x.
// Needs cols % 256 == 0; other shapes and formats use the generic kernel.
#include <cuda_fp16.h>

#include "lmc_blocks.cuh"
#include "lmc_common.cuh"
#include "lmc_internal.h"

#include <algorithm>
#include <math.h>

namespace {

constexpr int Q4K_UNIT = 2304, Q6K_UNIT = 3360;
constexpr int SMEM_LIMIT = 200 * 1024;
constexpr uint32_t LO4 = 0x0F0F0F0Fu;

__device__ __forceinline__ void imma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void imma_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}
__device__ __forceinline__ int ubyte(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xFFu); }
__device__ __forceinline__ int sbyte(uint32_t w, int i) { return (int)(int8_t)((w >> (8 * i)) & 0xFFu); }

// ---------------------------------------------------------------------------
// repack kernels (upload time)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t q4k_code(const uint8_t *blk, int k) {  // src/quant.c:293
    const int g = k >> 6, w = k & 63;
    const uint32_t b = blk[16 + 32 * g + (w & 31)];
    return (w & 32) ? (b >> 4) : (b & 15);
}
__device__ __forceinline__ uint32_t q6k_code(const uint8_t *blk, int k) {  // src/quant.c:403-406
    const int p = k >> 7, r = k & 127, kk = r >> 5, l = r & 31;
    const uint32_t lo = (blk[64 * p + ((kk & 1) ? 32 : 0) + l] >> ((kk >> 1) * 4)) & 15;
    const uint32_t hi = (blk[128 + 32 * p + l] >> (2 * kk)) & 3;
    return lo | (hi << 4);
}

// u32 number n (0..15) of lane t's code words: stored as 16-byte word n/4 of
// 32 interleaved lanes, so a warp's 16-byte shared-memory reads of one word
// index are contiguous (no bank conflicts).
__device__ __host__ __forceinline__ int code_word(int n, int t) { return ((n >> 2) * 32 + t) * 4 + (n & 3); }

__global__ void k_repack_q4k(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int M, int KB) {
    const int unit = blockIdx.x, rt = unit / KB, kb = unit % KB, t = threadIdx.x;
    uint8_t *u = dst + (size_t)unit * Q4K_UNIT;
    if (t < 16) {
        const int r = rt * 16 + t;
        for (int i = 0; i < 16; i++) u[16 * t + i] = r < M ? src[((size_t)r * KB + kb) * 144 + i] : 0;
    }
    const int g = t >> 2, c = t & 3;
    const uint8_t *b0 = rt * 16 + g < M ? src + ((size_t)(rt * 16 + g) * KB + kb) * 144 : nullptr;
    const uint8_t *b1 = rt * 16 + g + 8 < M ? src + ((size_t)(rt * 16 + g + 8) * KB + kb) * 144 : nullptr;
    uint32_t *o = reinterpret_cast<uint32_t *>(u + 256);
    for (int j = 0; j < 8; j++) {
        uint32_t p = 0, q = 0;
        for (int i = 0; i < 4; i++) {
            const int k0 = 32 * j + 4 * c + i, k1 = k0 + 16;
            if (b0) p |= (q4k_code(b0, k0) | (q4k_code(b0, k1) << 4)) << (8 * i);
            if (b1) q |= (q4k_code(b1, k0) | (q4k_code(b1, k1) << 4)) << (8 * i);
        }
        o[code_word(2 * j, t)] = p;
        o[code_word(2 * j + 1, t)] = q;
    }
}

__global__ void k_repack_q6k(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int M, int KB) {
    const int unit = blockIdx.x, rt = unit / KB, kb = unit % KB, t = threadIdx.x;
    uint8_t *u = dst + (size_t)unit * Q6K_UNIT;
    if (t < 16) {
        const int r = rt * 16 + t;
        const uint8_t *b = r < M ? src + ((size_t)r * KB + kb) * 210 : nullptr;
        for (int i = 0; i < 16; i++) u[16 * t + i] = b ? b[192 + i] : 0;
        u[256 + 2 * t] = b ? b[208] : 0;
        u[256 + 2 * t + 1] = b ? b[209] : 0;
    }
    const int g = t >> 2, c = t & 3;
    const uint8_t *b0 = rt * 16 + g < M ? src + ((size_t)(rt * 16 + g) * KB + kb) * 210 : nullptr;
    const uint8_t *b1 = rt * 16 + g + 8 < M ? src + ((size_t)(rt * 16 + g + 8) * KB + kb) * 210 : nullptr;
    uint32_t *lo = reinterpret_cast<uint32_t *>(u + 288);
    uint32_t *hi = reinterpret_cast<uint32_t *>(u + 288 + 2048);
    for (int j = 0; j < 16; j++) {
        uint32_t p = 0;
        for (int i = 0; i < 4; i++) {
            const int k = 16 * j + 4 * c + i;
            const uint32_t v0 = b0 ? q6k_code(b0, k) : 0, v1 = b1 ? q6k_code(b1, k) : 0;
            p |= ((v0 & 15) | ((v1 & 15) << 4)) << (8 * i);
        }
        lo[code_word(j, t)] = p;
    }
    for (int jp = 0; jp < 8; jp++) {
        uint32_t h = 0;
        for (int i = 0; i < 4; i++) {
            const int k = 32 * jp + 4 * c + i, k2 = k + 16;
            const uint32_t a = b0 ? q6k_code(b0, k) >> 4 : 0, b = b1 ? q6k_code(b1, k) >> 4 : 0;
            const uint32_t a2 = b0 ? q6k_code(b0, k2) >> 4 : 0, b2 = b1 ? q6k_code(b1, k2) >> 4 : 0;
            h |= (a | (b << 2) | (a2 << 4) | (b2 << 6)) << (8 * i);
        }
        hi[code_word(jp, t)] = h;
    }
}

// ---------------------------------------------------------------------------
// activations: int8 limbs in B-fragment order (per CTA, shared memory)
// ---------------------------------------------------------------------------
// B column n = 8*nt + g of n-tile nt carries limb (g % 3) of batch row
// 2*nt + g / 3 (g < 6); columns 6, 7 are zero.  xq = rint(x * 2^s_b) with
// |xq| <= 2^22, split xq = L0 + 2^8 L1 + 2^16 L2 with L0, L1 in [-128, 127].
__device__ __forceinline__ int limb_of(float x, float scale, int limb) {
    const int xi = __float2int_rn(x * scale);
    const int l0 = (int)(int8_t)(xi & 0xFF);
    const int r = (xi - l0) >> 8;
    const int l1 = (int)(int8_t)(r & 0xFF);
    return limb == 0 ? l0 : limb == 1 ? l1 : (r - l1) >> 8;
}
__device__ __forceinline__ uint32_t pack_limbs(float4 v, float s, int limb) {
    return (uint32_t)(limb_of(v.x, s, limb) & 0xFF) | ((uint32_t)(limb_of(v.y, s, limb) & 0xFF) << 8) |
           ((uint32_t)(limb_of(v.z, s, limb) & 0xFF) << 16) | ((uint32_t)(limb_of(v.w, s, limb) & 0xFF) << 24);
}

struct TArgs {
    const uint8_t *w;
    const float *x, *bias;
    float *y;
    int M, KB, RT, ldx, ldy, nb, epi;
    // prologue applied to x while it is quantized (LMC_PRO_*), its operands
    int pro;
    const float *pw, *pb, *x2;
    float eps;
    unsigned long long *keys;  // non-NULL: greedy-pick key per batch row (argmax epilogue)
    // stream-K split: U = RT*KB units; CTA c owns units [c*U/G, (c+1)*U/G)
    long long U;
    int maxrt;   // row tiles one CTA range can touch
    int stages;  // bulk-copy ring depth per warp
    float *ws;   // cross-CTA fixup sums [RT*16][8] (all zero between launches)
    int *cnt;    // cross-CTA arrival counters [RT] (all zero between launches)
};

constexpr int WARPS = 16;  // warps per CTA; one CTA per SM

// shared-memory layout (bytes)
template <int NT> struct Smem {
    int KB, CH, maxrt, stages, unit;  // CH = column chunks per unit: 8 (Q4_K, k32) or 16 (Q6_K, k16)
    __device__ __host__ size_t xf_bytes() const { return (size_t)KB * CH * NT * 32 * (CH == 8 ? 8 : 4); }
    __device__ __host__ size_t xs_off() const { return xf_bytes(); }  // per-chunk sums of x
    __device__ __host__ size_t xs_bytes() const { return (size_t)KB * CH * 2 * NT * 4; }
    __device__ __host__ size_t sc_off() const { return xs_off() + xs_bytes(); }  // scale, inverse, mean, rstd
    __device__ __host__ size_t red_off() const { return sc_off() + 128; }      // reduction scratch
    __device__ __host__ size_t acc_off() const { return red_off() + 256 * NT; }  // [maxrt][2NT][16] floats
    __device__ __host__ size_t ring_off() const {
        return (acc_off() + (size_t)maxrt * 2 * NT * 16 * 4 + 127) / 128 * 128;
    }
    __device__ __host__ size_t bar_off() const { return ring_off() + (size_t)WARPS * stages * unit; }
    __device__ __host__ size_t total() const { return bar_off() + (size_t)WARPS * stages * 8; }
};

// The activation a GEMV multiplies, after its prologue op:
//   LMC_PRO_NONE     x
//   LMC_PRO_LAYERNORM (x - mean) * rstd * w + b      (src/ops.c:47-59)
//   LMC_PRO_RMSNORM  (w * rs) * x                    (src/ops_llama.c:24-33)
//   LMC_PRO_SWIGLU   silu(x) * x2                    (src/ops_llama.c:150-151)
// so the norm / gate that precedes a projection needs no kernel of its own.
struct XView {
    const float *x, *x2, *w, *b;
    int ldx, pro;
    const float *mean, *rstd;  // per batch row (shared memory)
    __device__ __forceinline__ float at(int bi, int k) const {
        const float v = x[(size_t)bi * ldx + k];
        switch (pro) {
        case LMC_PRO_LAYERNORM: return (v - mean[bi]) * rstd[bi] * w[k] + b[k];
        case LMC_PRO_RMSNORM: return w[k] * rstd[bi] * v;
        case LMC_PRO_SWIGLU: return lmc_silu_f(v) * x2[(size_t)bi * ldx + k];
        default: return v;
        }
    }
    __device__ __forceinline__ float4 at4(int bi, int k) const {
        const float4 v = *reinterpret_cast<const float4 *>(x + (size_t)bi * ldx + k);
        if (pro == LMC_PRO_NONE) return v;
        if (pro == LMC_PRO_SWIGLU) {
            const float4 u = *reinterpret_cast<const float4 *>(x2 + (size_t)bi * ldx + k);
            return make_float4(lmc_silu_f(v.x) * u.x, lmc_silu_f(v.y) * u.y, lmc_silu_f(v.z) * u.z,
                               lmc_silu_f(v.w) * u.w);
        }
        const float4 ww = *reinterpret_cast<const float4 *>(w + k);
        if (pro == LMC_PRO_RMSNORM) {
            const float r = rstd[bi];
            return make_float4(ww.x * r * v.x, ww.y * r * v.y, ww.z * r * v.z, ww.w * r * v.w);
        }
        const float4 bb = *reinterpret_cast<const float4 *>(b + k);
        const float m = mean[bi], r = rstd[bi];
        return make_float4((v.x - m) * r * ww.x + bb.x, (v.y - m) * r * ww.y + bb.y, (v.z - m) * r * ww.z + bb.z,
                           (v.w - m) * r * ww.w + bb.w);
    }
};

// Block-wide sum of one value per thread (all threads get it); `red` holds 32 floats.
__device__ __forceinline__ float cta_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.0f;
    return warp_sum(t);
}

// Quantize the (prologue-transformed) x into B fragments (CH chunks per 256
// columns) and per-chunk sums.  Each thread quantizes 4 (Q6_K) or 8 (Q4_K)
// columns of one batch row once and writes all three limbs (the three lanes
// g = 3*(b%2) + limb).
template <int NT, int CH>
__device__ void build_x(uint8_t *smem, const Smem<NT> &L, const TArgs &a) {
    float *scl = reinterpret_cast<float *>(smem + L.sc_off());
    float *inv = scl + 2 * NT, *mean = inv + 2 * NT, *rstd = mean + 2 * NT;
    float *red = reinterpret_cast<float *>(smem + L.red_off());  // reduction scratch
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int K = a.KB * 256, nb = a.nb;
    const XView xv{a.x, a.x2, a.pw, a.pb, a.ldx, a.pro, mean, rstd};
    if (a.pro == LMC_PRO_LAYERNORM || a.pro == LMC_PRO_RMSNORM) {  // per-row statistics
        for (int b = 0; b < nb; b++) {
            const float *xb = a.x + (size_t)b * a.ldx;
            float s1 = 0.0f;
            for (int k = threadIdx.x; k < K; k += blockDim.x) s1 += a.pro == LMC_PRO_RMSNORM ? xb[k] * xb[k] : xb[k];
            s1 = cta_sum(s1, red);
            if (a.pro == LMC_PRO_RMSNORM) {
                if (threadIdx.x == 0) { mean[b] = 0.0f; rstd[b] = 1.0f / sqrtf(s1 / (float)K + a.eps); }
            } else {
                const float mu = s1 / (float)K;
                float s2 = 0.0f;
                for (int k = threadIdx.x; k < K; k += blockDim.x) { const float d = xb[k] - mu; s2 += d * d; }
                s2 = cta_sum(s2, red);
                if (threadIdx.x == 0) { mean[b] = mu; rstd[b] = 1.0f / sqrtf(s2 / (float)K + 1e-5f); }
            }
        }
        __syncthreads();
    }
    // max |x| per batch row, all threads
    for (int b = 0; b < nb; b++) {
        float m = 0.0f;
        for (int k = threadIdx.x * 4; k < K; k += blockDim.x * 4) {
            const float4 v = xv.at4(b, k);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        m = warp_max(m);
        if (lane == 0) red[b * 32 + wid] = m;
    }
    __syncthreads();
    if (threadIdx.x < 2 * NT) {
        const int b = threadIdx.x;
        float m = 0.0f;
        if (b < nb)
            for (int w = 0; w < nw; w++) m = fmaxf(m, red[b * 32 + w]);
        int e = 0;
        if (m > 0.0f) frexpf(m, &e);  // m < 2^e, so |x| * 2^(22-e) < 2^22
        scl[b] = m > 0.0f ? ldexpf(1.0f, 22 - e) : 1.0f;
        inv[b] = m > 0.0f ? ldexpf(1.0f, e - 22) : 0.0f;
    }
    __syncthreads();
    const int KB = a.KB;
    // fragments: one task = (kb, j, c, batch row b): 4 or 8 columns
    const int n_tasks = KB * CH * 4 * 2 * NT;
    for (int t = threadIdx.x; t < n_tasks; t += blockDim.x) {
        const int b = t % (2 * NT), c = (t / (2 * NT)) & 3, j = (t / (8 * NT)) % CH, kb = t / (8 * NT * CH);
        const int nt = b >> 1, g0 = 3 * (b & 1);
        uint32_t r0[3] = {0u, 0u, 0u}, r1[3] = {0u, 0u, 0u};
        if (b < nb) {
            const float s = scl[b];
            const int k0 = kb * 256 + (CH == 8 ? 32 : 16) * j + 4 * c;
            const float4 v0 = xv.at4(b, k0);
            const float va[4] = {v0.x, v0.y, v0.z, v0.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int xi = __float2int_rn(va[i] * s);
                const int l0 = (int)(int8_t)(xi & 0xFF), rr = (xi - l0) >> 8, l1 = (int)(int8_t)(rr & 0xFF);
                r0[0] |= (uint32_t)(l0 & 0xFF) << (8 * i);
                r0[1] |= (uint32_t)(l1 & 0xFF) << (8 * i);
                r0[2] |= (uint32_t)(((rr - l1) >> 8) & 0xFF) << (8 * i);
            }
            if (CH == 8) {
                const float4 v1 = xv.at4(b, k0 + 16);
                const float vb[4] = {v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int xi = __float2int_rn(vb[i] * s);
                    const int l0 = (int)(int8_t)(xi & 0xFF), rr = (xi - l0) >> 8, l1 = (int)(int8_t)(rr & 0xFF);
                    r1[0] |= (uint32_t)(l0 & 0xFF) << (8 * i);
                    r1[1] |= (uint32_t)(l1 & 0xFF) << (8 * i);
                    r1[2] |= (uint32_t)(((rr - l1) >> 8) & 0xFF) << (8 * i);
                }
            }
        }
        const size_t e0 = ((size_t)(kb * CH + j) * NT + nt) * 32 + 4 * g0 + c;  // lane g0*4 + c
#pragma unroll
        for (int limb = 0; limb < 3; limb++) {
            if (CH == 8) reinterpret_cast<uint2 *>(smem)[e0 + 4 * limb] = make_uint2(r0[limb], r1[limb]);
            else reinterpret_cast<uint32_t *>(smem)[e0 + 4 * limb] = r0[limb];
        }
    }
    // the two unused columns (g = 6, 7) of every chunk are zero
    const int n_zero = KB * CH * NT * 8;
    for (int t = threadIdx.x; t < n_zero; t += blockDim.x) {
        const size_t e = (size_t)(t >> 3) * 32 + 24 + (t & 7);
        if (CH == 8) reinterpret_cast<uint2 *>(smem)[e] = make_uint2(0u, 0u);
        else reinterpret_cast<uint32_t *>(smem)[e] = 0u;
    }
    // per-chunk sums of x (fp32): xs[(kb*CH + j)*2NT + b]
    float *xs = reinterpret_cast<float *>(smem + L.xs_off());
    const int span = CH == 8 ? 32 : 16;
    for (int e = wid; e < KB * CH * 2 * NT; e += nw) {
        const int b = e % (2 * NT), jj = (e / (2 * NT)) % CH, kb = e / (2 * NT * CH);
        float v = 0.0f;
        if (b < nb && lane < span) v = xv.at(b, kb * 256 + span * jj + lane);
        v = warp_sum(v);
        if (lane == 0) xs[e] = v;
    }
}

// ---------------------------------------------------------------------------
// bulk-copy ring: per warp, `stages` units in flight, tracked by mbarriers
// ---------------------------------------------------------------------------
__device__ int g_tiled_timeout;  // set when a bounded wait gives up (lmc_device_status)

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void issue_unit(uint64_t *bar, void *dst, const void *src, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after ~2^20 polls (each poll may itself suspend for
// a while), records the timeout and lets the caller skip the unit.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t t = 0; t < (1u << 20); t++)
        if (mbar_try(bar, parity)) return true;
    atomicExch(&g_tiled_timeout, 1);
    return false;
}

// Per-warp partial of the row tile currently being streamed:
//   tot[nt][i]  sum over units of (block scale d) x (int32 sum over chunks of
//               sub-scale x chunk product), C fragment element i (rows g / g+8,
//               columns 2c, 2c+1)
//   cor[b][h]   corrections (Q4_K mins, Q6_K -32 offsets) for batch row b and
//               row half h over this lane's share of the chunks
template <int NT> struct Part {
    float tot[NT][4];
    float cor[2 * NT][2];
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) tot[nt][i] = 0.0f;
#pragma unroll
        for (int b = 0; b < 2 * NT; b++) cor[b][0] = cor[b][1] = 0.0f;
    }
};

// Add a warp's partial into the CTA accumulator of its row tile: combine
// the limb columns (weights 1, 2^8, 2^16, times the vector's inverse scale),
// subtract the corrections, reduce the quad, one shared atomic per value.
template <int NT>
__device__ __forceinline__ void flush(const Part<NT> &p, float *acc_rt, const float *inv, int nb, int lane) {
    const int g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        float y0[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};  // [batch in tile][row half]
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const int col = 2 * c + q;
            if (col < 6) {
                const float wl = col % 3 == 0 ? 1.0f : (col % 3 == 1 ? 256.0f : 65536.0f);
                y0[col / 3][0] += wl * p.tot[nt][q];
                y0[col / 3][1] += wl * p.tot[nt][2 + q];
            }
        }
#pragma unroll
        for (int bb = 0; bb < 2; bb++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int b = 2 * nt + bb;
                float v = inv[b] * y0[bb][h] - p.cor[b][h];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                if (c == 2 * bb + h && b < nb) atomicAdd(acc_rt + b * 16 + g + 8 * h, v);
            }
    }
}

__device__ __forceinline__ void epilogue(const TArgs &a, int b, int row, float v) {
    if (row >= a.M || b >= a.nb) return;
    if (a.bias) v += a.bias[row];
    if (a.epi & LMC_EPI_GELU) v = lmc_gelu_f(v);
    float *o = a.y + (size_t)b * a.ldy + row;
    *o = (a.epi & LMC_EPI_ACCUM) ? *o + v : v;
    if (a.keys) atomicMax(a.keys + b, lmc_argmax_key(v, row));
}

// Q4_K unit (src/quant.c:275-303): d * sum_sub sc * (sum_32 q x) - dmin * sum_sub m * X_sub
template <int NT>
__device__ __forceinline__ void unit_q4k(Part<NT> &p, const uint8_t *u, const uint2 *xf, const float *xs, int kb,
                                         int lane) {
    const int g = lane >> 2, c = lane & 3;
    const uint4 H0 = *reinterpret_cast<const uint4 *>(u + 16 * g);
    const uint4 H1 = *reinterpret_cast<const uint4 *>(u + 16 * (g + 8));
    const uint4 *cw = reinterpret_cast<const uint4 *>(u + 256);
    const uint4 q0 = cw[lane], q1 = cw[32 + lane], q2 = cw[64 + lane], q3 = cw[96 + lane];
    const uint32_t qs[16] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w,
                             q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
    // 6-bit scales / mins, four at a time (src/quant.c:44-53)
    const uint32_t sc0a = H0.y & 0x3F3F3F3Fu, sc0b = (H0.w & LO4) | ((H0.y >> 2) & 0x30303030u);
    const uint32_t sc1a = H1.y & 0x3F3F3F3Fu, sc1b = (H1.w & LO4) | ((H1.y >> 2) & 0x30303030u);
    int it[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) it[nt][i] = 0;
    const uint2 *xk = xf + (size_t)kb * 8 * NT * 32 + lane;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int s0 = ubyte(j < 4 ? sc0a : sc0b, j & 3), s1 = ubyte(j < 4 ? sc1a : sc1b, j & 3);
        const uint32_t P = qs[2 * j], Q = qs[2 * j + 1];
        const uint32_t a0 = P & LO4, a2 = (P >> 4) & LO4, a1 = Q & LO4, a3 = (Q >> 4) & LO4;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const uint2 bx = xk[(j * NT + nt) * 32];
            int acc[4];
            imma_k32(acc, a0, a1, a2, a3, bx.x, bx.y);
            it[nt][0] += s0 * acc[0];
            it[nt][1] += s0 * acc[1];
            it[nt][2] += s1 * acc[2];
            it[nt][3] += s1 * acc[3];
        }
    }
    const float2 dd0 = __half22float2(*reinterpret_cast<const __half2 *>(&H0.x));  // (d, dmin)
    const float2 dd1 = __half22float2(*reinterpret_cast<const __half2 *>(&H1.x));
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        p.tot[nt][0] += dd0.x * (float)it[nt][0];
        p.tot[nt][1] += dd0.x * (float)it[nt][1];
        p.tot[nt][2] += dd1.x * (float)it[nt][2];
        p.tot[nt][3] += dd1.x * (float)it[nt][3];
    }
    // mins of sub-blocks 2c, 2c+1 (this lane's share of the 8)
    const uint32_t m0a = H0.z & 0x3F3F3F3Fu, m0b = ((H0.w >> 4) & LO4) | ((H0.z >> 2) & 0x30303030u);
    const uint32_t m1a = H1.z & 0x3F3F3F3Fu, m1b = ((H1.w >> 4) & LO4) | ((H1.z >> 2) & 0x30303030u);
    const uint32_t mw0 = c < 2 ? m0a : m0b, mw1 = c < 2 ? m1a : m1b;
    const int i0 = (2 * c) & 3;
    const float mg0 = dd0.y * (float)ubyte(mw0, i0), mg1 = dd0.y * (float)ubyte(mw0, i0 + 1);
    const float mh0 = dd1.y * (float)ubyte(mw1, i0), mh1 = dd1.y * (float)ubyte(mw1, i0 + 1);
    const float *xsk = xs + ((size_t)kb * 8 + 2 * c) * 2 * NT;
#pragma unroll
    for (int b = 0; b < 2 * NT; b++) {
        const float X0 = xsk[b], X1 = xsk[2 * NT + b];
        p.cor[b][0] += mg0 * X0 + mg1 * X1;
        p.cor[b][1] += mh0 * X0 + mh1 * X1;
    }
}

// Q6_K unit (src/quant.c:386-414): d * sum_chunks sc * (sum_16 q x - 32 X_chunk)
template <int NT>
__device__ __forceinline__ void unit_q6k(Part<NT> &p, const uint8_t *u, const uint32_t *xf, const float *xs, int kb,
                                         int lane) {
    const int g = lane >> 2, c = lane & 3;
    const uint4 s0v = *reinterpret_cast<const uint4 *>(u + 16 * g);
    const uint4 s1v = *reinterpret_cast<const uint4 *>(u + 16 * (g + 8));
    const float d0 = __half2float(*reinterpret_cast<const __half *>(u + 256 + 2 * g));
    const float d1 = __half2float(*reinterpret_cast<const __half *>(u + 256 + 2 * (g + 8)));
    const uint4 *lw = reinterpret_cast<const uint4 *>(u + 288), *hw = reinterpret_cast<const uint4 *>(u + 288 + 2048);
    const uint4 q0 = lw[lane], q1 = lw[32 + lane], q2 = lw[64 + lane], q3 = lw[96 + lane];
    const uint4 hq0 = hw[lane], hq1 = hw[32 + lane];
    const uint32_t lo[16] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w,
                             q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
    const uint32_t hs[8] = {hq0.x, hq0.y, hq0.z, hq0.w, hq1.x, hq1.y, hq1.z, hq1.w};
    const uint32_t sw0[4] = {s0v.x, s0v.y, s0v.z, s0v.w}, sw1[4] = {s1v.x, s1v.y, s1v.z, s1v.w};
    int it[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) it[nt][i] = 0;
    const uint32_t *xk = xf + (size_t)kb * 16 * NT * 32 + lane;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const int s0 = sbyte(sw0[j >> 2], j & 3), s1 = sbyte(sw1[j >> 2], j & 3);
        const uint32_t H = hs[j >> 1], P = lo[j];
        const uint32_t tg = ((j & 1) ? H : (H << 4)) & 0x30303030u;
        const uint32_t tg8 = ((j & 1) ? (H >> 2) : (H << 2)) & 0x30303030u;
        const uint32_t a0 = (P & LO4) | tg, a1 = ((P >> 4) & LO4) | tg8;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            int acc[4];
            imma_k16(acc, a0, a1, xk[(j * NT + nt) * 32]);
            it[nt][0] += s0 * acc[0];
            it[nt][1] += s0 * acc[1];
            it[nt][2] += s1 * acc[2];
            it[nt][3] += s1 * acc[3];
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        p.tot[nt][0] += d0 * (float)it[nt][0];
        p.tot[nt][1] += d0 * (float)it[nt][1];
        p.tot[nt][2] += d1 * (float)it[nt][2];
        p.tot[nt][3] += d1 * (float)it[nt][3];
    }
    // -32 offsets of chunks 4c..4c+3 (this lane's share of the 16)
    const float *xsk = xs + ((size_t)kb * 16 + 4 * c) * 2 * NT;
    const uint32_t swc0 = c == 0 ? sw0[0] : c == 1 ? sw0[1] : c == 2 ? sw0[2] : sw0[3];
    const uint32_t swc1 = c == 0 ? sw1[0] : c == 1 ? sw1[1] : c == 2 ? sw1[2] : sw1[3];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const float f0 = 32.0f * d0 * (float)sbyte(swc0, q);
        const float f1 = 32.0f * d1 * (float)sbyte(swc1, q);
#pragma unroll
        for (int b = 0; b < 2 * NT; b++) {
            const float X = xsk[q * 2 * NT + b];
            p.cor[b][0] += f0 * X;
            p.cor[b][1] += f1 * X;
        }
    }
}

// The streaming GEMV.  One CTA of WARPS warps per SM.  CTA c takes the
// contiguous unit range [c*U/G, (c+1)*U/G) of the row-tile-major unit order
// and splits it into WARPS contiguous sub-ranges; each warp streams its units
// through a `stages`-deep ring of bulk async copies (global -> shared), which
// it starts before pdl_wait() (weights do not depend on earlier kernels).
// Partial sums meet per row tile in shared memory; row tiles shared with a
// neighbouring CTA are finished through the fixup workspace by whichever CTA
// arrives last.
template <int NT, int QT>
__global__ void __launch_bounds__(WARPS * 32, 1) k_gemv_stream(TArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int CH = QT == 4 ? 8 : 16, UNIT = QT == 4 ? Q4K_UNIT : Q6K_UNIT;
    const Smem<NT> L{a.KB, CH, a.maxrt, a.stages, UNIT};
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const long long G = gridDim.x;
    const int u0 = (int)((long long)blockIdx.x * a.U / G), u1 = (int)(((long long)blockIdx.x + 1) * a.U / G);
    const int w0 = u0 + (int)((long long)(u1 - u0) * wid / WARPS);
    const int w1 = u0 + (int)((long long)(u1 - u0) * (wid + 1) / WARPS);
    uint8_t *ring = smem + L.ring_off() + (size_t)wid * a.stages * UNIT;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off()) + wid * a.stages;
    if (lane == 0) {
        for (int s = 0; s < a.stages; s++) mbar_init(&bars[s]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    pdl_launch_dependents();
    if (lane == 0)  // weights only: streams while the previous kernel finishes
        for (int s = 0; s < a.stages && w0 + s < w1; s++)
            issue_unit(&bars[s], ring + (size_t)s * UNIT, a.w + (size_t)(w0 + s) * UNIT, UNIT);
    pdl_wait();
    build_x<NT, CH>(smem, L, a);
    float *acc = reinterpret_cast<float *>(smem + L.acc_off());
    for (int i = threadIdx.x; i < a.maxrt * 2 * NT * 16; i += blockDim.x) acc[i] = 0.0f;
    __syncthreads();
    const float *inv = reinterpret_cast<const float *>(smem + L.sc_off()) + 2 * NT;
    const float *xs = reinterpret_cast<const float *>(smem + L.xs_off());
    const int rt0 = u0 / a.KB;
    Part<NT> p;
    p.zero();
    int cur = -1;
    bool ok = true;
    // unit i = rt * KB + kb lives in ring slot s, k-th refill of it (parity k & 1);
    // all advanced incrementally (no divisions in the loop)
    int rt = w0 / a.KB, kb = w0 - rt * a.KB, s = 0;
    uint32_t parity = 0;
    for (int i = w0; i < w1; i++) {
        if (ok) ok = mbar_wait(&bars[s], parity);
        if (rt != cur) {
            if (cur >= 0) flush<NT>(p, acc + (size_t)(cur - rt0) * 2 * NT * 16, inv, a.nb, lane);
            p.zero();
            cur = rt;
        }
        if (ok) {
            const uint8_t *u = ring + (size_t)s * UNIT;
            if (QT == 4) unit_q4k<NT>(p, u, reinterpret_cast<const uint2 *>(smem), xs, kb, lane);
            else unit_q6k<NT>(p, u, reinterpret_cast<const uint32_t *>(smem), xs, kb, lane);
        }
        __syncwarp();
        if (lane == 0 && ok && i + a.stages < w1) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // slot reads done before the refill
            issue_unit(&bars[s], ring + (size_t)s * UNIT, a.w + (size_t)(i + a.stages) * UNIT, UNIT);
        }
        if (++kb == a.KB) { kb = 0; rt++; }
        if (++s == a.stages) { s = 0; parity ^= 1u; }
    }
    if (cur >= 0) flush<NT>(p, acc + (size_t)(cur - rt0) * 2 * NT * 16, inv, a.nb, lane);
    if (!ok && lane == 0)  // copies of this warp may still be in flight: bounded drain
        for (int q = 0; q < a.stages && q < w1 - w0; q++) (void)mbar_wait(&bars[q], 0);
    __syncthreads();
    if (u1 <= u0) return;
    const int rt_last = (u1 - 1) / a.KB;
    for (int rt = rt0 + wid; rt <= rt_last; rt += WARPS) {
        const float *ar = acc + (size_t)(rt - rt0) * 2 * NT * 16;
        const long long f0 = (long long)rt * a.KB, f1 = f0 + a.KB;
        if (f0 >= u0 && f1 <= u1) {  // whole row tile in this CTA
            for (int e = lane; e < 16 * a.nb; e += 32) epilogue(a, e >> 4, rt * 16 + (e & 15), ar[e]);
            continue;
        }
        // shared with neighbour CTAs: add into the workspace; the last to arrive finishes
        for (int e = lane; e < 16 * a.nb; e += 32) atomicAdd(a.ws + ((size_t)rt * 16 + (e & 15)) * 8 + (e >> 4), ar[e]);
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            const long long cf = ((f0 + 1) * G - 1) / a.U, cl = (f1 * G - 1) / a.U;  // owners of the first/last unit
            last = atomicAdd(a.cnt + rt, 1) == (int)(cl - cf);
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence();
            for (int e = lane; e < 16 * a.nb; e += 32) {
                float *wp = a.ws + ((size_t)rt * 16 + (e & 15)) * 8 + (e >> 4);
                const float v = __ldcg(wp);
                *wp = 0.0f;
                epilogue(a, e >> 4, rt * 16 + (e & 15), v);
            }
            __syncwarp();
            if (lane == 0) a.cnt[rt] = 0;
        }
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// Fixup workspace shared by all tiled tensors of this device: launches are
// ordered on one stream (PDL lets a kernel start before the previous one
// ends, but it touches the workspace only after pdl_wait()).
static float *g_ws = NULL;
static int *g_cnt = NULL;
static int g_ws_rt = 0;

static int ensure_workspace(int RT) {
    if (RT <= g_ws_rt) return LMC_OK;
    if (g_ws) cudaFree(g_ws);
    if (g_cnt) cudaFree(g_cnt);
    g_ws = NULL;
    g_cnt = NULL;
    g_ws_rt = 0;
    LMC_CUDA_TRY(cudaMalloc(&g_ws, (size_t)RT * 16 * 8 * sizeof(float)));
    LMC_CUDA_TRY(cudaMalloc(&g_cnt, (size_t)RT * sizeof(int)));
    LMC_CUDA_TRY(cudaMemset(g_ws, 0, (size_t)RT * 16 * 8 * sizeof(float)));
    LMC_CUDA_TRY(cudaMemset(g_cnt, 0, (size_t)RT * sizeof(int)));
    g_ws_rt = RT;
    return LMC_OK;
}

extern "C" int lmc_device_status(void) {
    int v = 0;
    LMC_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_tiled_timeout, sizeof(int)));
    if (!v) return LMC_OK;
    const int zero = 0;
    LMC_CUDA_TRY(cudaMemcpyToSymbol(g_tiled_timeout, &zero, sizeof(int)));
    return lmc_set_error(LMC_ERR_TIMEOUT, "a kernel gave up a bounded wait (bulk copy not completed)");
}

template <int NT> static Smem<NT> layout(uint32_t type, int KB, int maxrt, int stages) {
    return Smem<NT>{KB, type == LMC_TYPE_Q4_K ? 8 : 16, maxrt, stages, type == LMC_TYPE_Q4_K ? Q4K_UNIT : Q6K_UNIT};
}

static int grid_for(long long U) { return (int)std::min<long long>(U, lmc_sm_count()); }
static int maxrt_for(long long U, int KB, int G) { return (int)(((U + G - 1) / G + KB - 1) / KB) + 1; }

// deepest ring (2..4 stages) that fits the shared-memory budget, 0 if none
template <int NT> static int pick_stages(uint32_t type, int KB, int maxrt) {
    for (int st = 4; st >= 2; st--)
        if (layout<NT>(type, KB, maxrt, st).total() <= SMEM_LIMIT) return st;
    return 0;
}

extern "C" int lmc_tiled_build(lmc_qtensor *t) {
    t->tiled = NULL;
    if ((t->type != LMC_TYPE_Q4_K && t->type != LMC_TYPE_Q6_K) || t->cols % 256) return LMC_OK;
    const int KB = t->cols / 256, RT = (t->rows + 15) / 16;
    const long long U = (long long)RT * KB;
    if (!pick_stages<1>(t->type, KB, maxrt_for(U, KB, grid_for(U)))) return LMC_OK;  // very long rows: generic path
    int rc = ensure_workspace(RT);
    if (rc) return rc;
    const size_t unit = t->type == LMC_TYPE_Q4_K ? Q4K_UNIT : Q6K_UNIT;
    const size_t bytes = (size_t)RT * KB * unit;
    LMC_CUDA_TRY(cudaMalloc(&t->tiled, bytes));
    if (t->type == LMC_TYPE_Q4_K)
        k_repack_q4k<<<RT * KB, 32>>>((const uint8_t *)t->blocks, (uint8_t *)t->tiled, t->rows, KB);
    else
        k_repack_q6k<<<RT * KB, 32>>>((const uint8_t *)t->blocks, (uint8_t *)t->tiled, t->rows, KB);
    LMC_LAUNCH_CHECK("repack");
    LMC_CUDA_TRY(cudaDeviceSynchronize());
    t->tiled_bytes = bytes;
    t->tiled_rows = RT * 16;
    return LMC_OK;
}

template <int NT>
static int launch_nt(const lmc_qtensor *t, TArgs a, cudaStream_t s) {
    const int G = grid_for(a.U);
    a.maxrt = maxrt_for(a.U, a.KB, G);
    a.stages = pick_stages<NT>(t->type, a.KB, a.maxrt);
    if (!a.stages) return LMC_ERR_UNSUPPORTED;
    const size_t smem = layout<NT>(t->type, a.KB, a.maxrt, a.stages).total();
    const void *fn = t->type == LMC_TYPE_Q4_K ? (const void *)k_gemv_stream<NT, 4> : (const void *)k_gemv_stream<NT, 6>;
    static thread_local struct { const void *fn; size_t max_smem; } attr[8];
    bool done = false;
    for (auto &e : attr)
        if (e.fn == fn) {
            if (smem > e.max_smem) {
                LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
                e.max_smem = smem;
            }
            done = true;
            break;
        }
    if (!done) {
        LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        for (auto &e : attr)
            if (!e.fn) { e.fn = fn; e.max_smem = smem; break; }
    }
    if (t->type == LMC_TYPE_Q4_K)
        LMC_LAUNCH("tiled gemv q4k", (k_gemv_stream<NT, 4>), G, WARPS * 32, smem, s, a);
    else
        LMC_LAUNCH("tiled gemv q6k", (k_gemv_stream<NT, 6>), G, WARPS * 32, smem, s, a);
    return LMC_OK;
}

extern "C" int lmc_tiled_gemv_launch(const lmc_qtensor *t, const float *d_x, int ldx, const float *d_bias, float *d_y,
                                     int ldy, int batch, int epi, cudaStream_t s) {
    if (((uintptr_t)d_x & 15) || (ldx & 3))  // float4 activation loads
        return lmc_gemv_generic_launch(t->type, t->blocks, t->rows, t->cols, d_x, ldx, d_bias, d_y, ldy, batch, epi, s);
    lmc_gemv_extra ex = {LMC_PRO_NONE, NULL, NULL, NULL, 0.0f, NULL};
    return lmc_tiled_gemv_ex(t, d_x, ldx, d_bias, d_y, ldy, batch, epi, &ex, s);
}

extern "C" int lmc_tiled_gemv_ex(const lmc_qtensor *t, const float *d_x, int ldx, const float *d_bias, float *d_y,
                                 int ldy, int batch, int epi, const lmc_gemv_extra *ex, cudaStream_t s) {
    if (!t->tiled) return lmc_set_error(LMC_ERR_UNSUPPORTED, "gemv_ex: no tiled layout");
    if (((uintptr_t)d_x & 15) || (ldx & 3) || (ex->x2 && ((uintptr_t)ex->x2 & 15)) ||
        (ex->w && ((uintptr_t)ex->w & 15)) || (ex->b && ((uintptr_t)ex->b & 15)))
        return lmc_set_error(LMC_ERR_INVALID, "gemv_ex: activations and prologue vectors must be 16-byte aligned");
    if (t->tiled_rows / 16 > g_ws_rt) return lmc_set_error(LMC_ERR_INVALID, "gemv_ex: fixup workspace too small");
    TArgs a;
    a.w = (const uint8_t *)t->tiled;
    a.bias = d_bias;
    a.M = t->rows;
    a.KB = t->cols / 256;
    a.RT = t->tiled_rows / 16;
    a.ldx = ldx;
    a.ldy = ldy;
    a.epi = epi;
    a.pro = ex->pro;
    a.pw = ex->w;
    a.pb = ex->b;
    a.eps = ex->eps;
    a.U = (long long)a.RT * a.KB;
    a.ws = g_ws;
    a.cnt = g_cnt;
    for (int b0 = 0; b0 < batch;) {
        const int nb = std::min(batch - b0, 8);
        a.x = d_x + (size_t)b0 * ldx;
        a.y = d_y + (size_t)b0 * ldy;
        a.x2 = ex->x2 ? ex->x2 + (size_t)b0 * ldx : NULL;
        a.keys = ex->keys ? ex->keys + b0 : NULL;
        a.nb = nb;
        int rc;
        if (nb <= 2) rc = launch_nt<1>(t, a, s);
        else if (nb <= 4) rc = launch_nt<2>(t, a, s);
        else rc = launch_nt<4>(t, a, s);
        if (rc == LMC_ERR_UNSUPPORTED) {  // shared memory: passes of 2 rows
            rc = LMC_OK;
            for (int q = 0; q < nb && !rc; q += 2) {
                TArgs a2 = a;
                a2.x += (size_t)q * ldx;
                a2.y += (size_t)q * ldy;
                if (a2.x2) a2.x2 += (size_t)q * ldx;
                if (a2.keys) a2.keys += q;
                a2.nb = std::min(2, nb - q);
                rc = launch_nt<1>(t, a2, s);
            }
        }
        if (rc == LMC_ERR_UNSUPPORTED)
            return lmc_set_error(rc, "tiled gemv: %d columns need too much shared memory", t->cols);
        if (rc) return rc;
        b0 += nb;
    }
    return LMC_OK;
}
