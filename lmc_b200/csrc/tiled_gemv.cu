// tiled_gemv.cu - K2 (tensor-core): dequant-GEMV for Q4_K, Q6_K and Q8_0 on
// a row-tiled copy of the GGUF blocks, on the integer tensor cores
// (mma.sync s8 x s8 -> s32).  Replaces LMc matmul_vec (src/ops.c:69-97) over
// dequant_q4k / dequant_q6k / dequant_q8_0 (src/quant.c:275-303, :386-414,
// :419-429) at decode batch sizes (1..8 rows per launch).
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
//   Q8_0 unit 4352 B = [16 rows x 8 fp16 d] [8 blocks x 32 lanes x 16 B: the
//     four A registers {row g k 4c.., row g+8 k 4c.., row g k 16+4c.., row g+8
//     k 16+4c..} of the block's m16n8k32 fragment, verbatim int8 codes].
// Needs cols % 256 == 0; other shapes and formats use the generic kernel.
//
// Work split: the row tiles are dealt to clusters of CL CTAs (one CTA per SM,
// contiguous row tiles per cluster); inside a cluster the units are split
// evenly (split-K) and partial row tiles are summed through distributed
// shared memory, so no partial sum goes through global memory.  A CTA uses
// at most ~112 KB of shared memory where it can, so the next GEMV of a decode
// step (programmatic dependent launch) is resident beside it and streams its
// weights while this one finishes.
#include <cuda_fp16.h>

#include "lmc_blocks.cuh"
#include "lmc_common.cuh"
#include "lmc_internal.h"

#include <algorithm>
#include <math.h>

namespace {

constexpr int Q4K_UNIT = 2304, Q6K_UNIT = 3360, Q80_UNIT = 4352;
constexpr int WARPS = 8;                   // warps per CTA
constexpr int NTHR = WARPS * 32;
constexpr int SMEM_PAIR = 112 * 1024;      // two such CTAs fit on one SM
constexpr int SMEM_LIMIT = 200 * 1024;     // one CTA per SM
constexpr int RING_TARGET = 80 * 1024;     // bulk-copy bytes in flight per CTA
// activation tasks a thread holds in registers in the longest-row variant
// (a shorter one holds 4)
__host__ __device__ constexpr int rx_tasks(int QT) { return QT == 6 ? 16 : 7; }
constexpr long long PF_BYTES = 40ll << 20;  // L2 prefetch ahead of the rings, per launch
constexpr uint32_t LO4 = 0x0F0F0F0Fu;

__host__ __device__ constexpr int unit_bytes(int qt) { return qt == 4 ? Q4K_UNIT : qt == 6 ? Q6K_UNIT : Q80_UNIT; }

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

// Q8_0 (src/quant.c:419-429): 34-byte blocks of 32, d (fp16) then int8[32].
__global__ void k_repack_q80(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int M, int KB) {
    const int unit = blockIdx.x, rt = unit / KB, kb = unit % KB, t = threadIdx.x;
    const size_t row_blocks = (size_t)KB * 8;
    uint8_t *u = dst + (size_t)unit * Q80_UNIT;
    if (t < 16) {
        const int r = rt * 16 + t;
        for (int j = 0; j < 8; j++) {
            const uint8_t *b = r < M ? src + ((size_t)r * row_blocks + kb * 8 + j) * 34 : nullptr;
            u[16 * t + 2 * j] = b ? b[0] : 0;
            u[16 * t + 2 * j + 1] = b ? b[1] : 0;
        }
    }
    const int g = t >> 2, c = t & 3;
    const int r0 = rt * 16 + g, r1 = r0 + 8;
    uint32_t *o = reinterpret_cast<uint32_t *>(u + 256);
    for (int j = 0; j < 8; j++) {
        const uint8_t *b0 = r0 < M ? src + ((size_t)r0 * row_blocks + kb * 8 + j) * 34 + 2 : nullptr;
        const uint8_t *b1 = r1 < M ? src + ((size_t)r1 * row_blocks + kb * 8 + j) * 34 + 2 : nullptr;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        for (int i = 0; i < 4; i++) {
            if (b0) w[0] |= (uint32_t)b0[4 * c + i] << (8 * i), w[2] |= (uint32_t)b0[16 + 4 * c + i] << (8 * i);
            if (b1) w[1] |= (uint32_t)b1[4 * c + i] << (8 * i), w[3] |= (uint32_t)b1[16 + 4 * c + i] << (8 * i);
        }
        for (int i = 0; i < 4; i++) o[(j * 32 + t) * 4 + i] = w[i];
    }
}

// ---------------------------------------------------------------------------
// kernel arguments and shared-memory layout
// ---------------------------------------------------------------------------
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
    int key_base;              // global index of row 0 in the keys
    int XL;      // B-fragment lanes stored per chunk: 12 per batch row (3 limbs x 4), 24 for two
    int CL;      // CTAs per cluster
    int NC;      // clusters; cluster c owns row tiles [c*RT/NC, (c+1)*RT/NC)
    int maxrt;   // row-tile slots of the CTA accumulator
    int stages;  // bulk-copy ring depth per warp
    int pf;      // L2 prefetch window per warp, in units beyond the ring
};

// Byte offsets.  CH = column chunks per unit (8 for the k32 formats, 16 for
// Q6_K's k16).  B fragments: for each unit column kb and n-tile nt a block of
// XL lanes x XSTR bytes; a lane's 64 bytes hold its fragment registers of all
// CH chunks (k32: chunk j at 8j, k16: chunk j at 4j), read as four 16-byte
// words.  The 80-byte lane stride keeps those reads free of bank conflicts.
constexpr int XSTR = 80;
template <int NT, int QT> struct Smem {
    static constexpr int CH = QT == 6 ? 16 : 8, NB = 2 * NT;
    int KB, XL, maxrt, stages;
    // + one block of slack: lanes >= XL read (and ignore) the bytes after the last block
    __device__ __host__ size_t xf_bytes() const { return (size_t)KB * NT * XL * XSTR + 32 * XSTR; }
    __device__ __host__ size_t xs_off() const { return (xf_bytes() + 15) / 16 * 16; }  // int chunk sums of xq
    __device__ __host__ size_t xs_bytes() const { return QT == 8 ? 0 : (size_t)KB * CH * NB * 4; }
    // correction B fragments: per (unit column kb, n-tile) 32 lanes x u32
    __device__ __host__ size_t xm_off() const { return xs_off() + xs_bytes(); }
    __device__ __host__ size_t xm_bytes() const { return QT == 8 ? 0 : (size_t)KB * NT * 32 * 4; }
    __device__ __host__ size_t sc_off() const { return xm_off() + xm_bytes(); }  // scale, inverse, mean, rstd [4][8]
    __device__ __host__ size_t red_off() const { return sc_off() + 128; }      // reduction scratch [8][WARPS]
    __device__ __host__ size_t acc_off() const { return red_off() + 8 * WARPS * 4; }  // [maxrt][NB][16] floats
    __device__ __host__ size_t ring_off() const { return (acc_off() + (size_t)maxrt * NB * 16 * 4 + 127) / 128 * 128; }
    __device__ __host__ size_t bar_off() const { return ring_off() + (size_t)WARPS * stages * unit_bytes(QT); }
    __device__ __host__ size_t total() const { return bar_off() + (size_t)WARPS * stages * 8; }
};

// silu(x) = x / (1 + e^-x) from the fast exponential and divide intrinsics
// (a few ulp, far inside the GEMV's 1e-3 bound).  With the full-precision
// expf and IEEE division the SwiGLU prologue cost the 8B model's decode step
// 8% at one sequence and 18% at four.  For x < -87 the divisor passes 2^126
// and the result is 0 (the exact value is below 1e-35 in magnitude).
__device__ __forceinline__ float silu_short(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// The activation a GEMV multiplies, after its prologue op:
//   LMC_PRO_NONE     x
//   LMC_PRO_LAYERNORM (x - mean) * rstd * w + b      (src/ops.c:47-59)
//   LMC_PRO_RMSNORM  (w * rs) * x                    (src/ops_llama.c:24-33)
//   LMC_PRO_SWIGLU   silu(x) * x2                    (src/ops_llama.c:150-151)
// so the norm / gate that precedes a projection needs no kernel of its own.
// x (and x2, w, b) are read through the non-coherent path: they were written
// by earlier kernels and nothing writes them during this one.
struct XView {
    const float *x, *x2, *w, *b;
    int ldx, pro;
    const float *mean, *rstd;  // per batch row (shared memory)
    __device__ __forceinline__ float4 raw4(int bi, int k) const {
        return __ldg(reinterpret_cast<const float4 *>(x + (size_t)bi * ldx + k));
    }
    __device__ __forceinline__ float4 at4(int bi, int k) const {
        const float4 v = raw4(bi, k);
        if (pro == LMC_PRO_NONE) return v;
        if (pro == LMC_PRO_SWIGLU) {
            const float4 u = __ldg(reinterpret_cast<const float4 *>(x2 + (size_t)bi * ldx + k));
            return make_float4(silu_short(v.x) * u.x, silu_short(v.y) * u.y, silu_short(v.z) * u.z,
                               silu_short(v.w) * u.w);
        }
        const float4 ww = __ldg(reinterpret_cast<const float4 *>(w + k));
        if (pro == LMC_PRO_RMSNORM) {
            const float r = rstd[bi];
            return make_float4(ww.x * r * v.x, ww.y * r * v.y, ww.z * r * v.z, ww.w * r * v.w);
        }
        const float4 bb = __ldg(reinterpret_cast<const float4 *>(b + k));
        const float m = mean[bi], r = rstd[bi];
        return make_float4((v.x - m) * r * ww.x + bb.x, (v.y - m) * r * ww.y + bb.y, (v.z - m) * r * ww.z + bb.z,
                           (v.w - m) * r * ww.w + bb.w);
    }
};

// CTA-wide reduction of N values per thread (sum or max); every thread gets
// the results.  `red` holds N * WARPS floats.
template <int N, bool MAX>
__device__ __forceinline__ void cta_reduce(float (&v)[N], float *red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < N; i++) v[i] = MAX ? warp_max(v[i]) : warp_sum(v[i]);
    __syncthreads();  // red is free
    if (lane == 0)
#pragma unroll
        for (int i = 0; i < N; i++) red[i * WARPS + wid] = v[i];
    __syncthreads();
#pragma unroll
    for (int i = 0; i < N; i++) {
        float t = red[i * WARPS];
#pragma unroll
        for (int w = 1; w < WARPS; w++) t = MAX ? fmaxf(t, red[i * WARPS + w]) : t + red[i * WARPS + w];
        v[i] = t;
    }
}

// Quantize the (prologue-transformed) x into B fragments and per-chunk sums.
// Each task (chunk q, batch row b, c) handles the 8 (k32) or 4 (k16) columns
// of lane column c and writes all three limbs; the 4 tasks of a chunk are
// adjacent lanes, so the chunk's integer sum is a 2-step shuffle.
template <int NT, int QT, int RX>
__device__ __forceinline__ void build_x(uint8_t *smem, const Smem<NT, QT> &L, const TArgs &a) {
    constexpr int NB = 2 * NT, CH = Smem<NT, QT>::CH, SPAN = QT == 6 ? 16 : 32;
    float *scl = reinterpret_cast<float *>(smem + L.sc_off());
    float *inv = scl + 8, *mean = inv + 8, *rstd = mean + 8;
    float *red = reinterpret_cast<float *>(smem + L.red_off());
    const int tid = threadIdx.x;
    const int K = a.KB * 256, nb = a.nb;
    const XView xv{a.x, a.x2, a.pw, a.pb, a.ldx, a.pro, mean, rstd};
    if (a.pro == LMC_PRO_LAYERNORM || a.pro == LMC_PRO_RMSNORM) {  // per-row statistics
        float s[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) s[b] = 0.0f;
#pragma unroll 4
        for (int k = tid * 4; k < K; k += NTHR * 4)
#pragma unroll
            for (int b = 0; b < NB; b++)
                if (b < nb) {
                    const float4 v = xv.raw4(b, k);
                    s[b] += a.pro == LMC_PRO_RMSNORM ? v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w
                                                     : v.x + v.y + v.z + v.w;
                }
        cta_reduce<NB, false>(s, red);
        float mu[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) mu[b] = a.pro == LMC_PRO_RMSNORM ? 0.0f : s[b] / (float)K;
        if (a.pro == LMC_PRO_LAYERNORM) {  // two-pass variance, as src/ops.c:52-54
#pragma unroll
            for (int b = 0; b < NB; b++) s[b] = 0.0f;
#pragma unroll 4
            for (int k = tid * 4; k < K; k += NTHR * 4)
#pragma unroll
                for (int b = 0; b < NB; b++)
                    if (b < nb) {
                        const float4 v = xv.raw4(b, k);
                        const float d0 = v.x - mu[b], d1 = v.y - mu[b], d2 = v.z - mu[b], d3 = v.w - mu[b];
                        s[b] += d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3;
                    }
            cta_reduce<NB, false>(s, red);
        }
        if (tid < NB) {
#pragma unroll
            for (int b = 0; b < NB; b++)
                if (tid == b) {
                    mean[b] = mu[b];
                    rstd[b] = 1.0f / sqrtf(s[b] / (float)K + (a.pro == LMC_PRO_RMSNORM ? a.eps : 1e-5f));
                }
        }
        __syncthreads();
    }
    // Tasks: t = 4 q + c covers, for every batch row, the columns
    // k0 + 0..3 (and k0 + 16..19 for the k32 formats) of chunk q, with
    // k0 = 256 (q / CH) + SPAN (q % CH) + 4 c: exactly the B-fragment bytes of
    // lane column group c.  The task count is a multiple of 32, so every warp
    // runs the loops uniformly (shuffles are safe).  For one or two batch rows
    // a thread's first task stays in registers between the two passes.
    constexpr int TV = QT == 6 ? 4 : 8;
    const int ntask = a.KB * CH * 4;
    auto load_task = [&](int t, int b, float (&v)[TV]) {
        const int c = t & 3, q = t >> 2;
        const int k0 = (q / CH) * 256 + SPAN * (q % CH) + 4 * c;
        const float4 x0 = xv.at4(b, k0);
        v[0] = x0.x, v[1] = x0.y, v[2] = x0.z, v[3] = x0.w;
        if (TV == 8) {
            const float4 x1 = xv.at4(b, k0 + 16);
            v[TV - 4] = x1.x, v[TV - 3] = x1.y, v[TV - 2] = x1.z, v[TV - 1] = x1.w;
        }
    };
    constexpr int NC0 = NT == 1 ? NB : 1;
    float c0[NC0][TV];
#pragma unroll
    for (int b = 0; b < NC0; b++)
#pragma unroll
        for (int i = 0; i < TV; i++) c0[b][i] = 0.0f;
    // pass 1: max |x| per batch row -> fixed-point scale 2^(22-e), max|x| < 2^e
    float m[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) m[b] = 0.0f;
    // RX > 0 (rows of one batch row with more than two tasks a thread):
    // every task of this thread, up to RX of them, stays in registers, all
    // its loads in flight at once, and pass 2 reads them back instead of
    // going to L2 again.  The host picks RX = 4 for three or four tasks a
    // thread and RX = rx_tasks(QT) above that, only when nb == 1.
    constexpr int MT = RX > 0 ? RX : 1;
    const bool regs = RX > 0 && nb == 1 && ntask <= MT * NTHR;
    float cv[MT][TV];
    if (RX > 0 && regs) {
#pragma unroll
        for (int jt = 0; jt < MT; jt++) {
            const int t = tid + jt * NTHR;
            if (t < ntask) {
                load_task(t, 0, cv[jt]);
            } else {
#pragma unroll
                for (int i = 0; i < TV; i++) cv[jt][i] = 0.0f;
            }
        }
#pragma unroll
        for (int jt = 0; jt < MT; jt++)
#pragma unroll
            for (int i = 0; i < TV; i++) m[0] = fmaxf(m[0], fabsf(cv[jt][i]));
    }
#pragma unroll 2
    for (int t = regs ? ntask : tid; t < ntask; t += NTHR) {
#pragma unroll
        for (int b = 0; b < NB; b++)
            if (b < nb) {
                float v[TV];
                load_task(t, b, v);
#pragma unroll
                for (int i = 0; i < TV; i++) m[b] = fmaxf(m[b], fabsf(v[i]));
                if (NT == 1 && t == tid)
#pragma unroll
                    for (int i = 0; i < TV; i++) c0[b < NC0 ? b : 0][i] = v[i];
            }
    }
    cta_reduce<NB, true>(m, red);
    float sc[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) {
        // e = frexp exponent of m (m < 2^e), from the float's bits; clamped so
        // that the scale stays finite for vectors of tiny values
        const int e = max((int)((__float_as_uint(m[b]) >> 23) & 0xFF) - 126, -100);
        sc[b] = m[b] > 0.0f ? __uint_as_float((uint32_t)(127 + 22 - e) << 23) : 1.0f;
        if (tid == 0) {
            scl[b] = sc[b];
            inv[b] = m[b] > 0.0f ? __uint_as_float((uint32_t)(127 - 22 + e) << 23) : 0.0f;
        }
    }
    // pass 2: limbs into the fragments, integer chunk sums (rows >= nb are zero)
    int *xs = reinterpret_cast<int *>(smem + L.xs_off());
    auto quant_task = [&](int t, int b, const float (&v)[TV]) {
        const int c = t & 3, q = t >> 2;
        {
            uint32_t r[2][3] = {{0u, 0u, 0u}, {0u, 0u, 0u}};
            int isum = 0;
#pragma unroll
            for (int i = 0; i < TV; i++) {
                const int xi = __float2int_rn(v[i] * sc[b]);
                const int l0 = (int)(int8_t)(xi & 0xFF), rr = (xi - l0) >> 8, l1 = (int)(int8_t)(rr & 0xFF);
                r[i >> 2][0] |= (uint32_t)(l0 & 0xFF) << (8 * (i & 3));
                r[i >> 2][1] |= (uint32_t)(l1 & 0xFF) << (8 * (i & 3));
                r[i >> 2][2] |= (uint32_t)(((rr - l1) >> 8) & 0xFF) << (8 * (i & 3));
                isum += xi;
            }
            const int nt = b >> 1, g0 = 3 * (b & 1);
            const int kb = q / CH, j = q % CH;
            uint8_t *blk = smem + ((kb * NT + nt) * a.XL) * XSTR + j * (QT == 6 ? 4 : 8);
#pragma unroll
            for (int limb = 0; limb < 3; limb++) {
                const int li = (g0 + limb) * 4 + c;  // fragment lane: column g0 + limb, k group c
                if (li < a.XL) {
                    if (QT == 6) *reinterpret_cast<uint32_t *>(blk + li * XSTR) = r[0][limb];
                    else *reinterpret_cast<uint2 *>(blk + li * XSTR) = make_uint2(r[0][limb], r[1][limb]);
                }
            }
            if (QT != 8) {
                isum += __shfl_xor_sync(0xffffffffu, isum, 1);
                isum += __shfl_xor_sync(0xffffffffu, isum, 2);
                if (c == 0) xs[(size_t)q * NB + b] = isum;
            }
        }
    };
    if (RX > 0 && regs) {  // task counts are multiples of 32: warps stay uniform (shuffles above)
        float z[TV];
#pragma unroll
        for (int i = 0; i < TV; i++) z[i] = 0.0f;
#pragma unroll
        for (int jt = 0; jt < MT; jt++) {
            const int t = tid + jt * NTHR;
            if (t < ntask) {
                quant_task(t, 0, cv[jt]);
#pragma unroll
                for (int b = 1; b < NB; b++) quant_task(t, b, z);
            }
        }
    } else {
        for (int t = tid; t < ntask; t += NTHR) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float v[TV];
#pragma unroll
                for (int i = 0; i < TV; i++) v[i] = 0.0f;
                if (b < nb) {
                    if (NT == 1 && t == tid) {
#pragma unroll
                        for (int i = 0; i < TV; i++) v[i] = c0[b < NC0 ? b : 0][i];
                    } else {
                        load_task(t, b, v);
                    }
                }
                quant_task(t, b, v);
            }
        }
    }
    if (QT == 8) return;
    // pass 3: B fragments of the correction MMA.  Its k index is the chunk of
    // the unit (8 sub-blocks for Q4_K, 16 for Q6_K) and its columns n = 4 bb +
    // l are the 4 int8 limbs l of the chunk sum X (|X| < 2^27) of batch row
    // 2 nt + bb, so one m16n8k32 per unit gives sum_chunk A'(row, chunk) X.
    __syncthreads();
    const uint32_t *xsu = reinterpret_cast<const uint32_t *>(xs);
    uint32_t *xm = reinterpret_cast<uint32_t *>(smem + L.xm_off());
    for (int w = tid; w < a.KB * NT * 32; w += NTHR) {
        const int ln = w & 31, kbnt = w >> 5, kb = kbnt / NT, nt = kbnt % NT;
        const int n = ln >> 2, c = ln & 3, b = 2 * nt + (n >> 2), l = n & 3;
        uint32_t word = 0;
        if (4 * c < CH)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int X = (int)xsu[(size_t)(kb * CH + 4 * c + i) * NB + b];
                const int l0 = (int)(int8_t)(X & 0xFF), r1 = (X - l0) >> 8;
                const int l1 = (int)(int8_t)(r1 & 0xFF), r2 = (r1 - l1) >> 8;
                const int l2 = (int)(int8_t)(r2 & 0xFF), l3 = (r2 - l2) >> 8;
                const int v = l == 0 ? l0 : l == 1 ? l1 : l == 2 ? l2 : l3;
                word |= (uint32_t)(v & 0xFF) << (8 * i);
            }
        xm[w] = word;
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
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(65536u)
        : "memory");
    return ok != 0;
}
// Bounded wait: each poll suspends the warp until the phase completes or
// about 64 us pass; after 2^14 polls (about one second) it gives up, records
// the timeout and lets the caller skip the unit.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t t = 0; t < (1u << 14); t++)
        if (mbar_try(bar, parity)) return true;
    atomicExch(&g_tiled_timeout, 1);
    return false;
}

// Pull one 128-byte line into this SM's L1 (a hint; no value is returned).
__device__ __forceinline__ void prefetch_l1(const void *p) { asm volatile("prefetch.global.L1 [%0];" ::"l"(p)); }

// cluster helpers (distributed shared memory)
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
__device__ __forceinline__ void red_cluster_add(uint32_t local_addr, uint32_t rank, float v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
    asm volatile("red.shared::cluster.add.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// Per-warp partial of the row tile currently being streamed:
//   tot[nt][i]  sum over units of (block scale d) x (int32 sum over chunks of
//               sub-scale x chunk product), C fragment element i (rows g / g+8,
//               columns 2c, 2c+1)
//   cor[nt][i]  corrections (Q4_K mins, Q6_K -32 offsets): C fragment element
//               i of the correction MMA, whose columns are 4 limbs per batch row
template <int NT> struct Part {
    float tot[NT][4];
    float cor[NT][4];
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) tot[nt][i] = cor[nt][i] = 0.0f;
    }
};

// Add a warp's partial into the CTA accumulator of its row tile: combine
// the limb columns (weights 1, 2^8, 2^16), subtract the corrections, scale by
// the vector's inverse scale, reduce the quad, one shared atomic per value.
template <int NT>
__device__ __forceinline__ void flush(const Part<NT> &p, float *acc_rt, const float *inv, int nb, int lane) {
    const int g = lane >> 2, c = lane & 3;
    // lane column group c holds C columns 2c, 2c+1 = (batch 0/1 of the tile, limb):
    // c=0: (0,L0) (0,L1); c=1: (0,L2) (1,L0); c=2: (1,L1) (1,L2); c=3: unused
    const float w0 = c == 0 ? 1.0f : c == 1 ? 65536.0f : c == 2 ? 0.0f : 0.0f;      // column 2c   -> batch 0
    const float w1 = c == 0 ? 256.0f : 0.0f;                                       // column 2c+1 -> batch 0
    const float v0 = c == 2 ? 256.0f : 0.0f;                                       // column 2c   -> batch 1
    const float v1 = c == 1 ? 1.0f : c == 2 ? 65536.0f : 0.0f;                     // column 2c+1 -> batch 1
    // correction columns 2c, 2c+1 = (batch c/2, limbs 2(c&1), 2(c&1)+1)
    const float cw0 = (c & 1) ? 65536.0f : 1.0f, cw1 = (c & 1) ? 16777216.0f : 256.0f;
    const bool cb1 = c >= 2;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const float k0 = cw0 * p.cor[nt][0] + cw1 * p.cor[nt][1], k1 = cw0 * p.cor[nt][2] + cw1 * p.cor[nt][3];
        float y0[2][2];  // [batch in tile][row half], compile-time indices only
        y0[0][0] = w0 * p.tot[nt][0] + w1 * p.tot[nt][1] - (cb1 ? 0.0f : k0);
        y0[0][1] = w0 * p.tot[nt][2] + w1 * p.tot[nt][3] - (cb1 ? 0.0f : k1);
        y0[1][0] = v0 * p.tot[nt][0] + v1 * p.tot[nt][1] - (cb1 ? k0 : 0.0f);
        y0[1][1] = v0 * p.tot[nt][2] + v1 * p.tot[nt][3] - (cb1 ? k1 : 0.0f);
#pragma unroll
        for (int bb = 0; bb < 2; bb++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int b = 2 * nt + bb;
                float v = inv[b] * y0[bb][h];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                if (c == 2 * bb + h && b < nb) atomicAdd(acc_rt + b * 16 + g + 8 * h, v);
            }
    }
}

// Stores output (b, row) and returns its greedy-pick key (0 when out of range).
__device__ __forceinline__ unsigned long long epilogue(const TArgs &a, int b, int row, float v) {
    if (row >= a.M || b >= a.nb) return 0ull;
    if (a.bias) v += a.bias[row];
    if (a.epi & LMC_EPI_GELU) v = lmc_gelu_f(v);
    float *o = a.y + (size_t)b * a.ldy + row;
    *o = (a.epi & LMC_EPI_ACCUM) ? *o + v : v;
    return lmc_argmax_key(v, row + a.key_base);
}
// Outputs e = lane + 32 j of a row tile (e < 16 nb: batch row e / 16, tile row
// e % 16); best[j] keeps the largest key this lane has seen for batch row
// 2 j + lane / 16.
__device__ __forceinline__ void epilogue_tile(const TArgs &a, int row0, const float *ar, int lane,
                                              unsigned long long (&best)[4]) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int e = lane + 32 * j;
        if (e < 16 * a.nb) {
            const unsigned long long k = epilogue(a, e >> 4, row0 + (e & 15), ar[e]);
            best[j] = k > best[j] ? k : best[j];
        }
    }
}

// Byte i of w, zero-extended / sign-extended (one PRMT each).
template <int I> __device__ __forceinline__ int ubyte_c(uint32_t w) { return (int)__byte_perm(w, 0u, 0x4440u + I); }
template <int I> __device__ __forceinline__ int sbyte_c(uint32_t w) {
    int r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "n"(I | ((8 | I) << 4) | ((8 | I) << 8) | ((8 | I) << 12)));
    return r;
}
template <int J> __device__ __forceinline__ uint32_t pick4(const uint4 &v) {
    return J == 0 ? v.x : J == 1 ? v.y : J == 2 ? v.z : v.w;
}

// The unit kernels below get: u = the unit's ring slot, xb = this lane's
// B-fragment words for the unit column (n-tile nt at xb + nt * xs), xm = this
// lane's correction B word (n-tile nt at xm + 32 nt).  Lanes whose MMA
// column carries no batch row read whatever follows their block (inside
// shared memory); their C columns are never used.

// Q4_K unit (src/quant.c:275-303): d * sum_sub sc * (sum_32 q x) - dmin * sum_sub m * X_sub
template <int NT>
__device__ __forceinline__ void unit_q4k(Part<NT> &p, const uint8_t *u, const uint8_t *xb, int xs, const uint32_t *xm,
                                         int lane) {
    const int g = lane >> 2, c = lane & 3;
    const uint4 H0 = *reinterpret_cast<const uint4 *>(u + 16 * g);
    const uint4 H1 = *reinterpret_cast<const uint4 *>(u + 16 * g + 128);
    const uint4 *cw = reinterpret_cast<const uint4 *>(u + 256) + lane;
    const uint4 q0 = cw[0], q1 = cw[32], q2 = cw[64], q3 = cw[96];
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
    uint4 B[NT];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        if ((j & 1) == 0)
#pragma unroll
            for (int nt = 0; nt < NT; nt++) B[nt] = *reinterpret_cast<const uint4 *>(xb + nt * xs + 8 * j);
        int s0, s1;
        switch (j) {
        case 0: s0 = ubyte_c<0>(sc0a), s1 = ubyte_c<0>(sc1a); break;
        case 1: s0 = ubyte_c<1>(sc0a), s1 = ubyte_c<1>(sc1a); break;
        case 2: s0 = ubyte_c<2>(sc0a), s1 = ubyte_c<2>(sc1a); break;
        case 3: s0 = ubyte_c<3>(sc0a), s1 = ubyte_c<3>(sc1a); break;
        case 4: s0 = ubyte_c<0>(sc0b), s1 = ubyte_c<0>(sc1b); break;
        case 5: s0 = ubyte_c<1>(sc0b), s1 = ubyte_c<1>(sc1b); break;
        case 6: s0 = ubyte_c<2>(sc0b), s1 = ubyte_c<2>(sc1b); break;
        default: s0 = ubyte_c<3>(sc0b), s1 = ubyte_c<3>(sc1b); break;
        }
        const uint32_t P = qs[2 * j], Q = qs[2 * j + 1];
        const uint32_t a0 = P & LO4, a2 = (P >> 4) & LO4, a1 = Q & LO4, a3 = (Q >> 4) & LO4;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const uint32_t b0 = (j & 1) ? B[nt].z : B[nt].x, b1 = (j & 1) ? B[nt].w : B[nt].y;
            int acc[4];
            imma_k32(acc, a0, a1, a2, a3, b0, b1);
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
    // mins: one MMA over the 8 sub-blocks (k) against the limbs of X_sub; A'
    // row g / g+8 holds m_0..m_3 in lanes c = 0 and m_4..m_7 in lanes c = 1
    // (src/quant.c:44-53 packing), zero elsewhere
    const uint32_t m0a = H0.z & 0x3F3F3F3Fu, m0b = ((H0.w >> 4) & LO4) | ((H0.z >> 2) & 0x30303030u);
    const uint32_t m1a = H1.z & 0x3F3F3F3Fu, m1b = ((H1.w >> 4) & LO4) | ((H1.z >> 2) & 0x30303030u);
    const uint32_t ma0 = c == 0 ? m0a : c == 1 ? m0b : 0u, ma1 = c == 0 ? m1a : c == 1 ? m1b : 0u;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        int mc[4];
        imma_k32(mc, ma0, ma1, 0u, 0u, xm[32 * nt], 0u);
        p.cor[nt][0] += dd0.y * (float)mc[0];
        p.cor[nt][1] += dd0.y * (float)mc[1];
        p.cor[nt][2] += dd1.y * (float)mc[2];
        p.cor[nt][3] += dd1.y * (float)mc[3];
    }
}

// Q6_K unit (src/quant.c:386-414): d * sum_chunks sc * (sum_16 q x - 32 X_chunk)
template <int NT>
__device__ __forceinline__ void unit_q6k(Part<NT> &p, const uint8_t *u, const uint8_t *xb, int xs, const uint32_t *xm,
                                         int lane) {
    const int g = lane >> 2, c = lane & 3;
    const uint4 s0v = *reinterpret_cast<const uint4 *>(u + 16 * g);
    const uint4 s1v = *reinterpret_cast<const uint4 *>(u + 16 * g + 128);
    const float d0 = __half2float(*reinterpret_cast<const __half *>(u + 256 + 2 * g));
    const float d1 = __half2float(*reinterpret_cast<const __half *>(u + 256 + 2 * g + 16));
    const uint4 *lw = reinterpret_cast<const uint4 *>(u + 288) + lane;
    const uint4 *hw = reinterpret_cast<const uint4 *>(u + 288 + 2048) + lane;
    const uint4 q0 = lw[0], q1 = lw[32], q2 = lw[64], q3 = lw[96];
    const uint4 hq0 = hw[0], hq1 = hw[32];
    const uint32_t lo[16] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w,
                             q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
    const uint32_t hs[8] = {hq0.x, hq0.y, hq0.z, hq0.w, hq1.x, hq1.y, hq1.z, hq1.w};
    int it[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) it[nt][i] = 0;
    uint4 B[NT];
#pragma unroll
    for (int j = 0; j < 16; j++) {
        if ((j & 3) == 0)
#pragma unroll
            for (int nt = 0; nt < NT; nt++) B[nt] = *reinterpret_cast<const uint4 *>(xb + nt * xs + 4 * j);
        int s0, s1;
        const uint32_t w0 = j < 4 ? s0v.x : j < 8 ? s0v.y : j < 12 ? s0v.z : s0v.w;
        const uint32_t w1 = j < 4 ? s1v.x : j < 8 ? s1v.y : j < 12 ? s1v.z : s1v.w;
        switch (j & 3) {
        case 0: s0 = sbyte_c<0>(w0), s1 = sbyte_c<0>(w1); break;
        case 1: s0 = sbyte_c<1>(w0), s1 = sbyte_c<1>(w1); break;
        case 2: s0 = sbyte_c<2>(w0), s1 = sbyte_c<2>(w1); break;
        default: s0 = sbyte_c<3>(w0), s1 = sbyte_c<3>(w1); break;
        }
        const uint32_t H = hs[j >> 1], P = lo[j];
        const uint32_t tg = ((j & 1) ? H : (H << 4)) & 0x30303030u;
        const uint32_t tg8 = ((j & 1) ? (H >> 2) : (H << 2)) & 0x30303030u;
        const uint32_t a0 = (P & LO4) | tg, a1 = ((P >> 4) & LO4) | tg8;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const uint32_t bx = (j & 3) == 0 ? B[nt].x : (j & 3) == 1 ? B[nt].y : (j & 3) == 2 ? B[nt].z : B[nt].w;
            int acc[4];
            imma_k16(acc, a0, a1, bx);
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
    // -32 offsets: one MMA over the 16 chunks (k) against the limbs of
    // X_chunk; A' row g / g+8 = the row's int8 scales (lane c: chunks 4c..4c+3)
    const uint32_t swc0 = c == 0 ? s0v.x : c == 1 ? s0v.y : c == 2 ? s0v.z : s0v.w;
    const uint32_t swc1 = c == 0 ? s1v.x : c == 1 ? s1v.y : c == 2 ? s1v.z : s1v.w;
    const float f0 = 32.0f * d0, f1 = 32.0f * d1;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        int mc[4];
        imma_k32(mc, swc0, swc1, 0u, 0u, xm[32 * nt], 0u);
        p.cor[nt][0] += f0 * (float)mc[0];
        p.cor[nt][1] += f0 * (float)mc[1];
        p.cor[nt][2] += f1 * (float)mc[2];
        p.cor[nt][3] += f1 * (float)mc[3];
    }
}

// Q8_0 unit (src/quant.c:419-429): sum_blocks d * (sum_32 q x)
template <int NT>
__device__ __forceinline__ void unit_q80(Part<NT> &p, const uint8_t *u, const uint8_t *xb, int xs, int lane) {
    const int g = lane >> 2;
    const uint4 H0 = *reinterpret_cast<const uint4 *>(u + 16 * g);
    const uint4 H1 = *reinterpret_cast<const uint4 *>(u + 16 * g + 128);
    const uint4 *cw = reinterpret_cast<const uint4 *>(u + 256) + lane;
    uint4 B[NT];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        if ((j & 1) == 0)
#pragma unroll
            for (int nt = 0; nt < NT; nt++) B[nt] = *reinterpret_cast<const uint4 *>(xb + nt * xs + 8 * j);
        const uint4 A = cw[32 * j];
        const uint32_t hw0 = j < 2 ? H0.x : j < 4 ? H0.y : j < 6 ? H0.z : H0.w;
        const uint32_t hw1 = j < 2 ? H1.x : j < 4 ? H1.y : j < 6 ? H1.z : H1.w;
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&hw0));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&hw1));
        const float d0 = (j & 1) ? f0.y : f0.x, d1 = (j & 1) ? f1.y : f1.x;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const uint32_t b0 = (j & 1) ? B[nt].z : B[nt].x, b1 = (j & 1) ? B[nt].w : B[nt].y;
            int acc[4];
            imma_k32(acc, A.x, A.y, A.z, A.w, b0, b1);
            p.tot[nt][0] += d0 * (float)acc[0];
            p.tot[nt][1] += d0 * (float)acc[1];
            p.tot[nt][2] += d1 * (float)acc[2];
            p.tot[nt][3] += d1 * (float)acc[3];
        }
    }
}

// Refill of a ring slot, issued by lane 0 under a predicate (no divergent
// branch in the streaming loop): expect the bytes, start the bulk copy, and
// optionally pull a unit further ahead into L2.
__device__ __forceinline__ void refill(bool leader, uint64_t *bar, void *dst, const void *src, uint32_t bytes,
                                       const void *pf_src, bool pf) {
    asm volatile(
        "{ .reg .pred p, q;\n\t"
        "setp.ne.u32 p, %0, 0;\n\t"
        "setp.ne.and.u32 q, %5, 0, p;\n\t"
        "@p mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %2;\n\t"
        "@p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%3], [%4], %2, [%1];\n\t"
        "@q cp.async.bulk.prefetch.L2.global [%6], %2;\n\t"
        "}" ::"r"((uint32_t)leader),
        "r"(smem_u32(bar)), "r"(bytes), "r"(smem_u32(dst)), "l"(src), "r"((uint32_t)pf), "l"(pf_src)
        : "memory");
}

// The streaming GEMV.  Cluster c owns row tiles [c*RT/NC, (c+1)*RT/NC); its
// Uc units (row-tile major) are split into CL contiguous CTA ranges, and each
// CTA's range into WARPS contiguous warp ranges.  A warp streams its units
// through a `stages`-deep ring of bulk async copies (global -> shared),
// started before pdl_wait() (weights do not depend on earlier kernels), and
// adds each finished row tile into the CTA accumulator.  Then every row tile
// is completed by the CTA holding its first unit: partial tiles of the other
// CTAs are added into it through distributed shared memory.
template <int NT, int QT, int RX>
__global__ void __launch_bounds__(NTHR, 2) k_gemv_tiled(TArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NB = 2 * NT, UNIT = unit_bytes(QT);
    const Smem<NT, QT> L{a.KB, a.XL, a.maxrt, a.stages};
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int rank = a.CL > 1 ? (int)cluster_rank() : 0;
    const int cid = a.CL > 1 ? (int)cluster_id_x() : (int)blockIdx.x;
    const int t0 = (int)((long long)cid * a.RT / a.NC), t1 = (int)((long long)(cid + 1) * a.RT / a.NC);
    const int Uc = (t1 - t0) * a.KB;  // units of this cluster
    const int cu0 = (int)((long long)rank * Uc / a.CL), cu1 = (int)((long long)(rank + 1) * Uc / a.CL);
    const int w0 = cu0 + (int)((long long)(cu1 - cu0) * wid / WARPS);
    const int w1 = cu0 + (int)((long long)(cu1 - cu0) * (wid + 1) / WARPS);
    const int stages = a.stages, KB = a.KB, pf = a.pf;
    const uint8_t *wbase = a.w + (size_t)t0 * KB * UNIT;  // cluster-local unit 0
    uint8_t *ring = smem + L.ring_off() + wid * stages * UNIT;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off()) + wid * stages;
    if (lane == 0) {
        for (int s = 0; s < stages; s++) mbar_init(&bars[s]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    pdl_launch_dependents();
    if (lane == 0) {  // weights only: stream while the previous kernel finishes
        for (int s = 0; s < stages && w0 + s < w1; s++)
            issue_unit(&bars[s], ring + s * UNIT, wbase + (size_t)(w0 + s) * UNIT, UNIT);
        // and the next `pf` units of this warp into L2, so HBM keeps streaming
        // through the dependent wait, the activation setup and the ring refills
        const int p0 = w0 + stages, p1 = min(w1, p0 + pf);
        for (int q = p0; q < p1; q++) prefetch_l2(wbase + (size_t)q * UNIT, UNIT);
    }
    float *acc = reinterpret_cast<float *>(smem + L.acc_off());
    for (int i = threadIdx.x; i < a.maxrt * NB * 16; i += NTHR) acc[i] = 0.0f;
    if (a.CL > 1) cluster_arrive();  // this CTA's accumulator is zero (phase 1)
    if (a.pro == LMC_PRO_LAYERNORM || a.pro == LMC_PRO_RMSNORM)  // norm weights: independent of the previous kernel
        for (int k = threadIdx.x * 32; k < a.KB * 256; k += NTHR * 32) {
            prefetch_l1(a.pw + k);
            if (a.pb) prefetch_l1(a.pb + k);
        }
    pdl_wait();
    build_x<NT, QT, RX>(smem, L, a);
    __syncthreads();
    const float *inv = reinterpret_cast<const float *>(smem + L.sc_off()) + 8;
    const int XS = a.XL * XSTR;                         // bytes per (kb, nt) fragment block
    const uint8_t *xbl = smem + lane * XSTR;            // this lane's fragments, block 0
    const uint32_t *xml = reinterpret_cast<const uint32_t *>(smem + L.xm_off()) + lane;
    const int rt0 = cu0 / KB;  // cluster-local row tile of accumulator slot 0
    Part<NT> p;
    p.zero();
    int cur = -1;
    bool ok = true;
    // unit i = rt * KB + kb lives in ring slot s, k-th refill of it (parity k & 1);
    // all advanced incrementally (no divisions in the loop)
    int rt = w0 / KB, kb = w0 - rt * KB, s = 0, i = w0;
    uint32_t parity = 0;
    for (; i < w1; i++) {
        if (!mbar_wait(&bars[s], parity)) {
            ok = false;
            break;
        }
        if (rt != cur) {
            if (cur >= 0) flush<NT>(p, acc + (cur - rt0) * NB * 16, inv, a.nb, lane);
            p.zero();
            cur = rt;
        }
        const uint8_t *u = ring + s * UNIT;
        const uint8_t *xb = xbl + kb * NT * XS;
        if (QT == 4) unit_q4k<NT>(p, u, xb, XS, xml + kb * NT * 32, lane);
        else if (QT == 6) unit_q6k<NT>(p, u, xb, XS, xml + kb * NT * 32, lane);
        else unit_q80<NT>(p, u, xb, XS, lane);
        __syncwarp();
        // every lane has consumed its reads of the slot (their values fed the
        // MMAs above) before the warp barrier, so the refill may overwrite it
        if (i + stages < w1)
            refill(lane == 0, &bars[s], ring + s * UNIT, wbase + (size_t)(i + stages) * UNIT, UNIT,
                   wbase + (size_t)(i + stages + pf) * UNIT, i + stages + pf < w1);
        if (++kb == KB) { kb = 0; rt++; }
        if (++s == stages) { s = 0; parity ^= 1u; }
    }
    if (cur >= 0 && ok) flush<NT>(p, acc + (cur - rt0) * NB * 16, inv, a.nb, lane);
    if (!ok && lane == 0) {
        // a bounded wait gave up at unit i: wait (bounded) for the copies this
        // warp still has in flight, i.e. the last phase of every slot it issued
        const int end = min(w1, i + stages);
        for (int q = max(w0, end - stages); q < end; q++)
            (void)mbar_wait(&bars[(q - w0) % stages], (uint32_t)(((q - w0) / stages) & 1));
    }
    __syncthreads();
    if (a.CL > 1) cluster_wait();  // every accumulator of the cluster is zero
    // Row tiles of this CTA: finish the ones it holds whole, push the ones
    // that started in an earlier CTA into that CTA's accumulator.
    unsigned long long best[4] = {0ull, 0ull, 0ull, 0ull};
    const int rt_last = cu1 > cu0 ? (cu1 - 1) / KB : rt0 - 1;
    for (int T = rt0 + wid; T <= rt_last; T += WARPS) {
        const float *ar = acc + (T - rt0) * NB * 16;
        const int f0 = T * KB, f1 = f0 + KB;
        if (f0 >= cu0) {
            if (f1 <= cu1) epilogue_tile(a, (t0 + T) * 16, ar, lane, best);
            continue;
        }
        const int owner = (int)(((long long)(f0 + 1) * a.CL - 1) / Uc);
        const int orow0 = (int)((long long)owner * Uc / a.CL) / KB;
        const uint32_t dst = smem_u32(acc + (T - orow0) * NB * 16);
        for (int e = lane; e < 16 * a.nb; e += 32) red_cluster_add(dst + 4 * e, (uint32_t)owner, ar[e]);
    }
    const bool own_shared = cu1 > cu0 && rt_last * KB >= cu0 && (rt_last + 1) * KB > cu1;
    if (a.CL > 1) {
        cluster_arrive();  // phase 2: pushes done
        cluster_wait();
    }
    if (own_shared && wid == 0)  // the tile this CTA owns and later CTAs added to
        epilogue_tile(a, (t0 + rt_last) * 16, acc + (rt_last - rt0) * NB * 16, lane, best);
    if (a.keys) {  // greedy keys: half-warp maxima, then one atomic per CTA and batch row
        // [WARPS][8] over the x fragments, dead once every unit is done
        auto kbest = reinterpret_cast<unsigned long long(*)[8]>(smem);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            unsigned long long k = best[j];
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) {
                const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
                k = o > k ? o : k;
            }
            if ((lane & 15) == 0) kbest[wid][2 * j + (lane >> 4)] = k;
        }
        __syncthreads();
        if ((int)threadIdx.x < a.nb) {
            unsigned long long k = 0ull;
            for (int w = 0; w < WARPS; w++) k = kbest[w][threadIdx.x] > k ? kbest[w][threadIdx.x] : k;
            if (k) atomicMax(a.keys + threadIdx.x, k);
        }
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
extern "C" int lmc_device_status(void) {
    int v = 0;
    LMC_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_tiled_timeout, sizeof(int)));
    const int g = lmc_gemm_status();
    if (g != LMC_OK && g != LMC_ERR_TIMEOUT) return g;
    if (!v && g == LMC_OK) return LMC_OK;
    const int zero = 0;
    LMC_CUDA_TRY(cudaMemcpyToSymbol(g_tiled_timeout, &zero, sizeof(int)));
    return lmc_set_error(LMC_ERR_TIMEOUT, "a kernel gave up a bounded wait (%s)",
                         v ? "bulk copy not completed" : "tensor-core MMA not completed");
}

static int qt_of(uint32_t type) { return type == LMC_TYPE_Q4_K ? 4 : type == LMC_TYPE_Q6_K ? 6 : 8; }

// the instantiations: NT in {1, 2, 4} x format
#define LMC_TILED_SWITCH(NT_, QT_, F)                                     \
    switch ((QT_) * 10 + (NT_)) {                                         \
    case 41: return F(1, 4);                                              \
    case 42: return F(2, 4);                                              \
    case 44: return F(4, 4);                                              \
    case 61: return F(1, 6);                                              \
    case 62: return F(2, 6);                                              \
    case 64: return F(4, 6);                                              \
    case 81: return F(1, 8);                                              \
    case 82: return F(2, 8);                                              \
    default: return F(4, 8);                                              \
    }
#define LMC_KERNEL_PTR(n, q) (const void *)k_gemv_tiled<n, q, 0>
static const void *kernel_for(int NT, int QT, int rx = 0) {
    if (rx == 4 && NT == 1) return QT == 4 ? (const void *)k_gemv_tiled<1, 4, 4>
                                   : QT == 6 ? (const void *)k_gemv_tiled<1, 6, 4>
                                             : (const void *)k_gemv_tiled<1, 8, 4>;
    if (rx > 4 && NT == 1) return QT == 4 ? (const void *)k_gemv_tiled<1, 4, rx_tasks(4)>
                                  : QT == 6 ? (const void *)k_gemv_tiled<1, 6, rx_tasks(6)>
                                            : (const void *)k_gemv_tiled<1, 8, rx_tasks(8)>;
    LMC_TILED_SWITCH(NT, QT, LMC_KERNEL_PTR)
}
static size_t smem_for(int NT, int QT, int KB, int XL, int maxrt, int stages) {
#define LMC_SMEM_TOTAL(n, q) Smem<n, q>{KB, XL, maxrt, stages}.total()
    LMC_TILED_SWITCH(NT, QT, LMC_SMEM_TOTAL)
#undef LMC_SMEM_TOTAL
}

struct Plan {
    int NT, XL, CL, NC, maxrt, stages;
    size_t smem;
};

// Clusters of `cl` CTAs that are resident at one CTA per SM (asked with a
// shared-memory size that allows only one CTA per SM); cached per device.
static int clusters_per_gpu(int cl) {
    static int cache[4][64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    const int li = cl == 1 ? 0 : cl == 2 ? 1 : cl == 4 ? 2 : 3;
    if (cache[li][dev]) return cache[li][dev];
    int n = 0;
    if (cl == 1) {
        n = lmc_sm_count();
    } else {
        const void *fn = kernel_for(1, 4);
        const size_t probe = 160 * 1024;
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)probe) == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(cl);
            cfg.blockDim = dim3(NTHR);
            cfg.dynamicSmemBytes = probe;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = cl;
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) n = 0;
        }
        (void)cudaGetLastError();
    }
    cache[li][dev] = n > 0 ? n : -1;
    return n > 0 ? n : -1;
}

// Cluster shape (fewest rounds of units for the busiest CTA, a split
// charged for its cluster synchronisation; ties go to more CTAs, then to
// smaller clusters), fragment width and ring depth for one launch.
static int plan_for(uint32_t type, int rows_tiled, int cols, int nb, Plan *P) {
    const int QT = qt_of(type), KB = cols / 256, RT = rows_tiled / 16;
    const int NT = nb <= 2 ? 1 : nb <= 4 ? 2 : 4;
    const int XL = NT == 1 ? 12 * nb : 24;
    const int unit = unit_bytes(QT);
    long long best = -1;
    Plan bestp = {};
    const int cls[4] = {1, 2, 4, 8};
    for (int ci = 0; ci < 4; ci++) {
        const int cl = cls[ci];
        const int cpg = clusters_per_gpu(cl);
        if (cpg <= 0) continue;
        const int NC = std::min(cpg, RT);
        const long long tiles = (RT + NC - 1) / NC;            // most row tiles of a cluster
        const long long per_cta = (tiles * KB + cl - 1) / cl;  // most units of a CTA
        const int maxrt = (int)((per_cta + KB - 1) / KB) + 1;
        // ring depth: the deepest with <= RING_TARGET bytes that keeps two
        // CTAs per SM, else the deepest within the one-CTA limit
        int stages = 0;
        size_t smem = 0;
        for (int pass = 0; pass < 2 && !stages; pass++)
            for (int st = 8; st >= 2; st--) {
                if (st > 2 && (size_t)st * WARPS * unit > RING_TARGET) continue;
                const size_t tot = smem_for(NT, QT, KB, XL, maxrt, st);
                if (tot <= (size_t)(pass == 0 ? SMEM_PAIR : SMEM_LIMIT)) {
                    stages = st;
                    smem = tot;
                    break;
                }
            }
        if (!stages) continue;
        // lower is better: rounds of units per warp of the busiest CTA (a
        // round ~0.3 us), plus ~5 rounds for a split's cluster barriers and
        // distributed-shared-memory pushes (measured 1.5-2.5 us), minus a
        // little per CTA engaged
        const long long rounds = (per_cta + WARPS - 1) / WARPS;
        const long long score = (rounds + (cl > 1 ? 5 : 0)) * 4096 - (long long)NC * cl * 8 + cl;
        if (best < 0 || score < best) {
            best = score;
            bestp = Plan{NT, XL, cl, NC, maxrt, stages, smem};
        }
    }
    if (best < 0) return LMC_ERR_UNSUPPORTED;
    *P = bestp;
    return LMC_OK;
}

extern "C" int lmc_tiled_build(lmc_qtensor *t) {
    t->tiled = NULL;
    if ((t->type != LMC_TYPE_Q4_K && t->type != LMC_TYPE_Q6_K && t->type != LMC_TYPE_Q8_0) || t->cols % 256)
        return LMC_OK;
    const int KB = t->cols / 256, RT = (t->rows + 15) / 16;
    Plan P;
    if (plan_for(t->type, RT * 16, t->cols, 1, &P)) return LMC_OK;  // very long rows: generic path
    const size_t bytes = (size_t)RT * KB * unit_bytes(qt_of(t->type));
    LMC_CUDA_TRY(cudaMalloc(&t->tiled, bytes));
    if (t->type == LMC_TYPE_Q4_K)
        k_repack_q4k<<<RT * KB, 32>>>((const uint8_t *)t->blocks, (uint8_t *)t->tiled, t->rows, KB);
    else if (t->type == LMC_TYPE_Q6_K)
        k_repack_q6k<<<RT * KB, 32>>>((const uint8_t *)t->blocks, (uint8_t *)t->tiled, t->rows, KB);
    else
        k_repack_q80<<<RT * KB, 32>>>((const uint8_t *)t->blocks, (uint8_t *)t->tiled, t->rows, KB);
    LMC_LAUNCH_CHECK("repack");
    LMC_CUDA_TRY(cudaDeviceSynchronize());
    t->tiled_bytes = bytes;
    t->tiled_rows = RT * 16;
    return LMC_OK;
}

static int launch_plan(const lmc_qtensor *t, TArgs a, const Plan &P, cudaStream_t s) {
    // one batch row whose activation tasks (32 per 256 columns, 64 for Q6_K)
    // come to more than two a thread: the register-held activation variant,
    // sized to the tasks (four slots, else the longest rows' rx_tasks; the
    // longest variant's unrolled code made three or four tasks slower than
    // the rolled loop).  Not behind a SwiGLU prologue: there the unrolled
    // gate arithmetic of all tasks made decode steps slower (the 8B model by
    // 6% at K = 14336, TinyLlama by 7% at K = 5632) than the rolled loop.
    const int QT = qt_of(t->type), ntask = a.KB * (QT == 6 ? 64 : 32);
    const int tpt = (ntask + NTHR - 1) / NTHR;
    const int rx = P.NT == 1 && a.nb == 1 && tpt > 2 && a.pro != LMC_PRO_SWIGLU
                       ? (tpt <= 4 ? 4 : tpt <= rx_tasks(QT) ? rx_tasks(QT) : 0)
                       : 0;
    const void *fn = kernel_for(P.NT, QT, rx);
    // dynamic shared-memory limit per kernel: only ever raised (lowering it
    // under a launch already queued on another stream is not allowed)
    static thread_local struct { const void *fn; size_t max_smem; } attr[16];
    bool done = false;
    for (auto &e : attr)
        if (e.fn == fn) {
            if (P.smem > e.max_smem) {
                LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P.smem));
                e.max_smem = P.smem;
            }
            done = true;
            break;
        }
    if (!done) {
        const size_t lim = std::max<size_t>(P.smem, 160 * 1024);
        LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lim));
        LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
        for (auto &e : attr)
            if (!e.fn) {
                e.fn = fn;
                e.max_smem = lim;
                break;
            }
    }
    a.XL = P.XL;
    a.CL = P.CL;
    a.NC = P.NC;
    a.maxrt = P.maxrt;
    a.stages = P.stages;
    {   // L2 prefetch window: up to PF_BYTES of this launch's weights ahead of the rings
        const long long ctas = (long long)P.NC * P.CL, unit = unit_bytes(qt_of(t->type));
        a.pf = (int)std::min<long long>(64, PF_BYTES / (ctas * WARPS * unit));
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P.NC * P.CL);
    cfg.blockDim = dim3(NTHR);
    cfg.dynamicSmemBytes = P.smem;
    cfg.stream = s;
    cudaLaunchAttribute at[3];
    int n = 0;
    if (lmc_pdl_enabled()) {
        at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[n].val.programmaticStreamSerializationAllowed = 1;
        n++;
    }
    if (P.CL > 1) {
        at[n].id = cudaLaunchAttributeClusterDimension;
        at[n].val.clusterDim.x = P.CL;
        at[n].val.clusterDim.y = 1;
        at[n].val.clusterDim.z = 1;
        n++;
        at[n].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
        at[n].val.clusterSchedulingPolicyPreference = cudaClusterSchedulingPolicySpread;
        n++;
    }
    cfg.attrs = at;
    cfg.numAttrs = n;
    void *args[1] = {&a};
    cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return lmc_set_error(LMC_ERR_CUDA, "tiled gemv launch: %s", cudaGetErrorString(e));
    return LMC_OK;
}

extern "C" int lmc_tiled_gemv_launch(const lmc_qtensor *t, const float *d_x, int ldx, const float *d_bias, float *d_y,
                                     int ldy, int batch, int epi, cudaStream_t s) {
    if (((uintptr_t)d_x & 15) || (ldx & 3))  // float4 activation loads
        return lmc_gemv_generic_launch(t->type, t->blocks, t->rows, t->cols, d_x, ldx, d_bias, d_y, ldy, batch, epi, s);
    lmc_gemv_extra ex = {LMC_PRO_NONE, NULL, NULL, NULL, 0.0f, NULL, 0};
    return lmc_tiled_gemv_ex(t, d_x, ldx, d_bias, d_y, ldy, batch, epi, &ex, s);
}

extern "C" int lmc_tiled_gemv_ex(const lmc_qtensor *t, const float *d_x, int ldx, const float *d_bias, float *d_y,
                                 int ldy, int batch, int epi, const lmc_gemv_extra *ex, cudaStream_t s) {
    if (batch > 8 && t->gemm_wscale > 0.0f) return lmc_gemm_launch(t, d_x, ldx, d_bias, d_y, ldy, batch, epi, ex, s);
    if (!t->tiled) return lmc_set_error(LMC_ERR_UNSUPPORTED, "gemv_ex: no tiled layout");
    if (((uintptr_t)d_x & 15) || (ldx & 3) || (ex->x2 && ((uintptr_t)ex->x2 & 15)) ||
        (ex->w && ((uintptr_t)ex->w & 15)) || (ex->b && ((uintptr_t)ex->b & 15)))
        return lmc_set_error(LMC_ERR_INVALID, "gemv_ex: activations and prologue vectors must be 16-byte aligned");
    TArgs a = {};
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
    a.key_base = ex->key_base;
    for (int b0 = 0; b0 < batch;) {
        int nb = std::min(batch - b0, 8);
        Plan P;
        int rc = plan_for(t->type, t->tiled_rows, t->cols, nb, &P);
        while (rc == LMC_ERR_UNSUPPORTED && nb > 1) {  // shared memory: fewer rows per launch
            nb = nb > 4 ? 4 : nb > 2 ? 2 : 1;
            rc = plan_for(t->type, t->tiled_rows, t->cols, nb, &P);
        }
        if (rc == LMC_ERR_UNSUPPORTED)
            return lmc_set_error(rc, "tiled gemv: %d columns need too much shared memory", t->cols);
        a.x = d_x + (size_t)b0 * ldx;
        a.y = d_y + (size_t)b0 * ldy;
        a.x2 = ex->x2 ? ex->x2 + (size_t)b0 * ldx : NULL;
        a.keys = ex->keys ? ex->keys + b0 : NULL;
        a.nb = nb;
        if ((rc = launch_plan(t, a, P, s))) return rc;
        b0 += nb;
    }
    return LMC_OK;
}
