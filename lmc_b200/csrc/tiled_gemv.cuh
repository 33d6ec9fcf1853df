// tiled_gemv.cuh - device code of the tensor-core GEMV (tiled_gemv.cu) shared
// with the persistent decode-step kernel (step_kernel.cu): kernel arguments,
// the shared-memory layout, the activation quantizer, the bulk-copy ring,
// the per-unit MMA bodies and the epilogue.  Each including translation unit
// gets its own copy (anonymous namespace).
#pragma once
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
    // Norm statistics of x supplied by whoever wrote x (the persistent step):
    // per batch row {sum x, sum x^2} in fp64, or NULL (build_x computes them)
    const double *stats;
    // non-NULL: the epilogue adds {sum y, sum y^2} of its final outputs here
    double *stats_out;
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
// CG: x and x2 were written earlier in the same launch (the persistent
// decode-step kernel) by other CTAs, so they are read through L2 (ld.cg)
// instead of the non-coherent path.
template <bool CG = false>
struct XView {
    const float *x, *x2, *w, *b;
    int ldx, pro;
    const float *mean, *rstd;  // per batch row (shared memory)
    __device__ __forceinline__ float4 act4(const float *p) const {
        return CG ? __ldcg(reinterpret_cast<const float4 *>(p)) : __ldg(reinterpret_cast<const float4 *>(p));
    }
    __device__ __forceinline__ float4 raw4(int bi, int k) const { return act4(x + (size_t)bi * ldx + k); }
    __device__ __forceinline__ float4 at4(int bi, int k) const {
        const float4 v = raw4(bi, k);
        if (pro == LMC_PRO_NONE) return v;
        if (pro == LMC_PRO_SWIGLU) {
            const float4 u = act4(x2 + (size_t)bi * ldx + k);
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
template <int NT, int QT, int RX, bool CG = false>
__device__ __forceinline__ void build_x(uint8_t *smem, const Smem<NT, QT> &L, const TArgs &a) {
    constexpr int NB = 2 * NT, CH = Smem<NT, QT>::CH, SPAN = QT == 6 ? 16 : 32;
    float *scl = reinterpret_cast<float *>(smem + L.sc_off());
    float *inv = scl + 8, *mean = inv + 8, *rstd = mean + 8;
    float *red = reinterpret_cast<float *>(smem + L.red_off());
    const int tid = threadIdx.x;
    const int K = a.KB * 256, nb = a.nb;
    const XView<CG> xv{a.x, a.x2, a.pw, a.pb, a.ldx, a.pro, mean, rstd};
    if ((a.pro == LMC_PRO_LAYERNORM || a.pro == LMC_PRO_RMSNORM) && a.stats) {
        // statistics accumulated in fp64 by the ops that wrote x: mean and
        // variance (E x^2 - mean^2; the two-pass float form of src/ops.c:52-54
        // agrees to ~1e-7 relative), or the mean square for RMSNorm
        if (tid < NB) {
#pragma unroll
            for (int b = 0; b < NB; b++)
                if (tid == b) {
                    const double sx = b < nb ? __ldcg(a.stats + 2 * b) : 0.0;
                    const double sq = b < nb ? __ldcg(a.stats + 2 * b + 1) : 0.0;
                    const double mu = a.pro == LMC_PRO_RMSNORM ? 0.0 : sx / (double)K;
                    const double var = fmax(sq / (double)K - mu * mu, 0.0);
                    mean[b] = (float)mu;
                    rstd[b] = 1.0f / sqrtf((float)var + (a.pro == LMC_PRO_RMSNORM ? a.eps : 1e-5f));
                }
        }
        __syncthreads();
    } else if (a.pro == LMC_PRO_LAYERNORM || a.pro == LMC_PRO_RMSNORM) {  // per-row statistics
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
__device__ __forceinline__ long long globaltimer_ns() {
    long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Limit of every bounded wait below (nanoseconds of %globaltimer); the host
// may shorten it (a test makes a wait run out this way).
__device__ long long g_wait_ns = 1000000000ll;
// Bounded wait: each poll suspends the warp until the phase completes or
// about 64 us pass; once g_wait_ns have gone by (about one second) it gives
// up, records the timeout and lets the caller skip the unit.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try(bar, parity)) return true;
        if (globaltimer_ns() - t0 > g_wait_ns) break;
    }
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
    // the residual read goes through L2: in the persistent step kernel another
    // CTA may have written this row earlier in the same launch
    *o = (a.epi & LMC_EPI_ACCUM) ? __ldcg(o) + v : v;
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

}  // namespace
