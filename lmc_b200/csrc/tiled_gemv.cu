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
#include "tiled_gemv.cuh"

namespace {

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
    const int st = lmc_step_status();
    if (st != LMC_OK) return st;
    const int at = lmc_attn_status();
    if (at != LMC_OK) return at;
    const int pe = lmc_peer_status();
    if (pe != LMC_OK) return pe;
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

// Failure-path self-test: one thread waits (bounded) on an mbarrier phase
// that nothing completes, so the wait runs out, records the timeout and the
// kernel returns normally.
__global__ void k_wait_selftest(int *gave_up) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x) return;
    mbar_init(&bar);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *gave_up = mbar_wait(&bar, 0u) ? 0 : 1;
}

extern "C" int lmc_tiled_wait_selftest(int *d_flag, cudaStream_t s) {
    k_wait_selftest<<<1, 32, 0, s>>>(d_flag);
    LMC_LAUNCH_CHECK("wait self-test");
    return LMC_OK;
}

extern "C" int lmc_tiled_set_wait_limit(long long ns) {
    const long long v = ns > 0 ? ns : 1000000000ll;
    LMC_CUDA_TRY(cudaMemcpyToSymbol(g_wait_ns, &v, sizeof v));
    return LMC_OK;
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
    {   // short matrices at batch <= 2: the latency GEMV (no per-CTA quantization of x)
        const int rc = lmc_ff_gemv_launch(t, d_x, ldx, d_bias, d_y, ldy, batch, epi, ex, s);
        if (rc != LMC_ERR_UNSUPPORTED) return rc;
    }
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
