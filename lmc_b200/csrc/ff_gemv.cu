// ff_gemv.cu - the standalone latency GEMV (K2, short matrices): for one or
// two batch rows and matrices small enough that a warp gets at most two
// units of the tiled layout at full grid, x is staged once as fp32 in shared
// memory and each unit is dotted with fp32 FMAs (ff_unit.cuh).  The
// tensor-core GEMV instead quantizes x into three int8 limbs in every CTA, a
// set-up that is most of a short GEMV's time (the GPT-2 and TinyLlama decode
// shapes).  Results agree with the tensor-core GEMV to fp32 rounding.
// Replaces matmul_vec (src/ops.c:69-97) on the tiled Q4_K / Q6_K / Q8_0
// layout, with the same prologues (LayerNorm, RMSNorm, SwiGLU) and
// epilogues (bias, GELU, residual add, greedy-pick key).
#include "tiled_gemv.cuh"

namespace {
#include "ff_unit.cuh"

// x after its prologue into xs[b][K] (x was written by an earlier kernel).
// A norm's statistics are the two-pass ones of LMc's layer_norm / rms_norm
// (src/ops.c:47-59, src/ops_llama.c:24-33) over the row staged here; mr:
// mean[2], rstd[2], 16 floats of reduction scratch.
__device__ __forceinline__ void ff_stage_x(float *xs, float *mr, const TArgs &a) {
    const int K = a.KB * 256, tid = threadIdx.x;
    const bool ln = a.pro == LMC_PRO_LAYERNORM, norm = ln || a.pro == LMC_PRO_RMSNORM;
    const bool glu = a.pro == LMC_PRO_SWIGLU;
    float s[2] = {0.0f, 0.0f};
#pragma unroll
    for (int b = 0; b < 2; b++) {
        if (b >= a.nb) break;
        const float *xr = a.x + (size_t)b * a.ldx, *x2r = glu ? a.x2 + (size_t)b * a.ldx : nullptr;
        for (int k0 = tid * 4; k0 < K; k0 += 4 * NTHR * 4) {  // four loads in flight per thread
            float4 v[4], u[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int k = k0 + q * NTHR * 4;
                if (k < K) {
                    v[q] = __ldg(reinterpret_cast<const float4 *>(xr + k));
                    if (glu) u[q] = __ldg(reinterpret_cast<const float4 *>(x2r + k));
                }
            }
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int k = k0 + q * NTHR * 4;
                if (k >= K) continue;
                float4 o = v[q];
                if (glu)
                    o = make_float4(silu_short(v[q].x) * u[q].x, silu_short(v[q].y) * u[q].y,
                                    silu_short(v[q].z) * u[q].z, silu_short(v[q].w) * u[q].w);
                else if (ln)
                    s[b] += (o.x + o.y) + (o.z + o.w);
                *reinterpret_cast<float4 *>(xs + b * K + k) = o;
            }
        }
    }
    if (!norm) {
        __syncthreads();
        return;
    }
    float *red = mr + 4;
    float mu[2] = {0.0f, 0.0f};
    if (ln) {
        cta_reduce<2, false>(s, red);  // (synchronises: the staged rows are complete)
        mu[0] = s[0] / (float)K;
        mu[1] = s[1] / (float)K;
    } else {
        __syncthreads();
    }
    float q[2] = {0.0f, 0.0f};
#pragma unroll
    for (int b = 0; b < 2; b++) {
        if (b >= a.nb) break;
        for (int k = tid * 4; k < K; k += NTHR * 4) {
            const float4 v = *reinterpret_cast<const float4 *>(xs + b * K + k);
            const float d0 = v.x - mu[b], d1 = v.y - mu[b], d2 = v.z - mu[b], d3 = v.w - mu[b];
            q[b] += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
        }
    }
    cta_reduce<2, false>(q, red);
    const float eps = ln ? 1e-5f : a.eps;
#pragma unroll
    for (int b = 0; b < 2; b++) {
        if (b >= a.nb) break;
        const float r = 1.0f / sqrtf(q[b] / (float)K + eps), m = mu[b];
        for (int k = tid * 4; k < K; k += NTHR * 4) {
            float4 v = *reinterpret_cast<const float4 *>(xs + b * K + k);
            const float4 w = __ldg(reinterpret_cast<const float4 *>(a.pw + k));
            if (ln) {
                const float4 c = __ldg(reinterpret_cast<const float4 *>(a.pb + k));
                v = make_float4((v.x - m) * r * w.x + c.x, (v.y - m) * r * w.y + c.y, (v.z - m) * r * w.z + c.z,
                                (v.w - m) * r * w.w + c.w);
            } else {
                v = make_float4(w.x * r * v.x, w.y * r * v.y, w.z * r * v.z, w.w * r * v.w);
            }
            *reinterpret_cast<float4 *>(xs + b * K + k) = v;
        }
    }
    __syncthreads();
}

// CTA c owns row tiles [c RT / NC, (c + 1) RT / NC); its units (row tile
// major) are split evenly over the 8 warps.  Each warp's weights are asked of
// L2 before the dependency wait (they do not depend on the previous kernel)
// and read with plain loads.
template <int QT>
__global__ void __launch_bounds__(NTHR) k_gemv_ff(TArgs a) {
    extern __shared__ __align__(16) float fsm[];
    constexpr int UNIT = unit_bytes(QT);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int K = a.KB * 256, nb = a.nb;
    float *xs = fsm, *mr = fsm + (size_t)nb * K, *acc = mr + 20;  // acc [tiles][2][16]
    const int t0 = (int)blockIdx.x * a.RT / a.NC, t1 = ((int)blockIdx.x + 1) * a.RT / a.NC;
    const int Uc = (t1 - t0) * a.KB, w0 = Uc * wid / WARPS, w1 = Uc * (wid + 1) / WARPS;
    const uint8_t *wbase = a.w + (size_t)t0 * a.KB * UNIT;
    if (lane == 0)
        for (int i = w0; i < w1; i++) prefetch_l2(wbase + (size_t)i * UNIT, (uint32_t)UNIT);
    for (int i = threadIdx.x; i < (t1 - t0) * 32; i += NTHR) acc[i] = 0.0f;
    pdl_wait();
    pdl_launch_dependents();
    ff_stage_x(xs, mr, a);
    FAcc fa;
    fa.zero();
    int cur = -1;
    for (int i = w0; i < w1; i++) {
        const int rt = i / a.KB, kb = i - rt * a.KB;
        if (rt != cur) {
            if (cur >= 0) fflush(fa, acc + cur * 32, nb, lane);
            fa.zero();
            cur = rt;
        }
        const uint8_t *u = wbase + (size_t)i * UNIT;
        if (nb == 1) {
            if (QT == 4) funit_q4k<1>(fa, u, xs, K, kb * 256, lane);
            else if (QT == 6) funit_q6k<1>(fa, u, xs, K, kb * 256, lane);
            else funit_q80<1>(fa, u, xs, K, kb * 256, lane);
        } else {
            if (QT == 4) funit_q4k<2>(fa, u, xs, K, kb * 256, lane);
            else if (QT == 6) funit_q6k<2>(fa, u, xs, K, kb * 256, lane);
            else funit_q80<2>(fa, u, xs, K, kb * 256, lane);
        }
    }
    if (cur >= 0) fflush(fa, acc + cur * 32, nb, lane);
    __syncthreads();
    // epilogue: lane = 16 * batch row + tile row (batch <= 2)
    unsigned long long best = 0ull;
    for (int T = wid; T < t1 - t0; T += WARPS) {
        const int b = lane >> 4, row = (t0 + T) * 16 + (lane & 15);
        if (b >= nb || row >= a.M) continue;
        float v = acc[T * 32 + lane];
        if (a.bias) v += __ldg(a.bias + row);
        if (a.epi & LMC_EPI_GELU) v = lmc_gelu_f(v);
        float *o = a.y + (size_t)b * a.ldy + row;
        *o = (a.epi & LMC_EPI_ACCUM) ? *o + v : v;
        const unsigned long long k = lmc_argmax_key(v, row + a.key_base);
        best = k > best ? k : best;
    }
    if (a.keys) {  // greedy keys: half-warp maxima, one atomic per CTA and batch row
        __shared__ unsigned long long kbest[WARPS][2];
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
            best = o > best ? o : best;
        }
        if ((lane & 15) == 0) kbest[wid][lane >> 4] = best;
        __syncthreads();
        if ((int)threadIdx.x < nb) {
            unsigned long long k = 0ull;
            for (int w = 0; w < WARPS; w++) k = kbest[w][threadIdx.x] > k ? kbest[w][threadIdx.x] : k;
            if (k) atomicMax(a.keys + threadIdx.x, k);
        }
    }
}

}  // namespace

// The latency GEMV when the shape suits it (batch <= 2; at most three units a
// warp at batch 1, two at batch 2, with two CTAs per SM; x and the CTA's
// accumulators within 100 KB of shared memory); LMC_ERR_UNSUPPORTED otherwise
// (the caller launches the tensor-core GEMV).  LMC_GEMV_FF=0 disables it.
extern "C" int lmc_ff_gemv_suits(const lmc_qtensor *t, int batch, int epi) {
    // units a warp at most: 3 at batch 1, 2 at batch 2 (TinyLlama decode: 3
    // at batch 1 gained 3.6 %, at batch 2 it lost 7 % against 2)
    static int off = -1, upw_env = 0;
    if (off < 0) {
        const char *e = getenv("LMC_GEMV_FF");
        off = e && e[0] == '0';
        const char *u = getenv("LMC_GEMV_FF_UNITS");
        if (u && atoi(u) > 0) upw_env = atoi(u);
    }
    const int upw = upw_env ? upw_env : batch == 1 ? 3 : 2;
    if (off || !t || !t->tiled || batch < 1 || batch > 2 || (epi & ~(LMC_EPI_GELU | LMC_EPI_ACCUM))) return 0;
    if (t->type != LMC_TYPE_Q4_K && t->type != LMC_TYPE_Q6_K && t->type != LMC_TYPE_Q8_0) return 0;
    const int KB = t->cols / 256, RT = t->tiled_rows / 16;
    const int NC = std::min(RT, 2 * lmc_sm_count());
    const int maxrt = (RT + NC - 1) / NC;
    if ((long long)maxrt * KB > (long long)upw * WARPS) return 0;  // more units a warp than that
    return ((size_t)batch * KB * 256 + 20 + (size_t)maxrt * 32) * sizeof(float) <= 100 * 1024;
}

extern "C" int lmc_ff_gemv_launch(const lmc_qtensor *t, const float *d_x, int ldx, const float *d_bias, float *d_y,
                                  int ldy, int batch, int epi, const lmc_gemv_extra *ex, cudaStream_t s) {
    if (!lmc_ff_gemv_suits(t, batch, epi)) return LMC_ERR_UNSUPPORTED;
    const int qt = t->type == LMC_TYPE_Q4_K ? 4 : t->type == LMC_TYPE_Q6_K ? 6 : 8;
    const int KB = t->cols / 256, RT = t->tiled_rows / 16;
    const int NC = std::min(RT, 2 * lmc_sm_count());
    const int maxrt = (RT + NC - 1) / NC;
    const size_t smem = ((size_t)batch * KB * 256 + 20 + (size_t)maxrt * 32) * sizeof(float);
    TArgs a = {};
    a.w = (const uint8_t *)t->tiled;
    a.x = d_x;
    a.bias = d_bias;
    a.y = d_y;
    a.M = t->rows;
    a.KB = KB;
    a.RT = RT;
    a.ldx = ldx;
    a.ldy = ldy;
    a.nb = batch;
    a.epi = epi;
    a.pro = ex->pro;
    a.pw = ex->w;
    a.pb = ex->b;
    a.x2 = ex->x2;
    a.eps = ex->eps;
    a.keys = ex->keys;
    a.key_base = ex->key_base;
    a.NC = NC;
    a.CL = 1;
    void (*fn)(TArgs) = qt == 4 ? k_gemv_ff<4> : qt == 6 ? k_gemv_ff<6> : k_gemv_ff<8>;
    static thread_local size_t set_smem[3];
    const int fi = qt == 4 ? 0 : qt == 6 ? 1 : 2;
    if (smem > 48 * 1024 && smem > set_smem[fi]) {
        LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024));
        set_smem[fi] = 100 * 1024;
    }
    LMC_LAUNCH("latency gemv", fn, NC, NTHR, smem, s, a);
    return LMC_OK;
}
