// sample.cuh - top-p (nucleus) sampling with temperature on the device,
// shared by the standalone kernel (sample.cu) and the persistent decode step.
//
// LMc's sample_top_p (src/lmc.c:42-59): below temperature 1e-6 the greedy
// pick (first maximum); otherwise logits *= 1/temperature, softmax
// (src/ops.c:32-44), sort descending, the nucleus = the shortest prefix whose
// running sum reaches top_p, renormalise, and walk the nucleus until the
// running probability passes r = rng_float() (xorshift64, src/lmc.c:29-33);
// if rounding leaves r above the last cdf, the nucleus' last token.
//
// Here nothing is sorted.  The probabilities are positive floats, so their
// bit patterns order like their values, and "the shortest prefix of the
// descending order whose sum reaches x" is a weighted select on those 32-bit
// keys: four passes of a 256-bucket histogram (counts and probability sums,
// most significant byte first) find the key T where the sum of everything
// above it first reaches x.  One select finds the nucleus boundary (x =
// top_p), a second one the sampled token inside it (x = r * nucleus sum).
// Tokens with exactly equal probabilities are taken in index order (LMc
// leaves their order to qsort).  The sums are fp32 in a different order from
// LMc's running sums, so a draw within ~1e-7 of a cdf boundary may land on
// the neighbouring token.
#pragma once
#include "lmc_common.cuh"

namespace {

constexpr int SMP_HIST = 8;  // sub-histograms (warp w adds into w % 8)

struct SampleSmem {
    float hs[SMP_HIST][256];
    int hc[SMP_HIST][256];
    float bs[256];
    int bc[256];
    float red[32];
    int ired[32];
    float f[8];
    int i[8];
};

__device__ __forceinline__ unsigned long long lmc_xorshift64(unsigned long long s) {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return s;
}

template <int NTH>
__device__ __forceinline__ float smp_block_sum(float v, float *red) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < NTH / 32; w++) t += red[w];  // fixed order: every thread the same value
    return t;
}
template <int NTH>
__device__ __forceinline__ float smp_block_max(float v, float *red) {
    v = warp_max(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = red[0];
    for (int w = 1; w < NTH / 32; w++) t = fmaxf(t, red[w]);
    return t;
}

// Probability of token i: the softmax of the scaled logits, as
// src/ops.c:32-44 computes it (e^(z - max) * (1 / sum), or 1/V when the sum
// is below 1e-30).
struct Probs {
    const float *lg;
    float inv_t, mx, inv_sum, uni;
    __device__ __forceinline__ float operator()(int i) const {
        if (uni > 0.0f) return uni;
        return expf(__ldcg(lg + i) * inv_t - mx) * inv_sum;
    }
};

// Weighted select over the keys >= lo: the largest key T such that the sum
// of p over keys >= T reaches x (strict: exceeds x).  Returns T; *above = the
// sum over keys > T, *ties = the count of key == T.  When the whole sum falls
// short of x (rounding), T is the smallest key >= lo that occurs.
template <int NTH>
__device__ uint32_t smp_select(const Probs &P, int V, uint32_t lo, float x, bool strict, float *above, int *ties,
                               SampleSmem &S) {
    uint32_t prefix = 0, mask = 0;
    float A = 0.0f;
    const int wh = (threadIdx.x >> 5) % SMP_HIST;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int j = threadIdx.x; j < SMP_HIST * 256; j += NTH) {
            (&S.hs[0][0])[j] = 0.0f;
            (&S.hc[0][0])[j] = 0;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < V; i += NTH) {
            const float p = P(i);
            const uint32_t k = __float_as_uint(p);
            if (k >= lo && (k & mask) == prefix) {
                const int d = (int)((k >> shift) & 255u);
                atomicAdd(&S.hs[wh][d], p);
                atomicAdd(&S.hc[wh][d], 1);
            }
        }
        __syncthreads();
        for (int j = threadIdx.x; j < 256; j += NTH) {
            float s = 0.0f;
            int c = 0;
            for (int h = 0; h < SMP_HIST; h++) {
                s += S.hs[h][j];
                c += S.hc[h][j];
            }
            S.bs[j] = s;
            S.bc[j] = c;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int dig = -1, low = -1;
            float a = A;
            for (int j = 255; j >= 0; j--) {
                if (!S.bc[j]) continue;
                low = j;
                const float t = a + S.bs[j];
                if (strict ? t > x : t >= x) {
                    dig = j;
                    break;
                }
                a = t;
            }
            if (dig < 0) {  // the sum falls short of x: the lowest occupied bucket
                dig = low < 0 ? 0 : low;
                a = A;
                for (int j = 255; j > dig; j--) a += S.bs[j];
            }
            S.i[0] = dig;
            S.f[0] = a;
            S.i[1] = S.bc[dig];
        }
        __syncthreads();
        prefix |= (uint32_t)S.i[0] << shift;
        mask |= 255u << shift;
        A = S.f[0];
        __syncthreads();
    }
    *above = A;
    *ties = S.i[1];
    return prefix;
}

// Index of the j-th (0-based) token, in index order, whose key is exactly k.
template <int NTH>
__device__ int smp_nth_equal(const Probs &P, int V, uint32_t k, int j, SampleSmem &S) {
    const int C = (V + NTH - 1) / NTH, i0 = threadIdx.x * C, i1 = min(V, i0 + C);
    int c = 0;
    for (int i = i0; i < i1; i++) c += __float_as_uint(P(i)) == k;
    // exclusive scan of the per-thread counts (threads own contiguous ranges)
    int incl = c;
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if ((threadIdx.x & 31) >= o) incl += v;
    }
    if ((threadIdx.x & 31) == 31) S.ired[threadIdx.x >> 5] = incl;
    __syncthreads();
    int base = 0;
    for (int w = 0; w < (int)(threadIdx.x >> 5); w++) base += S.ired[w];
    const int excl = base + incl - c;
    if (threadIdx.x == 0) S.i[2] = -1;
    __syncthreads();
    if (j >= excl && j < excl + c) {
        int seen = excl;
        for (int i = i0; i < i1; i++)
            if (__float_as_uint(P(i)) == k) {
                if (seen == j) {
                    S.i[2] = i;
                    break;
                }
                seen++;
            }
    }
    __syncthreads();
    return S.i[2];
}

// One row: the sampled token of logits lg[0..V) into *out; rng advanced once
// unless the pick is greedy.  Every thread of the CTA calls it.
template <int NTH>
__device__ void sample_row(const float *lg, int V, float temperature, float top_p, unsigned long long *rng, int *out,
                           SampleSmem &S) {
    if (temperature < 1e-6f) {  // greedy: first maximum (src/lmc.c:45-47)
        unsigned long long best = 0ull;
        for (int i = threadIdx.x; i < V; i += NTH) {
            const unsigned long long k = lmc_argmax_key(__ldcg(lg + i), i);
            best = k > best ? k : best;
        }
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
            best = k > best ? k : best;
        }
        __syncthreads();
        auto kb = reinterpret_cast<unsigned long long *>(&S.hs[0][0]);
        if ((threadIdx.x & 31) == 0) kb[threadIdx.x >> 5] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < NTH / 32; w++) best = kb[w] > best ? kb[w] : best;
            best = kb[0] > best ? kb[0] : best;
            *out = lmc_key_index(best);
        }
        __syncthreads();
        return;
    }
    Probs P;
    P.lg = lg;
    P.inv_t = 1.0f / temperature;
    P.uni = 0.0f;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < V; i += NTH) m = fmaxf(m, __ldcg(lg + i) * P.inv_t);
    P.mx = smp_block_max<NTH>(m, S.red);
    float s = 0.0f;
    for (int i = threadIdx.x; i < V; i += NTH) s += expf(__ldcg(lg + i) * P.inv_t - P.mx);
    s = smp_block_sum<NTH>(s, S.red);
    if (s < 1e-30f) P.uni = 1.0f / (float)V;
    P.inv_sum = 1.0f / s;
    // nucleus: all keys above T, then ties at T in index order until top_p is reached
    float aT;
    int cT;
    const uint32_t T = smp_select<NTH>(P, V, 0u, top_p, false, &aT, &cT, S);
    const float pT = __uint_as_float(T);
    int nT = cT;
    if (pT > 0.0f && aT + (float)cT * pT >= top_p) {
        nT = (int)ceilf((top_p - aT) / pT);
        nT = max(1, min(cT, nT));
    }
    const float ns = aT + (float)nT * pT;
    // the draw (src/lmc.c:31-33,56-58): the first nucleus token whose running
    // probability passes r, i.e. the key where the sum above reaches r * ns
    unsigned long long st = 0;
    if (threadIdx.x == 0) {
        st = lmc_xorshift64(*rng);
        *rng = st;
        S.f[4] = (float)(st >> 11) / (float)(1ULL << 53);
    }
    __syncthreads();
    const float r = S.f[4];
    float aU;
    int cU;
    const uint32_t U = smp_select<NTH>(P, V, T, r * ns, true, &aU, &cU, S);
    int j;
    uint32_t key;
    const float pU = __uint_as_float(U);
    if (U > T) {
        key = U;
        j = pU > 0.0f ? (int)floorf((r * ns - aU) / pU) : 0;
        j = max(0, min(cU - 1, j));
    } else {  // inside the ties at T, of which the nucleus holds nT
        key = T;
        j = pT > 0.0f ? (int)floorf((r * ns - aU) / pT) : nT - 1;
        j = max(0, min(nT - 1, j));
    }
    const int idx = smp_nth_equal<NTH>(P, V, key, j, S);
    if (threadIdx.x == 0) *out = idx < 0 ? 0 : idx;
    __syncthreads();
}

}  // namespace
