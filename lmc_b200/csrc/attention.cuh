// attention.cuh - device code of the CUDA-core decode attention (attention.cu)
// shared with the persistent decode-step kernel (step_kernel.cu): arguments,
// the split body and the in-launch merge of the splits.  NTH is the CTA size.
#pragma once
#include <cuda_fp16.h>

#include "lmc_common.cuh"
#include "lmc_internal.h"

#ifndef ATT_THREADS
#define ATT_THREADS 128
#endif

namespace {

template <typename KV> __device__ __forceinline__ float kv_ld(const KV *p);
template <> __device__ __forceinline__ float kv_ld<float>(const float *p) { return *p; }
template <> __device__ __forceinline__ float kv_ld<__half>(const __half *p) { return __half2float(*p); }
template <typename KV> __device__ __forceinline__ KV kv_cvt(float v);
template <> __device__ __forceinline__ float kv_cvt<float>(float v) { return v; }
template <> __device__ __forceinline__ __half kv_cvt<__half>(float v) { return __float2half_rn(v); }

// int8 K/V rows (LMC_KV_Q8): a row is Dh int8 codes followed by a 16-byte
// tail whose first 4 bytes are the row's fp32 scale; value = code * scale.
// KvQ8 is the element type of such a cache (one byte); its row stride in
// elements is Dh + 16.
struct KvQ8 {
    int8_t v;
};
template <typename KV> struct KvT {
    static constexpr bool Q8 = false;
};
template <> struct KvT<KvQ8> {
    static constexpr bool Q8 = true;
};
template <typename KV> __host__ __device__ constexpr int kv_rs(int Dh) { return KvT<KV>::Q8 ? Dh + 16 : Dh; }
template <> __device__ __forceinline__ float kv_ld<KvQ8>(const KvQ8 *p) { return (float)p->v; }
__device__ __forceinline__ float kv_q8_scale(const KvQ8 *row, int Dh) {
    return *reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(row) + Dh);
}
// One warp quantizes one new row (K rotated first when rc is given): m =
// max|x|, code = clamp(rint(x * (127 / m)), +-127), scale = m / 127 (all zero
// when m is 0).  Lane takes element pairs d = lane + 32 i (Dh <= 512).
__device__ __forceinline__ void kv_q8_store_row(KvQ8 *row, const float *src, const float *rc, const float *rs, int Dh,
                                                int lane) {
    float v[16];
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int d = lane + 32 * i;
        v[2 * i] = v[2 * i + 1] = 0.0f;
        if (2 * d < Dh) {
            float x0 = src[2 * d], x1 = src[2 * d + 1];
            if (rc) {
                const float c = rc[d], sn = rs[d];
                const float r0 = x0 * c - x1 * sn, r1 = x0 * sn + x1 * c;
                x0 = r0;
                x1 = r1;
            }
            v[2 * i] = x0;
            v[2 * i + 1] = x1;
            m = fmaxf(m, fmaxf(fabsf(x0), fabsf(x1)));
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float inv = m > 0.0f ? 127.0f / m : 0.0f;
    int8_t *q = reinterpret_cast<int8_t *>(row);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int d = lane + 32 * i;
        if (2 * d < Dh) {
            const int q0 = max(-127, min(127, __float2int_rn(__fmul_rn(v[2 * i], inv))));
            const int q1 = max(-127, min(127, __float2int_rn(__fmul_rn(v[2 * i + 1], inv))));
            q[2 * d] = (int8_t)q0;
            q[2 * d + 1] = (int8_t)q1;
        }
    }
    if (lane == 0) *reinterpret_cast<float *>(q + Dh) = m / 127.0f;
}

struct AttnArgs {
    float *out;
    const float *q, *k_new, *v_new;
    void *k_cache, *v_cache;
    const int *pos;
    float *ws;  // [batch][H][nsplit][Dh + 2]
    int H, Hkv, Dh, S, CH, nsplit;
    int ldo, ldq, ldkv;  // row strides (floats) between sequences
    // RoPE tables [S][Dh/2] (LLaMA, src/ops_llama.c:75-78) applied to q and to
    // the new K row here, or NULL
    const float *rope_cos, *rope_sin;
    int *cnt;  // [batch][Hkv] arrival counters, zero between launches, or NULL (separate combine kernel)
    // Row -> cache sequence (NULL: row b uses sequence b).  Rows may share a
    // sequence (a prompt chunk of one sequence, one position per row); their
    // K/V rows are then appended by k_kv_append before this launch and
    // `append` is 0, so every row sees the rows of earlier positions.
    const int *seq;
    int append;
    // Paged cache (NULL: contiguous [batch][Hkv][S][row]): k_cache / v_cache
    // are pools of pages [page][Hkv][P][row], P = 1 << page_shift positions;
    // pages[seq * max_pages + t / P] is the page of position t.  A page id
    // outside [0, n_pages) is not read (page 0 is, and g_attn_page_err is set).
    const int *pages;
    int page_shift, max_pages, n_pages;
};
__device__ int g_attn_page_err;  // an out-of-range page id was met (lmc_device_status)

// Row t of cache sequence cs, kv head kh in a paged pool (a.pages set):
// page a.pages[cs * max_pages + t / P], slot t % P of that page's kv head kh.
// A page id outside [0, n_pages) is not followed: page 0 is used instead and
// g_attn_page_err is set.
template <typename KV>
__device__ __forceinline__ KV *kv_page_row(const AttnArgs &a, KV *pool, size_t cs, int kh, int t, int RS) {
    int pg = __ldg(a.pages + cs * a.max_pages + (t >> a.page_shift));
    if (pg < 0 || pg >= a.n_pages) {
        atomicExch(&g_attn_page_err, 1);
        pg = 0;
    }
    return pool + ((((size_t)pg * a.Hkv + kh) << a.page_shift) + (t & ((1 << a.page_shift) - 1))) * RS;
}


// One non-empty split: append the new K/V row when it falls here, scores,
// softmax statistics and the unnormalised accumulator (or the final output
// when there is one split).  Query heads go in groups of up to 8:
//   scores: lane = position (32 per warp and pass), the K row read as 16-byte
//     vectors all issued before the first use (up to 256 bytes at a time, so
//     one memory latency per row instead of one per 8 elements), q broadcast
//     from shared memory, the 8 dot products in registers (sequential over d
//     as src/ops.c:145-149), no shuffles;
//   out = sum_t p_t v_t: warp w takes positions t = w (mod 4), four of them
//     per batch with every load issued first; lane holds dims lane + 32 i of
//     every head of the group, so each V element is loaded once; the 4 warps'
//     partials are added in shared memory.
// Chunk c (8 elements) of a block of raw 16-byte K words -> 8 floats.  The
// words come from plain loads: the row at `pos` was written by this CTA
// earlier in the launch.
template <typename KV, int NV> __device__ __forceinline__ void kv_chunk(const uint4 (&raw)[NV], int c, float (&v)[8]);
template <int NV> __device__ __forceinline__ void kv_chunk_f32(const uint4 (&raw)[NV], int c, float (&v)[8]) {
    const uint4 x = raw[2 * c], y = raw[2 * c + 1];
    v[0] = __uint_as_float(x.x); v[1] = __uint_as_float(x.y); v[2] = __uint_as_float(x.z); v[3] = __uint_as_float(x.w);
    v[4] = __uint_as_float(y.x); v[5] = __uint_as_float(y.y); v[6] = __uint_as_float(y.z); v[7] = __uint_as_float(y.w);
}
template <int NV> __device__ __forceinline__ void kv_chunk_q8(const uint4 (&raw)[NV], int c, float (&v)[8]) {
    const uint4 u = raw[c >> 1];
    const uint32_t w0 = (c & 1) ? u.z : u.x, w1 = (c & 1) ? u.w : u.y;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        v[i] = (float)(int)(int8_t)(w0 >> (8 * i));
        v[4 + i] = (float)(int)(int8_t)(w1 >> (8 * i));
    }
}
template <int NV> __device__ __forceinline__ void kv_chunk_f16(const uint4 (&raw)[NV], int c, float (&v)[8]) {
    const uint4 u = raw[c];
    const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}
constexpr int ATT_GROUP = 8;  // query heads per pass

// RBMAX: K bytes loaded per block of the scores loop (registers: RBMAX / 4).
// ch: positions per split when the caller coarsened the plan (0: a.CH);
// single: this is the only split holding positions (the output is final).
template <typename KV, int DH, int NTH = ATT_THREADS, int RBMAX = 256>
__device__ __forceinline__ void split_body(const AttnArgs &a, float *sm, int sp, int kh, int b, int pos, int t0, int t1,
                                           float *wsb, size_t hstride, int ch = 0, bool single = false) {
    const int G = a.H / a.Hkv, Dh = DH ? DH : a.Dh, CH = ch ? ch : a.CH, RS = kv_rs<KV>(Dh);
    constexpr bool Q8 = KvT<KV>::Q8;
    constexpr int ESZ = (int)sizeof(KV);
    constexpr int RB = DH ? (DH * ESZ < RBMAX ? DH * ESZ : RBMAX) : 128;  // K bytes per load block
    constexpr int NV = RB / 16, NC = RB / (8 * ESZ);                  // 16-byte words, 8-element chunks
    constexpr int DPLC = DH ? DH / 32 : 8;                            // dims per lane (bound)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = NTH / 32;
    float *qs = sm;                 // [G][Dh]
    float *sc = sm + G * Dh;        // [G][CH]
    float *ml = sc + G * CH;        // [G][2]
    float *red = ml + 2 * G;        // [nw][ATT_GROUP][Dh]
    const size_t cs = a.seq ? (size_t)a.seq[b] : (size_t)b;  // cache sequence of this row
    KV *const kpool = reinterpret_cast<KV *>(a.k_cache), *const vpool = reinterpret_cast<KV *>(a.v_cache);
    KV *kc = kpool + (cs * a.Hkv + kh) * a.S * RS;
    KV *vc = vpool + (cs * a.Hkv + kh) * a.S * RS;
    // row t of this (sequence, kv head): contiguous, or through the page table
    auto row = [&](KV *seqbase, KV *pool, int t) -> KV * {
        return a.pages ? kv_page_row<KV>(a, pool, cs, kh, t, RS) : seqbase + (size_t)t * RS;
    };
    const float *rc = a.rope_cos ? a.rope_cos + (size_t)pos * (Dh / 2) : nullptr;
    const float *rs = a.rope_sin ? a.rope_sin + (size_t)pos * (Dh / 2) : nullptr;
    if (Q8 && a.append && pos >= t0 && pos < t1) {  // quantize the new rows: warp 0 K, warp 1 V
        if (warp < 2)
            kv_q8_store_row(reinterpret_cast<KvQ8 *>(warp ? row(vc, vpool, pos) : row(kc, kpool, pos)),
                            (warp ? a.v_new : a.k_new) + (size_t)b * a.ldkv + (size_t)kh * Dh, warp ? nullptr : rc,
                            rs, Dh, lane);
    } else if (a.append && pos >= t0 && pos < t1) {  // append this step's K/V row (K rotated first when RoPE applies)
        const float *kn = a.k_new + (size_t)b * a.ldkv + (size_t)kh * Dh;
        const float *vn = a.v_new + (size_t)b * a.ldkv + (size_t)kh * Dh;
        KV *kp = row(kc, kpool, pos), *vp = row(vc, vpool, pos);
        for (int d = threadIdx.x; d < Dh / 2; d += NTH) {
            float k0 = kn[2 * d], k1 = kn[2 * d + 1];
            if (rc) {
                const float c = rc[d], sn = rs[d];
                const float r0 = k0 * c - k1 * sn, r1 = k0 * sn + k1 * c;
                k0 = r0;
                k1 = r1;
            }
            if constexpr (!Q8) {
                kp[2 * d] = kv_cvt<KV>(k0);
                kp[2 * d + 1] = kv_cvt<KV>(k1);
                vp[2 * d] = kv_cvt<KV>(vn[2 * d]);
                vp[2 * d + 1] = kv_cvt<KV>(vn[2 * d + 1]);
            }
        }
    }
    const float *qb = a.q + (size_t)b * a.ldq + (size_t)kh * G * Dh;
    for (int i = threadIdx.x; i < G * Dh / 2; i += NTH) {  // q pairs (rotated when RoPE applies)
        const int gq = i / (Dh / 2), d = i % (Dh / 2);
        float q0 = qb[gq * Dh + 2 * d], q1 = qb[gq * Dh + 2 * d + 1];
        if (rc) {
            const float c = rc[d], sn = rs[d];
            const float r0 = q0 * c - q1 * sn, r1 = q0 * sn + q1 * c;
            q0 = r0;
            q1 = r1;
        }
        qs[gq * Dh + 2 * d] = q0;
        qs[gq * Dh + 2 * d + 1] = q1;
    }
    __syncthreads();  // the new row (read back below) and q are in place
    const float scale = 1.0f / sqrtf((float)Dh);
    const int n = t1 - t0;
    for (int g0 = 0; g0 < G; g0 += ATT_GROUP) {
        const int gn = min(ATT_GROUP, G - g0);
        for (int tb = warp * 32; tb < n; tb += nw * 32) {
            const int tl = tb + lane;
            if (tl >= n) continue;
            const KV *kr = row(kc, kpool, t0 + tl);
            float sg[ATT_GROUP];
#pragma unroll
            for (int g = 0; g < ATT_GROUP; g++) sg[g] = 0.0f;
            const int rowb = Dh * ESZ;
            for (int ob = 0; ob < rowb; ob += RB) {
                uint4 raw[NV];
#pragma unroll
                for (int i = 0; i < NV; i++)
                    if (ob + 16 * i < rowb) raw[i] = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(kr) + ob + 16 * i);
#pragma unroll
                for (int c = 0; c < NC; c++) {
                const int d0 = ob / ESZ + 8 * c;
                if (d0 >= Dh) break;
                float kv[8];
                if (ESZ == 4) kv_chunk_f32<NV>(raw, c, kv);
                else if (Q8) kv_chunk_q8<NV>(raw, c, kv);
                else kv_chunk_f16<NV>(raw, c, kv);
#pragma unroll
                for (int g = 0; g < ATT_GROUP; g++) {
                    if (g < gn) {
                        const float4 qa = *reinterpret_cast<const float4 *>(qs + (g0 + g) * Dh + d0);
                        const float4 qc = *reinterpret_cast<const float4 *>(qs + (g0 + g) * Dh + d0 + 4);
                        float t = sg[g];
                        t = fmaf(qa.x, kv[0], t);
                        t = fmaf(qa.y, kv[1], t);
                        t = fmaf(qa.z, kv[2], t);
                        t = fmaf(qa.w, kv[3], t);
                        t = fmaf(qc.x, kv[4], t);
                        t = fmaf(qc.y, kv[5], t);
                        t = fmaf(qc.z, kv[6], t);
                        t = fmaf(qc.w, kv[7], t);
                        sg[g] = t;
                    }
                }
                }
            }
            const float rsc = Q8 ? kv_q8_scale(reinterpret_cast<const KvQ8 *>(kr), Dh) : 1.0f;
#pragma unroll
            for (int g = 0; g < ATT_GROUP; g++)
                if (g < gn) sc[(g0 + g) * CH + tl] = (Q8 ? sg[g] * rsc : sg[g]) * scale;
        }
    }
    __syncthreads();
    for (int g = warp; g < G; g += nw) {
        float m = -INFINITY;
        for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[g * CH + t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < n; t += 32) {
            const float e = expf(sc[g * CH + t] - m);
            sc[g * CH + t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { ml[2 * g] = m; ml[2 * g + 1] = l; }
    }
    __syncthreads();
    const int dpl = Dh / 32;  // dims per lane (<= 8)
    for (int g0 = 0; g0 < G; g0 += ATT_GROUP) {
        const int gn = min(ATT_GROUP, G - g0);
        float acc[ATT_GROUP][DPLC];
#pragma unroll
        for (int g = 0; g < ATT_GROUP; g++)
#pragma unroll
            for (int i = 0; i < DPLC; i++) acc[g][i] = 0.0f;
        constexpr int U = 4;  // positions per batch of loads
        for (int t = warp; t < n; t += U * nw) {
            float v[U][DPLC];
#pragma unroll
            for (int uu = 0; uu < U; uu++) {
                const int tt = t + uu * nw;
                const KV *vrow = row(vc, vpool, t0 + min(tt, n - 1)), *vr = vrow + lane;
#pragma unroll
                for (int i = 0; i < DPLC; i++) v[uu][i] = (tt < n && i < dpl) ? kv_ld<KV>(vr + 32 * i) : 0.0f;
                if (Q8 && tt < n) {
                    const float vs = kv_q8_scale(reinterpret_cast<const KvQ8 *>(vrow), Dh);
#pragma unroll
                    for (int i = 0; i < DPLC; i++) v[uu][i] *= vs;
                }
            }
#pragma unroll
            for (int uu = 0; uu < U; uu++) {
                const int tt = t + uu * nw;
                if (tt >= n) break;
#pragma unroll
                for (int g = 0; g < ATT_GROUP; g++) {
                    if (g < gn) {
                        const float pt = sc[(g0 + g) * CH + tt];
#pragma unroll
                        for (int i = 0; i < DPLC; i++)
                            if (i < dpl) acc[g][i] = fmaf(pt, v[uu][i], acc[g][i]);
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < ATT_GROUP; g++)
            if (g < gn)
#pragma unroll
                for (int i = 0; i < DPLC; i++)
                    if (i < dpl) red[(warp * ATT_GROUP + g) * Dh + lane + 32 * i] = acc[g][i];
        __syncthreads();
        for (int idx = threadIdx.x; idx < gn * Dh; idx += NTH) {
            const int gl = idx / Dh, d = idx % Dh, g = g0 + gl;
            float s = 0.0f;
            for (int w = 0; w < nw; w++) s += red[(w * ATT_GROUP + gl) * Dh + d];
            if (a.nsplit == 1 || single) {
                a.out[(size_t)b * a.ldo + ((size_t)kh * G + g) * Dh + d] = s / ml[2 * g + 1];
            } else {
                wsb[g * hstride + d] = s;
                if (d == 0) { wsb[g * hstride + Dh] = ml[2 * g]; wsb[g * hstride + Dh + 1] = ml[2 * g + 1]; }
            }
        }
        __syncthreads();  // red is reused by the next group
    }
}

// After split_body, with arrival counters: the last of the splits that hold
// positions (0..pos) to arrive merges them (as k_attn_combine); empty splits
// take no part.  `last` is one int of shared memory.  Every thread of the
// CTA calls this (it synchronises the CTA).
template <int NTH>
__device__ __forceinline__ void attn_merge_last(const AttnArgs &a, const float *wsb, size_t hstride, int kh, int b,
                                                int pos, int *last, int ch = 0) {
    const int G = a.H / a.Hkv, Dh = a.Dh;
    const int active = min(a.nsplit, pos / (ch ? ch : a.CH) + 1);
    if (active == 1) {  // the only split: normalise its own accumulator
        __syncthreads();
        for (int i = threadIdx.x; i < G * Dh; i += NTH) {
            const int g = i / Dh, d = i % Dh;
            a.out[(size_t)b * a.ldo + ((size_t)kh * G + g) * Dh + d] = wsb[g * hstride + d] / wsb[g * hstride + Dh + 1];
        }
        return;
    }
    __threadfence();  // this CTA's partials are visible to the merging CTA
    __syncthreads();
    if (threadIdx.x == 0) *last = atomicAdd(a.cnt + (size_t)b * a.Hkv + kh, 1) == active - 1;
    __syncthreads();
    if (!*last) return;
    __threadfence();
    for (int i = threadIdx.x; i < G * Dh; i += NTH) {
        const int g = i / Dh, d = i % Dh;
        const float *w = a.ws + ((size_t)b * a.H + (size_t)kh * G + g) * hstride;
        float M = -INFINITY;
        for (int s2 = 0; s2 < active; s2++) M = fmaxf(M, __ldcg(w + s2 * (Dh + 2) + Dh));
        float L = 0.0f, acc = 0.0f;
        for (int s2 = 0; s2 < active; s2++) {
            const float l = __ldcg(w + s2 * (Dh + 2) + Dh + 1);
            if (l == 0.0f) continue;
            const float f = expf(__ldcg(w + s2 * (Dh + 2) + Dh) - M);
            L += l * f;
            acc += __ldcg(w + s2 * (Dh + 2) + d) * f;
        }
        a.out[(size_t)b * a.ldo + ((size_t)kh * G + g) * Dh + d] = acc / L;
    }
    if (threadIdx.x == 0) a.cnt[(size_t)b * a.Hkv + kh] = 0;  // ready for the next step
}

}  // namespace
