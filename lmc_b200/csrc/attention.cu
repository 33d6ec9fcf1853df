// attention.cu - K4: decode-step attention over the head-major KV cache.
//
// Replaces the cache write and per-head read of LMc attention_forward
// (src/ops.c:122-178) and llama_attention_forward (src/ops_llama.c:80-134):
// scores = q . k_t / sqrt(Dh) for t <= pos, softmax, out = sum_t p_t v_t.
//
// Split-K over the context (flash-decoding): CTA (split, kv head, sequence)
// covers CH positions and all G = H / Hkv query heads of its kv head, so each
// K/V row is read from HBM once per group, not once per query head.  A split
// writes (max, exp-sum, unnormalised accumulator) to the caller's workspace;
// k_attn_combine merges the splits -- or, with arrival counters (the model's
// step), the last split CTA of each (sequence, kv head) to finish merges them
// in the same launch.  The CTA whose range holds `pos` first
// appends the new K/V row to the cache (rounded to the cache type, so the
// step reads exactly what later steps will read).
#include <cuda_fp16.h>

#include "lmc_common.cuh"
#include "lmc_internal.h"

#define ATT_THREADS 128
#define ATT_MAX_SPLITS 16

#include "attention.cuh"

template <typename KV, int DH>
__device__ __forceinline__ void split_body_tc(const AttnArgs &a, float *sm, int kh, int b, int pos, int t0, int t1,
                                              float *wsb, size_t hstride);

// DH: the head size when it is 64 or 128 (compile-time register layout), 0 for any other.
// TC: the tensor-core body (fp16 cache, DH 64 / 128, at most 8 query heads per kv head).
template <typename KV, int DH, bool TC>
__global__ void __launch_bounds__(ATT_THREADS) k_attn_split(AttnArgs a) {
    extern __shared__ float sm[];
    const int sp = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
    const int G = a.H / a.Hkv, Dh = a.Dh, CH = a.CH;
    pdl_wait();
    pdl_launch_dependents();
    const int pos = a.pos[b];
    if (pos < 0 || pos >= a.S) return;  // the host validates positions; never index outside the cache
    const int t0 = sp * CH, t1 = min(t0 + CH, pos + 1);
    float *wsb = a.ws + (((size_t)b * a.H + (size_t)kh * G) * a.nsplit + sp) * (Dh + 2);
    const size_t hstride = (size_t)a.nsplit * (Dh + 2);
    if (t0 > pos) {  // empty split
        if (a.nsplit > 1 && !a.cnt)  // mark it so the combine kernel skips it
            for (int g = threadIdx.x; g < G; g += ATT_THREADS) {
                wsb[g * hstride + Dh] = -INFINITY;
                wsb[g * hstride + Dh + 1] = 0.0f;
            }
        return;
    }
    if constexpr (TC) split_body_tc<KV, DH>(a, sm, kh, b, pos, t0, t1, wsb, hstride);
    else split_body<KV, DH>(a, sm, sp, kh, b, pos, t0, t1, wsb, hstride);
    if (!a.cnt || a.nsplit == 1) return;
    __shared__ int last;
    attn_merge_last<ATT_THREADS>(a, wsb, hstride, kh, b, pos, &last);
}

// ---------------------------------------------------------------------------
// Tensor-core split body (fp16 cache).  The group's G <= 8 query heads are
// the rows of mma.sync m16n8k16 tiles (rows G..15 zero):
//   scores: A = q (fp16 hi + lo parts, two MMAs, so the product carries q to
//     ~22 bits; K is exact in fp16), B = 8 cached positions x 16 dims read
//     straight from the cache, one 16-byte load per lane and 32 dims (the k
//     index is permuted within each 32 dims, identically in A and B);
//   out = P V: A = the probabilities e^(s - m) (hi + lo), B = V rows staged in
//     shared memory (padded rows) and read transposed with ldmatrix; each
//     warp owns DH / 32 of the 8-dim column tiles, so no cross-warp sum.
// Same statistics and outputs as split_body; fp32 accumulation throughout.
__device__ __forceinline__ void hmma16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void split_h2(float x, float y, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 f = __half22float2(h);
    const __half2 l = __floats2half2_rn(x - f.x, y - f.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}
// Dim of logical k (0..15) of slice ks (within its 32-dim pair kp = ks / 2)
// for lane group tig: the 16-byte load of dims 32 kp + 8 tig .. + 7 feeds
// b0 / b1 of slices 2 kp and 2 kp + 1.
__device__ __forceinline__ int qk_dim(int ks, int tig, int e, bool second) {
    return 32 * (ks >> 1) + 8 * tig + 4 * (ks & 1) + (second ? 2 : 0) + e;
}

// 8 int8 codes (one 8-byte word) -> 8 exact halves: (code ^ 0x80) under the
// fp16 1024 (0x64xx = 1024 + byte), minus 1152.
__device__ __forceinline__ uint4 q8x8_to_h8(uint2 w) {
    const uint32_t a = w.x ^ 0x80808080u, c = w.y ^ 0x80808080u;
    const __half2 off = __floats2half2_rn(1152.0f, 1152.0f);
    uint4 r;
    __half2 h;
    h = __hsub2(*reinterpret_cast<const __half2 *>(&(const uint32_t &)__byte_perm(a, 0x64646464u, 0x4140u)), off);
    r.x = *reinterpret_cast<uint32_t *>(&h);
    h = __hsub2(*reinterpret_cast<const __half2 *>(&(const uint32_t &)__byte_perm(a, 0x64646464u, 0x4342u)), off);
    r.y = *reinterpret_cast<uint32_t *>(&h);
    h = __hsub2(*reinterpret_cast<const __half2 *>(&(const uint32_t &)__byte_perm(c, 0x64646464u, 0x4140u)), off);
    r.z = *reinterpret_cast<uint32_t *>(&h);
    h = __hsub2(*reinterpret_cast<const __half2 *>(&(const uint32_t &)__byte_perm(c, 0x64646464u, 0x4342u)), off);
    r.w = *reinterpret_cast<uint32_t *>(&h);
    return r;
}

// KV: __half (fp16 rows) or KvQ8 (int8 rows: the codes go into the MMAs as
// exact halves; the K row scale multiplies the score, the V row scale is
// folded into the probability after the softmax sum).
template <typename KV, int DH>
__device__ __forceinline__ void split_body_tc(const AttnArgs &a, float *sm, int kh, int b, int pos, int t0, int t1,
                                              float *wsb, size_t hstride) {
    constexpr int KS = DH / 16, VSTR = DH + 8;  // k slices; V staging row stride (halves, conflict-free ldmatrix)
    constexpr bool Q8 = KvT<KV>::Q8;
    constexpr int RS = kv_rs<KV>(DH);  // row stride in elements of KV
    const int G = a.H / a.Hkv, CH = a.CH;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = ATT_THREADS / 32;
    const int g = lane >> 2, tig = lane & 3;
    float *qs = sm;            // [G][DH]
    float *sc = sm + G * DH;   // [G][CH16]
    const int CH16 = (CH + 15) & ~15;
    float *ml = sc + G * CH16;  // [G][2]
    float *vsc = ml + 2 * G;    // [CH16] V row scales (int8 rows)
    __half *vt = reinterpret_cast<__half *>(sm + ((G * DH + G * CH16 + 2 * G + (Q8 ? CH16 : 0) + 3) & ~3));  // [CH16][VSTR], 16-byte aligned
    const size_t cs = a.seq ? (size_t)a.seq[b] : (size_t)b;
    KV *const kpool = reinterpret_cast<KV *>(a.k_cache), *const vpool = reinterpret_cast<KV *>(a.v_cache);
    KV *kc = kpool + (cs * a.Hkv + kh) * a.S * RS;
    KV *vc = vpool + (cs * a.Hkv + kh) * a.S * RS;
    // row t of this (sequence, kv head): contiguous, or through the page table
    auto row = [&](KV *seqbase, KV *pool, int t) -> KV * {
        return a.pages ? kv_page_row<KV>(a, pool, cs, kh, t, RS) : seqbase + (size_t)t * RS;
    };
    const float *rc = a.rope_cos ? a.rope_cos + (size_t)pos * (DH / 2) : nullptr;
    const float *rs = a.rope_sin ? a.rope_sin + (size_t)pos * (DH / 2) : nullptr;
    if (Q8 && a.append && pos >= t0 && pos < t1) {  // quantize the new rows: warp 0 K, warp 1 V
        if (warp < 2)
            kv_q8_store_row(reinterpret_cast<KvQ8 *>(warp ? row(vc, vpool, pos) : row(kc, kpool, pos)),
                            (warp ? a.v_new : a.k_new) + (size_t)b * a.ldkv + (size_t)kh * DH, warp ? nullptr : rc,
                            rs, DH, lane);
    } else if (a.append && pos >= t0 && pos < t1) {  // append this step's K/V row (K rotated first when RoPE applies)
        const float *kn = a.k_new + (size_t)b * a.ldkv + (size_t)kh * DH;
        const float *vn = a.v_new + (size_t)b * a.ldkv + (size_t)kh * DH;
        KV *kp = row(kc, kpool, pos), *vp = row(vc, vpool, pos);
        for (int d = threadIdx.x; d < DH / 2; d += ATT_THREADS) {
            float k0 = kn[2 * d], k1 = kn[2 * d + 1];
            if (rc) {
                const float c = rc[d], sn = rs[d];
                const float r0 = k0 * c - k1 * sn, r1 = k0 * sn + k1 * c;
                k0 = r0;
                k1 = r1;
            }
            if constexpr (!Q8) {
                kp[2 * d] = __float2half_rn(k0);
                kp[2 * d + 1] = __float2half_rn(k1);
                vp[2 * d] = __float2half_rn(vn[2 * d]);
                vp[2 * d + 1] = __float2half_rn(vn[2 * d + 1]);
            }
        }
    }
    const float *qb = a.q + (size_t)b * a.ldq + (size_t)kh * G * DH;
    for (int i = threadIdx.x; i < G * DH / 2; i += ATT_THREADS) {  // q pairs (rotated when RoPE applies)
        const int gq = i / (DH / 2), d = i % (DH / 2);
        float q0 = qb[gq * DH + 2 * d], q1 = qb[gq * DH + 2 * d + 1];
        if (rc) {
            const float c = rc[d], sn = rs[d];
            const float r0 = q0 * c - q1 * sn, r1 = q0 * sn + q1 * c;
            q0 = r0;
            q1 = r1;
        }
        qs[gq * DH + 2 * d] = q0;
        qs[gq * DH + 2 * d + 1] = q1;
    }
    __syncthreads();  // the new row (read back below) and q are in place
    const int n = t1 - t0, n16 = (n + 15) & ~15;
    // stage V rows [t0, t0 + n) (zero rows up to n16): fp16 rows by
    // asynchronous 16-byte copies that land while the scores are computed
    // (waited before the output); int8 rows converted to halves here, their
    // scales kept in vsc
    if constexpr (Q8) {
        for (int i = threadIdx.x; i < n16 * (DH / 8); i += ATT_THREADS) {
            const int r = i / (DH / 8), c8 = i % (DH / 8);
            const KV *vrow = row(vc, vpool, t0 + (r < n ? r : 0));
            const uint2 w = r < n ? *reinterpret_cast<const uint2 *>(reinterpret_cast<const uint8_t *>(vrow) + 8 * c8)
                                  : make_uint2(0x80808080u ^ 0x80808080u, 0u);
            *reinterpret_cast<uint4 *>(vt + r * VSTR + 8 * c8) = r < n ? q8x8_to_h8(w) : make_uint4(0u, 0u, 0u, 0u);
            if (c8 == 0) vsc[r] = r < n ? kv_q8_scale(reinterpret_cast<const KvQ8 *>(vrow), DH) : 0.0f;
        }
    } else {
        for (int i = threadIdx.x; i < n16 * (DH / 8); i += ATT_THREADS) {
            const int r = i / (DH / 8), c8 = i % (DH / 8);
            const KV *src = row(vc, vpool, t0 + (r < n ? r : 0)) + 8 * c8;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(vt + r * VSTR + 8 * c8)),
                         "l"(src), "r"(r < n ? 16 : 0)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    // q fragments: row g (query head g of the group), hi and lo
    uint32_t qa0h[KS], qa0l[KS], qa2h[KS], qa2l[KS];
#pragma unroll
    for (int ks = 0; ks < KS; ks++) {
        float x0 = 0.f, x1 = 0.f, y0 = 0.f, y1 = 0.f;
        if (g < G) {
            const float *qr = qs + g * DH;
            x0 = qr[qk_dim(ks, tig, 0, false)], x1 = qr[qk_dim(ks, tig, 1, false)];
            y0 = qr[qk_dim(ks, tig, 0, true)], y1 = qr[qk_dim(ks, tig, 1, true)];
        }
        split_h2(x0, x1, qa0h[ks], qa0l[ks]);
        split_h2(y0, y1, qa2h[ks], qa2l[ks]);
    }
    const float scale = 1.0f / sqrtf((float)DH);
    constexpr int TB = DH == 128 ? 2 : 4;  // tiles per warp whose K loads are issued together
    for (int j0 = warp; 8 * j0 < n; j0 += TB * nw) {  // 8-position tiles j0, j0 + nw, ...
        uint4 kv[TB][KS / 2];
        float ksc[TB];  // int8 rows: the scale of this lane's K row
#pragma unroll
        for (int u = 0; u < TB; u++) {
            const int p = 8 * (j0 + u * nw) + g;  // this lane's B column (position within the split)
            if constexpr (Q8) {
                const KV *krow = row(kc, kpool, t0 + (p < n ? p : 0));
                const uint8_t *kr = reinterpret_cast<const uint8_t *>(krow) + 8 * tig;
#pragma unroll
                for (int kp = 0; kp < KS / 2; kp++)
                    kv[u][kp] = p < n ? q8x8_to_h8(*reinterpret_cast<const uint2 *>(kr + 32 * kp))
                                      : make_uint4(0u, 0u, 0u, 0u);
                ksc[u] = p < n ? kv_q8_scale(reinterpret_cast<const KvQ8 *>(krow), DH) : 0.0f;
            } else {
                const KV *kr = row(kc, kpool, t0 + (p < n ? p : 0)) + 8 * tig;
#pragma unroll
                for (int kp = 0; kp < KS / 2; kp++)
                    kv[u][kp] = p < n ? *reinterpret_cast<const uint4 *>(kr + 32 * kp) : make_uint4(0u, 0u, 0u, 0u);
                ksc[u] = 1.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < TB; u++) {
            const int j = j0 + u * nw;
            if (8 * j >= n) break;
            float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kp = 0; kp < KS / 2; kp++) {
                hmma16816(d, qa0h[2 * kp], qa2h[2 * kp], kv[u][kp].x, kv[u][kp].y);
                hmma16816(d, qa0l[2 * kp], qa2l[2 * kp], kv[u][kp].x, kv[u][kp].y);
                hmma16816(d, qa0h[2 * kp + 1], qa2h[2 * kp + 1], kv[u][kp].z, kv[u][kp].w);
                hmma16816(d, qa0l[2 * kp + 1], qa2l[2 * kp + 1], kv[u][kp].z, kv[u][kp].w);
            }
            // d[0], d[1]: head g at positions 8 j + 2 tig, + 1 (rows 8-15 are padding)
            const int c0 = 8 * j + 2 * tig;
            if (Q8) {  // K row scales of positions 2 tig, 2 tig + 1: held by lanes with g = 2 tig, 2 tig + 1
                d[0] *= __shfl_sync(0xffffffffu, ksc[u], 8 * tig);
                d[1] *= __shfl_sync(0xffffffffu, ksc[u], 8 * tig + 4);
            }
            if (g < G) {
                if (c0 < n) sc[g * CH16 + c0] = d[0] * scale;
                if (c0 + 1 < n) sc[g * CH16 + c0 + 1] = d[1] * scale;
            }
        }
    }
    __syncthreads();
    for (int gg = warp; gg < G; gg += nw) {
        float m = -INFINITY;
        for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[gg * CH16 + t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < n16; t += 32) {
            const float e = t < n ? expf(sc[gg * CH16 + t] - m) : 0.0f;
            sc[gg * CH16 + t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { ml[2 * gg] = m; ml[2 * gg + 1] = l; }
    }
    if (Q8) {  // the V row scales into the probabilities (the sum above is of the unscaled ones)
        __syncthreads();  // vsc is written by the staging loop
        for (int i = threadIdx.x; i < G * n16; i += ATT_THREADS) sc[(i / n16) * CH16 + i % n16] *= vsc[i % n16];
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // this thread's V copies landed
    __syncthreads();                                   // and every thread's
    // out = P V: warp w owns the 8-dim column tiles w, w + nw, ...
    constexpr int NTW = DH / 8 / (ATT_THREADS / 32);
    float o[NTW][4];
#pragma unroll
    for (int i = 0; i < NTW; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    const uint32_t vbase = (uint32_t)__cvta_generic_to_shared(vt);
    for (int kk = 0; kk < n16; kk += 16) {
        float x0 = 0.f, x1 = 0.f, y0 = 0.f, y1 = 0.f;
        if (g < G) {
            const float *pr = sc + g * CH16 + kk;
            x0 = pr[2 * tig], x1 = pr[2 * tig + 1], y0 = pr[8 + 2 * tig], y1 = pr[8 + 2 * tig + 1];
        }
        uint32_t pa0h, pa0l, pa2h, pa2l;
        split_h2(x0, x1, pa0h, pa0l);
        split_h2(y0, y1, pa2h, pa2l);
#pragma unroll
        for (int i = 0; i < NTW; i++) {
            const int nt = warp + i * nw;
            // lanes 0-15 address rows kk + lane of the 16 x 8 V tile (column block nt)
            const uint32_t addr = vbase + (uint32_t)(((kk + (lane & 15)) * VSTR + 8 * nt) * 2);
            uint32_t b0, b1;
            asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(addr));
            hmma16816(o[i], pa0h, pa2h, b0, b1);
            hmma16816(o[i], pa0l, pa2l, b0, b1);
        }
    }
    if (g < G) {
#pragma unroll
        for (int i = 0; i < NTW; i++) {
            const int d = 8 * (warp + i * nw) + 2 * tig;
            if (a.nsplit == 1) {
                const float inv = 1.0f / ml[2 * g + 1];
                float *op = a.out + (size_t)b * a.ldo + ((size_t)kh * G + g) * DH + d;
                op[0] = o[i][0] * inv;
                op[1] = o[i][1] * inv;
            } else {
                wsb[g * hstride + d] = o[i][0];
                wsb[g * hstride + d + 1] = o[i][1];
                if (d == 0) { wsb[g * hstride + DH] = ml[2 * g]; wsb[g * hstride + DH + 1] = ml[2 * g + 1]; }
            }
        }
    }
}

// K/V append for rows that share a cache sequence: row b's new K (rotated
// when RoPE applies) and V rows go to position pos[b] of sequence seq[b],
// before the attention launch reads them.  One CTA per (kv head, row).
template <typename KV>
__global__ void k_kv_append(AttnArgs a) {
    pdl_wait();
    pdl_launch_dependents();
    const int kh = blockIdx.x, b = blockIdx.y, Dh = a.Dh;
    const int pos = a.pos[b];
    if (pos < 0 || pos >= a.S) return;
    const size_t cs = (size_t)a.seq[b];
    const int RS = kv_rs<KV>(Dh);
    KV *const kpool = reinterpret_cast<KV *>(a.k_cache), *const vpool = reinterpret_cast<KV *>(a.v_cache);
    KV *kc = a.pages ? kv_page_row<KV>(a, kpool, cs, kh, pos, RS) : kpool + ((cs * a.Hkv + kh) * a.S + pos) * RS;
    KV *vc = a.pages ? kv_page_row<KV>(a, vpool, cs, kh, pos, RS) : vpool + ((cs * a.Hkv + kh) * a.S + pos) * RS;
    const float *kn = a.k_new + (size_t)b * a.ldkv + (size_t)kh * Dh;
    const float *vn = a.v_new + (size_t)b * a.ldkv + (size_t)kh * Dh;
    const float *rc = a.rope_cos ? a.rope_cos + (size_t)pos * (Dh / 2) : nullptr;
    const float *rs = a.rope_sin ? a.rope_sin + (size_t)pos * (Dh / 2) : nullptr;
    if constexpr (KvT<KV>::Q8) {  // two warps: K, V
        const int w = threadIdx.x >> 5;
        if (w < 2)
            kv_q8_store_row(reinterpret_cast<KvQ8 *>(w ? vc : kc), w ? vn : kn, w ? nullptr : rc, rs, Dh,
                            threadIdx.x & 31);
    } else {
    for (int d = threadIdx.x; d < Dh / 2; d += blockDim.x) {
        float k0 = kn[2 * d], k1 = kn[2 * d + 1];
        if (rc) {
            const float c = rc[d], sn = rs[d];
            const float r0 = k0 * c - k1 * sn, r1 = k0 * sn + k1 * c;
            k0 = r0;
            k1 = r1;
        }
        kc[2 * d] = kv_cvt<KV>(k0);
        kc[2 * d + 1] = kv_cvt<KV>(k1);
        vc[2 * d] = kv_cvt<KV>(vn[2 * d]);
        vc[2 * d + 1] = kv_cvt<KV>(vn[2 * d + 1]);
    }
    }
}

// Merge the splits of one (sequence, query head): rescale each split's sum
// and accumulator to the global maximum.
__global__ void k_attn_combine(AttnArgs a) {
    pdl_wait();
    pdl_launch_dependents();
    const int h = blockIdx.x, b = blockIdx.y, Dh = a.Dh;
    const float *w = a.ws + ((size_t)b * a.H + h) * a.nsplit * (Dh + 2);
    float M = -INFINITY;
    for (int s = 0; s < a.nsplit; s++) M = fmaxf(M, w[s * (Dh + 2) + Dh]);
    for (int d = threadIdx.x; d < Dh; d += blockDim.x) {
        float L = 0.0f, acc = 0.0f;
        for (int s = 0; s < a.nsplit; s++) {
            const float l = w[s * (Dh + 2) + Dh + 1];
            if (l == 0.0f) continue;
            const float f = expf(w[s * (Dh + 2) + Dh] - M);
            L += l * f;
            acc += w[s * (Dh + 2) + d] * f;
        }
        a.out[(size_t)b * a.ldo + (size_t)h * Dh + d] = acc / L;
    }
}

// Split length: 64 positions, longer while the context would need more than
// ATT_MAX_SPLITS splits.  When the splits are merged in the launch (`fine`:
// arrival counters given) and there are few (sequence, head) pairs (bh =
// batch x heads, a batch-1 decode), shorter, down to 16 positions and
// ATT_MAX_SPLITS_FEW splits, so that more CTAs stream the cache at once (a
// separate merge kernel over that many splits costs more than it saves).
#define ATT_MAX_SPLITS_FEW 64
static void attn_plan(int S, int bh, bool fine, int *CH, int *nsplit) {
    int ch = 64;
    while ((S + ch - 1) / ch > ATT_MAX_SPLITS) ch *= 2;
    while (fine && ch > 16 && (long long)bh * ((S + ch - 1) / ch) < 2048 &&
           (S + ch / 2 - 1) / (ch / 2) <= ATT_MAX_SPLITS_FEW)
        ch /= 2;
    *CH = ch;
    *nsplit = (S + ch - 1) / ch;
}

extern "C" void lmc_attn_plan(int S, int bh, int fine, int *CH, int *nsplit) { attn_plan(S, bh, fine != 0, CH, nsplit); }

extern "C" size_t lmc_attention_workspace_bytes(int batch, int H, int Dh, int S) {
    int CH, ns;
    attn_plan(S, batch * H, true, &CH, &ns);  // the larger of the two plans
    return ns > 1 ? (size_t)batch * H * ns * (Dh + 2) * sizeof(float) : 0;
}

extern "C" int lmc_attention_launch(float *out, int ldo, const float *q, int ldq, const float *k_new,
                                    const float *v_new, int ldkv, void *k_cache, void *v_cache, int kv_dtype,
                                    const int *d_pos, int batch, int H, int Hkv, int Dh, int S, void *d_ws,
                                    size_t ws_bytes, int *d_cnt, cudaStream_t s) {
    return lmc_attention_rope_launch(out, ldo, q, ldq, k_new, v_new, ldkv, k_cache, v_cache, kv_dtype, d_pos, batch, H,
                                     Hkv, Dh, S, d_ws, ws_bytes, NULL, NULL, d_cnt, s);
}

extern "C" int lmc_attention_rope_launch(float *out, int ldo, const float *q, int ldq, const float *k_new,
                                         const float *v_new, int ldkv, void *k_cache, void *v_cache, int kv_dtype,
                                         const int *d_pos, int batch, int H, int Hkv, int Dh, int S, void *d_ws,
                                         size_t ws_bytes, const float *rope_cos, const float *rope_sin, int *d_cnt,
                                         cudaStream_t s) {
    return lmc_attention_rows_launch(out, ldo, q, ldq, k_new, v_new, ldkv, k_cache, v_cache, kv_dtype, d_pos, NULL,
                                     batch, H, Hkv, Dh, S, d_ws, ws_bytes, rope_cos, rope_sin, d_cnt, s);
}

// pages: NULL, or the page table of a paged cache (attention.cuh AttnArgs)
static int attention_impl(float *out, int ldo, const float *q, int ldq, const float *k_new, const float *v_new,
                          int ldkv, void *k_cache, void *v_cache, int kv_dtype, const int *d_pos, const int *d_seq,
                          int batch, int H, int Hkv, int Dh, int S, void *d_ws, size_t ws_bytes,
                          const float *rope_cos, const float *rope_sin, int *d_cnt, const int *pages, int page_shift,
                          int max_pages, int n_pages, cudaStream_t s) {
    if (!out || !q || !k_new || !v_new || !k_cache || !v_cache || !d_pos)
        return lmc_set_error(LMC_ERR_INVALID, "attention: null pointer");
    if (batch <= 0 || H <= 0 || Hkv <= 0 || H % Hkv || Dh % 32 || Dh > 256 || S <= 0)
        return lmc_set_error(LMC_ERR_INVALID, "attention: H=%d Hkv=%d Dh=%d S=%d (need H%%Hkv==0, Dh%%32==0, Dh<=256)",
                             H, Hkv, Dh, S);
    if (kv_dtype != LMC_KV_F32 && kv_dtype != LMC_KV_F16 && kv_dtype != LMC_KV_Q8)
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "attention: kv dtype %d", kv_dtype);
    if (kv_dtype == LMC_KV_Q8 && (Dh % 16 || Dh > 512))
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "attention: int8 rows need a head size that is a multiple of 16, <= 512");
    AttnArgs a;
    a.out = out; a.q = q; a.k_new = k_new; a.v_new = v_new; a.k_cache = k_cache; a.v_cache = v_cache;
    a.pos = d_pos; a.H = H; a.Hkv = Hkv; a.Dh = Dh; a.S = S;
    a.ldo = ldo; a.ldq = ldq; a.ldkv = ldkv;
    a.rope_cos = rope_cos; a.rope_sin = rope_sin;
    a.cnt = d_cnt;
    a.seq = d_seq;
    a.append = d_seq ? 0 : 1;
    a.pages = pages;
    a.page_shift = page_shift;
    a.max_pages = max_pages;
    a.n_pages = n_pages;
    attn_plan(S, batch * H, d_cnt != NULL, &a.CH, &a.nsplit);
    const size_t need = a.nsplit > 1 ? (size_t)batch * H * a.nsplit * (Dh + 2) * sizeof(float) : 0;  // this launch's plan
    if (need > ws_bytes || (need && !d_ws))
        return lmc_set_error(LMC_ERR_INVALID, "attention: workspace %zu bytes < %zu needed", ws_bytes, need);
    a.ws = (float *)d_ws;
    const int G = H / Hkv;
    // tensor-core body: fp16 cache, head 64 / 128, 1-8 query heads per kv head
    // (LMC_ATTN_TC=0 selects the CUDA-core body; both give the same result)
    const char *tce = getenv("LMC_ATTN_TC");
    const bool tc = (kv_dtype == LMC_KV_F16 || kv_dtype == LMC_KV_Q8) && (Dh == 64 || Dh == 128) && G <= 8 &&
                    !(tce && tce[0] == '0');
    const int CH16 = (a.CH + 15) & ~15;
    const size_t smem = tc ? (size_t)(G * Dh + G * CH16 + 2 * G + CH16 + 2) * sizeof(float) + 16 + (size_t)CH16 * (Dh + 8) * 2
                           : (size_t)(G * Dh + G * a.CH + 2 * G + (ATT_THREADS / 32) * ATT_GROUP * Dh) * sizeof(float);
    if (smem > 200 * 1024) return lmc_set_error(LMC_ERR_UNSUPPORTED, "attention: group too large");
    dim3 grid(a.nsplit, Hkv, batch);
    if (d_seq) {  // rows share cache sequences: append every row's K/V first
        if (kv_dtype == LMC_KV_F32) LMC_LAUNCH("kv append", k_kv_append<float>, dim3(Hkv, batch), 64, 0, s, a);
        else if (kv_dtype == LMC_KV_Q8) LMC_LAUNCH("kv append", k_kv_append<KvQ8>, dim3(Hkv, batch), 64, 0, s, a);
        else LMC_LAUNCH("kv append", k_kv_append<__half>, dim3(Hkv, batch), 64, 0, s, a);
    }
    if (kv_dtype == LMC_KV_F32) {
        void (*fn)(AttnArgs) = Dh == 64 ? k_attn_split<float, 64, false> : Dh == 128 ? k_attn_split<float, 128, false>
                                                                      : k_attn_split<float, 0, false>;
        if (smem > 48 * 1024) LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        LMC_LAUNCH("attention", fn, grid, ATT_THREADS, smem, s, a);
    } else if (kv_dtype == LMC_KV_Q8) {
        void (*fn)(AttnArgs) = tc ? (Dh == 64 ? k_attn_split<KvQ8, 64, true> : k_attn_split<KvQ8, 128, true>)
                                  : Dh == 64 ? k_attn_split<KvQ8, 64, false> : Dh == 128 ? k_attn_split<KvQ8, 128, false>
                                                                                : k_attn_split<KvQ8, 0, false>;
        if (smem > 48 * 1024) LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        LMC_LAUNCH("attention", fn, grid, ATT_THREADS, smem, s, a);
    } else {
        void (*fn)(AttnArgs) = tc ? (Dh == 64 ? k_attn_split<__half, 64, true> : k_attn_split<__half, 128, true>)
                                  : Dh == 64 ? k_attn_split<__half, 64, false> : Dh == 128 ? k_attn_split<__half, 128, false>
                                                                                  : k_attn_split<__half, 0, false>;
        if (smem > 48 * 1024) LMC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        LMC_LAUNCH("attention", fn, grid, ATT_THREADS, smem, s, a);
    }
    if (a.nsplit > 1 && !d_cnt) {
        LMC_LAUNCH("attention combine", k_attn_combine, dim3(H, batch), Dh, 0, s, a);
    }
    return LMC_OK;
}

extern "C" int lmc_attention_rows_launch(float *out, int ldo, const float *q, int ldq, const float *k_new,
                                         const float *v_new, int ldkv, void *k_cache, void *v_cache, int kv_dtype,
                                         const int *d_pos, const int *d_seq, int batch, int H, int Hkv, int Dh, int S,
                                         void *d_ws, size_t ws_bytes, const float *rope_cos, const float *rope_sin,
                                         int *d_cnt, cudaStream_t s) {
    return attention_impl(out, ldo, q, ldq, k_new, v_new, ldkv, k_cache, v_cache, kv_dtype, d_pos, d_seq, batch, H,
                          Hkv, Dh, S, d_ws, ws_bytes, rope_cos, rope_sin, d_cnt, NULL, 0, 0, 0, s);
}

extern "C" int lmc_attention_rows_paged_launch(float *out, int ldo, const float *q, int ldq, const float *k_new,
                                               const float *v_new, int ldkv, void *k_pool, void *v_pool, int kv_dtype,
                                               const int *d_pos, const int *d_seq, int batch, int H, int Hkv, int Dh,
                                               const int *d_pages, int max_pages, int page_shift, int n_pages,
                                               void *d_ws, size_t ws_bytes, const float *rope_cos,
                                               const float *rope_sin, int *d_cnt, cudaStream_t s) {
    if (!d_pages || n_pages <= 0 || max_pages <= 0 || page_shift < 0 || page_shift > 24 ||
        (long long)max_pages << page_shift > (1 << 24))
        return lmc_set_error(LMC_ERR_INVALID, "attention_rows_paged: pages %d, table %d x page 2^%d", n_pages,
                             max_pages, page_shift);
    return attention_impl(out, ldo, q, ldq, k_new, v_new, ldkv, k_pool, v_pool, kv_dtype, d_pos, d_seq, batch, H, Hkv,
                          Dh, max_pages << page_shift, d_ws, ws_bytes, rope_cos, rope_sin, d_cnt, d_pages, page_shift,
                          max_pages, n_pages, s);
}

extern "C" int lmc_attention_decode_paged(float *out, const float *q, const float *k_new, const float *v_new,
                                          void *k_pool, void *v_pool, int kv_dtype, int n_pages, const int *d_pages,
                                          int max_pages, int page_size, const int *d_pos, int batch, int H, int Hkv,
                                          int Dh, void *d_ws, size_t ws_bytes, void *stream) {
    if (!d_pages || n_pages <= 0 || max_pages <= 0 || page_size < 16 || (page_size & (page_size - 1)) ||
        (long long)max_pages * page_size > (1 << 24))
        return lmc_set_error(LMC_ERR_INVALID, "attention_paged: pages %d, table %d x page %d", n_pages, max_pages,
                             page_size);
    int shift = 0;
    while ((1 << shift) < page_size) shift++;
    return attention_impl(out, H * Dh, q, H * Dh, k_new, v_new, Hkv * Dh, k_pool, v_pool, kv_dtype, d_pos, NULL,
                          batch, H, Hkv, Dh, max_pages * page_size, d_ws, ws_bytes, NULL, NULL, NULL, d_pages, shift,
                          max_pages, n_pages, lmc_stream(stream));
}

// LMC_OK, or LMC_ERR_INVALID once after a paged attention met a page id
// outside its pool (the flag is cleared).
extern "C" int lmc_attn_status(void) {
    int v = 0;
    LMC_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_attn_page_err, sizeof(int)));
    if (!v) return LMC_OK;
    const int zero = 0;
    LMC_CUDA_TRY(cudaMemcpyToSymbol(g_attn_page_err, &zero, sizeof(int)));
    return lmc_set_error(LMC_ERR_INVALID, "paged attention: a page id outside the pool (page 0 read instead)");
}

extern "C" int lmc_attention_decode(float *out, const float *q, const float *k_new, const float *v_new,
                                    void *k_cache, void *v_cache, int kv_dtype, const int *d_pos, int batch,
                                    int H, int Hkv, int Dh, int S, void *d_ws, size_t ws_bytes, void *stream) {
    return lmc_attention_launch(out, H * Dh, q, H * Dh, k_new, v_new, Hkv * Dh, k_cache, v_cache, kv_dtype, d_pos,
                                batch, H, Hkv, Dh, S, d_ws, ws_bytes, NULL, lmc_stream(stream));
}

// ---------------------------------------------------------------------------
// Allocation-free variant of lmc_attention_decode.
//
// Some callers cannot allocate device memory at the point where they decode:
// code recorded into a CUDA graph (cudaMalloc is not a stream operation and
// cannot be captured), latency-critical loops that must not let cudaMalloc /
// cudaFree synchronize the device, and host applications that hand out all
// device memory themselves and forbid other allocations.  For them this entry
// point takes its split-context scratch from a fixed array compiled into the
// library instead of a caller-supplied workspace.
//
// The array below is file-scope device memory: every GPU that loads the
// library holds these 4 MiB until the process exits.  In host code its name
// is only a host-side stand-in, so its device address is looked up with
// cudaGetSymbolAddress once per device (on the first call made with that
// device current) and that address is what the kernels receive.
// ---------------------------------------------------------------------------
#include <mutex>

#define LMC_ATTN_STATIC_SCRATCH_BYTES (4u << 20)
#define LMC_MAX_DEVICES 64

static __device__ __align__(256) unsigned char g_attn_static_scratch[LMC_ATTN_STATIC_SCRATCH_BYTES];
static void *g_attn_static_ptr[LMC_MAX_DEVICES];
static std::mutex g_attn_static_mu;

extern "C" int lmc_attention_decode_noalloc(float *out, const float *q, const float *k_new, const float *v_new,
                                            void *k_cache, void *v_cache, int kv_dtype, const int *d_pos,
                                            int batch, int H, int Hkv, int Dh, int S, void *stream) {
    // every argument check comes before the first CUDA call (the symbol
    // lookup below may create the context and load the module)
    if (!out || !q || !k_new || !v_new || !k_cache || !v_cache || !d_pos)
        return lmc_set_error(LMC_ERR_INVALID, "attention_noalloc: null pointer");
    if (batch <= 0 || H <= 0 || Hkv <= 0 || H % Hkv || Dh <= 0 || Dh % 32 || Dh > 256 || S <= 0)
        return lmc_set_error(LMC_ERR_INVALID, "attention_noalloc: batch=%d H=%d Hkv=%d Dh=%d S=%d", batch, H, Hkv,
                             Dh, S);
    if (kv_dtype != LMC_KV_F32 && kv_dtype != LMC_KV_F16 && kv_dtype != LMC_KV_Q8)
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "attention_noalloc: kv dtype %d", kv_dtype);
    const size_t need = lmc_attention_workspace_bytes(batch, H, Dh, S);
    if (need > LMC_ATTN_STATIC_SCRATCH_BYTES)
        return lmc_set_error(LMC_ERR_INVALID,
                             "attention_noalloc: this shape needs %zu bytes of scratch, more than the fixed %u "
                             "(batch x heads x context splits x (head_dim + 2) x 4 bytes); use "
                             "lmc_attention_decode with a workspace",
                             need, LMC_ATTN_STATIC_SCRATCH_BYTES);
    int dev = 0;
    LMC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= LMC_MAX_DEVICES)
        return lmc_set_error(LMC_ERR_INVALID, "attention_noalloc: device %d beyond %d", dev, LMC_MAX_DEVICES);
    void *scratch;
    {
        std::lock_guard<std::mutex> lock(g_attn_static_mu);
        if (!g_attn_static_ptr[dev]) {
            void *p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
            if (e != cudaSuccess || !p)
                return lmc_set_error(LMC_ERR_CUDA, "attention_noalloc: cudaGetSymbolAddress: %s",
                                     cudaGetErrorString(e));
            g_attn_static_ptr[dev] = p;
        }
        scratch = g_attn_static_ptr[dev];
    }
    return lmc_attention_launch(out, H * Dh, q, H * Dh, k_new, v_new, Hkv * Dh, k_cache, v_cache, kv_dtype, d_pos,
                                batch, H, Hkv, Dh, S, scratch, LMC_ATTN_STATIC_SCRATCH_BYTES, NULL, lmc_stream(stream));
}
