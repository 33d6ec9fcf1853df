// lmc_blocks.cuh - bit-exact device decoders for the 13 GGUF block formats.
//
// decode8<TYPE>(block, j, y) writes the 8 consecutive fp32 weights starting
// at element j (a multiple of 8) of one block.  Each format follows LMc's
// dequant_* function (nile-agi/LMc src/quant.c, lines cited below) with the
// same float operations in the same order; products and sums use the _rn
// intrinsics so nvcc cannot contract them into FMAs, which would change the
// rounding.  Every block size is even and every fp16 field sits at an even
// offset, so 16-bit loads are aligned; 32-bit fields are assembled from two
// 16-bit loads because most block sizes are not multiples of 4.
#pragma once
#include <stdint.h>

#include "../../include/lmc_cuda.h"

#define LMC_CB_QUALIFIER static __device__ const
#include "lmc_codebooks.h"
#undef LMC_CB_QUALIFIER

namespace lmcq {

__device__ __forceinline__ uint32_t ldb(const uint8_t *p) { return __ldg(p); }
__device__ __forceinline__ uint32_t ld16(const uint8_t *p) {
    return __ldg(reinterpret_cast<const unsigned short *>(p));
}
__device__ __forceinline__ uint32_t ld32(const uint8_t *p) { return ld16(p) | (ld16(p + 2) << 16); }

// src/quant.c:19-38.  Integer-only so the result (NaN payloads included)
// matches LMc's bit manipulation exactly; __clz replaces the normalising loop.
__device__ __forceinline__ float h2f(uint32_t h) {
    uint32_t sign = (h >> 15) << 31, ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int sh = __clz(man) - 21;  // shifts until bit 10 is set
            bits = sign | ((uint32_t)(113 - sh) << 23) | (((man << sh) & 0x3FFu) << 13);
        }
    } else if (ex == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((ex + 112u) << 23) | (man << 13);
    }
    return __uint_as_float(bits);
}
__device__ __forceinline__ float f16at(const uint8_t *p) { return h2f(ld16(p)); }

// src/quant.c:44-53
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t *s, int &sc, int &m) {
    if (j < 4) {
        sc = ldb(s + j) & 63;
        m = ldb(s + j + 4) & 63;
    } else {
        sc = (ldb(s + j + 4) & 0x0F) | ((ldb(s + j - 4) >> 6) << 4);
        m = (ldb(s + j + 4) >> 4) | ((ldb(s + j) >> 6) << 4);
    }
}

template <int T> struct Fmt;
// clang-format off
template <> struct Fmt<LMC_TYPE_Q4_0>    { static constexpr int BE = 32,  BB = 18;  };
template <> struct Fmt<LMC_TYPE_Q4_1>    { static constexpr int BE = 32,  BB = 20;  };
template <> struct Fmt<LMC_TYPE_Q5_0>    { static constexpr int BE = 32,  BB = 22;  };
template <> struct Fmt<LMC_TYPE_Q5_1>    { static constexpr int BE = 32,  BB = 24;  };
template <> struct Fmt<LMC_TYPE_Q8_0>    { static constexpr int BE = 32,  BB = 34;  };
template <> struct Fmt<LMC_TYPE_Q2_K>    { static constexpr int BE = 256, BB = 84;  };
template <> struct Fmt<LMC_TYPE_Q3_K>    { static constexpr int BE = 256, BB = 110; };
template <> struct Fmt<LMC_TYPE_Q4_K>    { static constexpr int BE = 256, BB = 144; };
template <> struct Fmt<LMC_TYPE_Q5_K>    { static constexpr int BE = 256, BB = 176; };
template <> struct Fmt<LMC_TYPE_Q6_K>    { static constexpr int BE = 256, BB = 210; };
template <> struct Fmt<LMC_TYPE_IQ3_XXS> { static constexpr int BE = 256, BB = 98;  };
template <> struct Fmt<LMC_TYPE_IQ3_S>   { static constexpr int BE = 256, BB = 110; };
template <> struct Fmt<LMC_TYPE_IQ4_XS>  { static constexpr int BE = 256, BB = 136; };
template <> struct Fmt<LMC_TYPE_F32>     { static constexpr int BE = 8,   BB = 32;  };
template <> struct Fmt<LMC_TYPE_F16>     { static constexpr int BE = 8,   BB = 16;  };
// clang-format on
// (F32/F16 are treated as 8-element "blocks" so the generic kernels can
// address them like the block formats.)

template <int T> __device__ __forceinline__ void decode8(const uint8_t *b, int j, float *y);

// src/quant.c:240-252
template <> __device__ __forceinline__ void decode8<LMC_TYPE_Q4_0>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b);
    const int sh = j >= 16 ? 4 : 0, o = j & 15;
#pragma unroll
    for (int i = 0; i < 8; i++) y[i] = __fmul_rn(d, (float)((int)((ldb(b + 2 + o + i) >> sh) & 0x0F) - 8));
}
// src/quant.c:257-270
template <> __device__ __forceinline__ void decode8<LMC_TYPE_Q4_1>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b), m = f16at(b + 2);
    const int sh = j >= 16 ? 4 : 0, o = j & 15;
#pragma unroll
    for (int i = 0; i < 8; i++) y[i] = __fadd_rn(__fmul_rn(d, (float)((ldb(b + 4 + o + i) >> sh) & 0x0F)), m);
}
// src/quant.c:308-323: fifth bit of element e is bit e (e < 16) or bit e-4
// (e >= 16, quant.c:318) of qh; the 5-bit code is sign-extended.
template <> __device__ __forceinline__ void decode8<LMC_TYPE_Q5_0>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b);
    const uint32_t qh = ld32(b + 2);
    const int sh = j >= 16 ? 4 : 0, o = j & 15, hb = j >= 16 ? j - 4 : j;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int v = (int)((ldb(b + 6 + o + i) >> sh) & 0x0F) | (int)(((qh >> (hb + i)) & 1u) << 4);
        v = v >= 16 ? v - 32 : v;
        y[i] = __fmul_rn(d, (float)v);
    }
}
// src/quant.c:328-344
template <> __device__ __forceinline__ void decode8<LMC_TYPE_Q5_1>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b), m = f16at(b + 2);
    const uint32_t qh = ld32(b + 4);
    const int sh = j >= 16 ? 4 : 0, o = j & 15, hb = j >= 16 ? j - 4 : j;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int v = (int)((ldb(b + 8 + o + i) >> sh) & 0x0F) | (int)(((qh >> (hb + i)) & 1u) << 4);
        y[i] = __fadd_rn(__fmul_rn(d, (float)v), m);
    }
}
// src/quant.c:419-429
template <> __device__ __forceinline__ void decode8<LMC_TYPE_Q8_0>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b);
#pragma unroll
    for (int i = 0; i < 8; i++) y[i] = __fmul_rn((float)(int8_t)ldb(b + 2 + j + i), d);
}
// src/quant.c:178-205: element e = 128*half + 32*jj + 16*part + l.
template <> __device__ __forceinline__ void decode8<LMC_TYPE_Q2_K>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b + 80), dmin = f16at(b + 82);
    const int half = j >> 7, jj = (j >> 5) & 3, part = (j >> 4) & 1, l0 = j & 15;
    const int sc = ldb(b + 8 * half + 2 * jj + part);
    const float dl = __fmul_rn(d, (float)(sc & 0x0F)), ml = __fmul_rn(dmin, (float)(sc >> 4));
    const uint8_t *q = b + 16 + 32 * half + 16 * part + l0;
#pragma unroll
    for (int i = 0; i < 8; i++) y[i] = __fsub_rn(__fmul_rn(dl, (float)((ldb(q + i) >> (2 * jj)) & 3)), ml);
}
// src/quant.c:210-235: 4 elements per qs byte (e >> 2), hmask bit e >> 5 of
// byte e & 31, signed 6-bit scale of sub-block e >> 4 via kmask1/kmask2.
template <> __device__ __forceinline__ void decode8<LMC_TYPE_Q3_K>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b + 108);
    const int sub = j >> 4;
    // byte `sub` of aux[] (quant.c:223-227): aux word sub>>2 takes the low
    // (even word) or high (odd word) nibble of sc[4*(sub>>3) + (sub&3)] and
    // bits 2*(sub>>2)..+1 of sc[8 + (sub&3)].
    const uint32_t w = ldb(b + 96 + ((sub >> 3) << 2) + (sub & 3));
    const uint32_t lo = ((sub >> 2) & 1) ? (w >> 4) : (w & 0x0F);
    const uint32_t t = ldb(b + 96 + 8 + (sub & 3));
    const uint32_t hi = (t >> (2 * (sub >> 2))) & 3;
    const int scv = (int)(lo | (hi << 4)) - 32;
    const float ds = __fmul_rn(d, (float)scv);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int e = j + i;
        const int q2 = (ldb(b + 32 + (e >> 2)) >> (2 * (e & 3))) & 3;
        const int hb = (ldb(b + (e & 31)) >> (e >> 5)) & 1;
        y[i] = __fmul_rn(ds, (float)((q2 | (hb << 2)) - 4));
    }
}
// src/quant.c:275-303
template <> __device__ __forceinline__ void decode8<LMC_TYPE_Q4_K>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b), dmin = f16at(b + 2);
    const int g = j >> 6, hi = (j >> 5) & 1, l0 = j & 31;
    int sc, m;
    scale_min_k4(2 * g + hi, b + 4, sc, m);
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
    const uint8_t *q = b + 16 + 32 * g + l0;
#pragma unroll
    for (int i = 0; i < 8; i++) y[i] = __fsub_rn(__fmul_rn(d1, (float)((ldb(q + i) >> (4 * hi)) & 0x0F)), m1);
}
// src/quant.c:349-381
template <> __device__ __forceinline__ void decode8<LMC_TYPE_Q5_K>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b), dmin = f16at(b + 2);
    const int g = j >> 6, hi = (j >> 5) & 1, l0 = j & 31;
    int sc, m;
    scale_min_k4(2 * g + hi, b + 4, sc, m);
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
    const uint8_t *q = b + 48 + 32 * g + l0, *qh = b + 16 + l0;
    const int hs = 2 * g + hi;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int v = (int)((ldb(q + i) >> (4 * hi)) & 0x0F) | (int)(((ldb(qh + i) >> hs) & 1) << 4);
        y[i] = __fsub_rn(__fmul_rn(d1, (float)v), m1);
    }
}
// src/quant.c:386-414: element 128p + 32k + l, scale sc[8p + 2k + l/16],
// evaluated (d * sc) * q.
template <> __device__ __forceinline__ void decode8<LMC_TYPE_Q6_K>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b + 208);
    const int p = j >> 7, k = (j >> 5) & 3, l0 = j & 31;
    const float ds = __fmul_rn(d, (float)(int8_t)ldb(b + 192 + 8 * p + 2 * k + (l0 >> 4)));
    const uint8_t *ql = b + 64 * p + ((k & 1) ? 32 : 0) + l0, *qh = b + 128 + 32 * p + l0;
    const int lsh = (k >> 1) * 4, hsh = 2 * k;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int q = (int)(((ldb(ql + i) >> lsh) & 0x0F) | (((ldb(qh + i) >> hsh) & 3) << 4)) - 32;
        y[i] = __fmul_rn(ds, (float)q);
    }
}
// src/quant.c:435-458
template <> __device__ __forceinline__ void decode8<LMC_TYPE_IQ3_XXS>(const uint8_t *b, int j, float *y) {
    const float d = __fmul_rn(f16at(b), 0.5f);
    const int g = j >> 5, k = (j >> 3) & 3;
    const uint32_t gas = ld32(b + 66 + 4 * g);
    const float dl = __fmul_rn(d, (float)(2 * (int)(gas & 0xFF) + 1));
    const uint32_t signs = lmc_ksigns_iq2xs[(gas >> (8 + 7 * k)) & 0x7F];
    const uint32_t e0 = __ldg(&lmc_iq3xxs_grid[ldb(b + 2 + 8 * g + 2 * k)]);
    const uint32_t e1 = __ldg(&lmc_iq3xxs_grid[ldb(b + 2 + 8 * g + 2 * k + 1)]);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t ent = i < 4 ? e0 : e1;
        const float v = (float)(int8_t)((ent >> (8 * (i & 3))) & 0xFF);
        y[i] = __fmul_rn(dl, ((signs >> i) & 1) ? -v : v);
    }
}
// src/quant.c:464-487: one 9-bit grid index per 8 outputs, unsigned bytes.
template <> __device__ __forceinline__ void decode8<LMC_TYPE_IQ3_S>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b);
    const int g = j >> 5, i8 = j >> 3;
    const float dl = __fmul_rn(d, (float)(2 * ((ldb(b + 106 + (g >> 1)) >> (4 * (g & 1))) & 0x0F) + 1));
    const int hb = (ldb(b + 66 + (i8 >> 3)) >> (i8 & 7)) & 1;
    const uint32_t ent = __ldg(&lmc_iq3s_grid[ldb(b + 2 + i8) | (hb << 8)]);
    const uint32_t sg = ldb(b + 74 + i8);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float v = (float)((ent >> (8 * (i & 3))) & 0xFF);
        y[i] = __fmul_rn(dl, ((sg >> i) & 1) ? -v : v);
    }
}
// src/quant.c:499-521 (codes at byte 10: the block's last two code bytes are
// the next block's first two bytes).
template <> __device__ __forceinline__ void decode8<LMC_TYPE_IQ4_XS>(const uint8_t *b, int j, float *y) {
    const float d = f16at(b);
    const int g = j >> 5, i0 = j & 31;
    const uint32_t sh = ld32(b + 2);
    const uint32_t sl = ldb(b + 6 + (g >> 1));
    int sc = (int)(((g & 1) ? (sl >> 4) : (sl & 0x0F)) | (((sh >> (2 * g)) & 3) << 4));
    sc = (sc - 32) * 2 + 1;
    const float dl = __fmul_rn(d, (float)sc);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t byte = ldb(b + 10 + 16 * g + ((i0 + i) >> 1));
        const int n = ((i0 + i) & 1) ? (byte >> 4) : (byte & 0x0F);
        y[i] = __fmul_rn(dl, (float)lmc_iq4nl_table[n]);
    }
}
// F32 / F16 tensors (src/gguf.c:317-327), addressed as 8-element groups.
template <> __device__ __forceinline__ void decode8<LMC_TYPE_F32>(const uint8_t *b, int j, float *y) {
    const float4 *p = reinterpret_cast<const float4 *>(b);
    const float4 a = __ldg(p), c = __ldg(p + 1);
    y[0] = a.x; y[1] = a.y; y[2] = a.z; y[3] = a.w; y[4] = c.x; y[5] = c.y; y[6] = c.z; y[7] = c.w;
}
template <> __device__ __forceinline__ void decode8<LMC_TYPE_F16>(const uint8_t *b, int j, float *y) {
#pragma unroll
    for (int i = 0; i < 8; i++) y[i] = h2f(ld16(b + 2 * i));
}

}  // namespace lmcq

// Expands MACRO(T) for every supported type.
#define LMC_FOR_EACH_TYPE(MACRO)                                                   \
    MACRO(LMC_TYPE_F32) MACRO(LMC_TYPE_F16) MACRO(LMC_TYPE_Q4_0) MACRO(LMC_TYPE_Q4_1) \
    MACRO(LMC_TYPE_Q5_0) MACRO(LMC_TYPE_Q5_1) MACRO(LMC_TYPE_Q8_0) MACRO(LMC_TYPE_Q2_K) \
    MACRO(LMC_TYPE_Q3_K) MACRO(LMC_TYPE_Q4_K) MACRO(LMC_TYPE_Q5_K) MACRO(LMC_TYPE_Q6_K) \
    MACRO(LMC_TYPE_IQ3_XXS) MACRO(LMC_TYPE_IQ3_S) MACRO(LMC_TYPE_IQ4_XS)
