/* lmc_oracle.c - CPU restatement of LMc's quantized-weight hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the oracle, never the product): see
 * lmc_oracle.h.  Compiled with -ffp-contract=off and without -ffast-math so
 * every float operation happens in the order written, which is the order LMc
 * writes them in quant.c.  Parity with LMc's own compiled sources is pinned
 * by tests/test_oracle.py and the fixtures in tests/golden/.
 */
#include "lmc_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../lmc_b200/csrc/lmc_codebooks.h"

/* ------------------------------------------------------------------------ */
/* Block geometry: LMc src/quant.h:54-99                                      */
/* ------------------------------------------------------------------------ */
int orc_block_geometry(uint32_t type, int *be, int *bb) {
    int e = 0, b = 0;
    switch (type) {
    case ORC_F32:     e = 1;   b = 4;   break;
    case ORC_F16:     e = 1;   b = 2;   break;
    case ORC_Q4_0:    e = 32;  b = 18;  break;
    case ORC_Q4_1:    e = 32;  b = 20;  break;
    case ORC_Q5_0:    e = 32;  b = 22;  break;
    case ORC_Q5_1:    e = 32;  b = 24;  break;
    case ORC_Q8_0:    e = 32;  b = 34;  break;
    case ORC_Q2_K:    e = 256; b = 84;  break;
    case ORC_Q3_K:    e = 256; b = 110; break;
    case ORC_Q4_K:    e = 256; b = 144; break;
    case ORC_Q5_K:    e = 256; b = 176; break;
    case ORC_Q6_K:    e = 256; b = 210; break;
    case ORC_IQ3_XXS: e = 256; b = 98;  break;
    case ORC_IQ3_S:   e = 256; b = 110; break;
    case ORC_IQ4_XS:  e = 256; b = 136; break;
    default: return -1;
    }
    if (be) *be = e;
    if (bb) *bb = b;
    return 0;
}

/* quant.c:19-38 - IEEE half to float by bit manipulation (subnormals are
 * renormalised, Inf/NaN keep their payload). */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t ex = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = 1;
            while (!(man & 0x400u)) { man <<= 1; e--; }
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(e + 112) << 23) | (man << 13);
        }
    } else if (ex == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((ex + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* IEEE binary16 rounding of a float (nearest, ties to even), back in fp32:
 * keep 11 significant bits at the half's precision (subnormal halves have a
 * fixed 2^-24 step), overflow to infinity. */
float orc_f32_to_f16_to_f32(float x) {
    if (x != x) return x;
    const float ax = fabsf(x);
    if (ax >= 65520.0f) return x < 0 ? -INFINITY : INFINITY; /* rounds past the largest half, 65504 */
    int e;
    frexpf(ax, &e);                              /* ax = f * 2^e, f in [0.5, 1) */
    const int step_e = e - 11 < -24 ? -24 : e - 11; /* ulp of the half holding ax */
    const float step = ldexpf(1.0f, step_e);
    const float r = rintf(ax / step) * step;     /* exact: division and product by a power of two */
    return x < 0 ? -r : r;
}

void orc_kv_q8_row(const float *x, int n, int8_t *q, float *scale) {
    float m = 0.0f;
    for (int i = 0; i < n; i++) m = fmaxf(m, fabsf(x[i]));
    if (m == 0.0f) {
        for (int i = 0; i < n; i++) q[i] = 0;
        *scale = 0.0f;
        return;
    }
    const float inv = 127.0f / m;
    for (int i = 0; i < n; i++) {
        float r = rintf(x[i] * inv);
        r = r > 127.0f ? 127.0f : r < -127.0f ? -127.0f : r;
        q[i] = (int8_t)r;
    }
    *scale = m / 127.0f;
}

void orc_kv_round_row(float *row, int n, int mode) {
    if (mode == 1) {
        for (int i = 0; i < n; i++) row[i] = orc_f32_to_f16_to_f32(row[i]);
    } else if (mode == 2) {
        int8_t q[1024];
        float sc;
        if (n > 1024) return;
        orc_kv_q8_row(row, n, q, &sc);
        for (int i = 0; i < n; i++) row[i] = (float)q[i] * sc;
    }
}

static float rd_f16(const uint8_t *p) { uint16_t h; memcpy(&h, p, 2); return orc_f16_to_f32(h); }
static uint32_t rd_u32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return v; }

/* quant.c:44-53 - (scale, min) pair j of the 12-byte 6-bit field. */
static void scale_min_k4(int j, const uint8_t *s, int *sc, int *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Per-element decoders.  Each writes the 32 or 256 outputs of one block and
 * names the LMc lines it restates. */

/* quant.c:240-252 */
static void blk_q4_0(const uint8_t *b, float *y) {
    float d = rd_f16(b);
    for (int j = 0; j < 16; j++) {
        y[j] = d * (float)((int)(b[2 + j] & 0x0F) - 8);
        y[j + 16] = d * (float)((int)(b[2 + j] >> 4) - 8);
    }
}
/* quant.c:257-270 */
static void blk_q4_1(const uint8_t *b, float *y) {
    float d = rd_f16(b), m = rd_f16(b + 2);
    for (int j = 0; j < 16; j++) {
        y[j] = d * (float)(b[4 + j] & 0x0F) + m;
        y[j + 16] = d * (float)(b[4 + j] >> 4) + m;
    }
}
/* quant.c:308-323.  The fifth bit of element j+16 is bit (j+12) of qh
 * (quant.c:318), and the 5-bit code is sign-extended (quant.c:319-320). */
static int sext5(int v) { return v >= 16 ? v - 32 : v; }
static void blk_q5_0(const uint8_t *b, float *y) {
    float d = rd_f16(b);
    uint32_t qh = rd_u32(b + 2);
    for (int j = 0; j < 16; j++) {
        int h0 = (qh >> j) & 1, h1 = (qh >> (j + 12)) & 1;
        y[j] = d * (float)sext5((b[6 + j] & 0x0F) | (h0 << 4));
        y[j + 16] = d * (float)sext5((b[6 + j] >> 4) | (h1 << 4));
    }
}
/* quant.c:328-344 (same qh bit choice as Q5_0, unsigned code). */
static void blk_q5_1(const uint8_t *b, float *y) {
    float d = rd_f16(b), m = rd_f16(b + 2);
    uint32_t qh = rd_u32(b + 4);
    for (int j = 0; j < 16; j++) {
        int h0 = (qh >> j) & 1, h1 = (qh >> (j + 12)) & 1;
        y[j] = d * (float)((b[8 + j] & 0x0F) | (h0 << 4)) + m;
        y[j + 16] = d * (float)((b[8 + j] >> 4) | (h1 << 4)) + m;
    }
}
/* quant.c:419-429 */
static void blk_q8_0(const uint8_t *b, float *y) {
    float d = rd_f16(b);
    for (int i = 0; i < 32; i++) y[i] = (float)(int8_t)b[2 + i] * d;
}
/* quant.c:178-205: element e = 128*half + 32*j + 16*part + l uses
 * qs[32*half + 16*part + l] >> 2j and scale byte 8*half + 2j + part. */
static void blk_q2_k(const uint8_t *b, float *y) {
    float d = rd_f16(b + 80), dmin = rd_f16(b + 82);
    for (int e = 0; e < 256; e++) {
        int half = e >> 7, j = (e >> 5) & 3, part = (e >> 4) & 1, l = e & 15;
        int sc = b[8 * half + 2 * j + part];
        float dl = d * (float)(sc & 0x0F), ml = dmin * (float)(sc >> 4);
        int q = (b[16 + 32 * half + 16 * part + l] >> (2 * j)) & 3;
        y[e] = dl * (float)q - ml;
    }
}
/* quant.c:210-235 (LMc's element order: 4 consecutive elements per qs
 * byte, hmask bit e>>5 of byte e&31; scales unpacked with kmask1/kmask2). */
static void blk_q3_k(const uint8_t *b, float *y) {
    const uint8_t *hm = b, *qs = b + 32, *s = b + 96;
    float d = rd_f16(b + 108);
    uint32_t tmp = rd_u32(s + 8), w0 = rd_u32(s), w1 = rd_u32(s + 4);
    uint32_t aux[4];
    aux[0] = (w0 & 0x0f0f0f0fu) | ((tmp & 0x03030303u) << 4);
    aux[1] = ((w0 >> 4) & 0x0f0f0f0fu) | (((tmp >> 2) & 0x03030303u) << 4);
    aux[2] = (w1 & 0x0f0f0f0fu) | (((tmp >> 4) & 0x03030303u) << 4);
    aux[3] = ((w1 >> 4) & 0x0f0f0f0fu) | (((tmp >> 6) & 0x03030303u) << 4);
    for (int e = 0; e < 256; e++) {
        int scv = (int)(int8_t)((aux[(e >> 4) >> 2] >> (8 * ((e >> 4) & 3))) & 0xFF) - 32;
        int q2 = (qs[e >> 2] >> (2 * (e & 3))) & 3;
        int hb = (hm[e & 31] >> (e >> 5)) & 1;
        y[e] = d * (float)scv * (float)((q2 | (hb << 2)) - 4);
    }
}
/* quant.c:275-303 */
static void blk_q4_k(const uint8_t *b, float *y) {
    float d = rd_f16(b), dmin = rd_f16(b + 2);
    const uint8_t *s = b + 4, *qs = b + 16;
    for (int g = 0; g < 4; g++) {
        int sc, m;
        scale_min_k4(2 * g, s, &sc, &m);
        float d1 = d * (float)sc, m1 = dmin * (float)m;
        scale_min_k4(2 * g + 1, s, &sc, &m);
        float d2 = d * (float)sc, m2 = dmin * (float)m;
        for (int l = 0; l < 32; l++) {
            y[64 * g + l] = d1 * (float)(qs[32 * g + l] & 0x0F) - m1;
            y[64 * g + 32 + l] = d2 * (float)(qs[32 * g + l] >> 4) - m2;
        }
    }
}
/* quant.c:349-381 */
static void blk_q5_k(const uint8_t *b, float *y) {
    float d = rd_f16(b), dmin = rd_f16(b + 2);
    const uint8_t *s = b + 4, *qh = b + 16, *qs = b + 48;
    for (int g = 0; g < 4; g++) {
        int sc, m;
        scale_min_k4(2 * g, s, &sc, &m);
        float d1 = d * (float)sc, m1 = dmin * (float)m;
        scale_min_k4(2 * g + 1, s, &sc, &m);
        float d2 = d * (float)sc, m2 = dmin * (float)m;
        for (int l = 0; l < 32; l++) {
            int lo = qs[32 * g + l] & 0x0F, hi = (qh[l] >> (2 * g)) & 1;
            y[64 * g + l] = d1 * (float)(lo | (hi << 4)) - m1;
            lo = qs[32 * g + l] >> 4;
            hi = (qh[l] >> (2 * g + 1)) & 1;
            y[64 * g + 32 + l] = d2 * (float)(lo | (hi << 4)) - m2;
        }
    }
}
/* quant.c:386-414: (d * sc) * q, evaluated left to right. */
static void blk_q6_k(const uint8_t *b, float *y) {
    float d = rd_f16(b + 208);
    for (int p = 0; p < 2; p++) {
        const uint8_t *ql = b + 64 * p, *qh = b + 128 + 32 * p;
        const int8_t *sc = (const int8_t *)(b + 192 + 8 * p);
        float *yp = y + 128 * p;
        for (int l = 0; l < 32; l++) {
            int is = l >> 4;
            int q1 = ((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
            int q2 = ((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
            int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            yp[l] = d * (float)sc[is] * (float)q1;
            yp[l + 32] = d * (float)sc[is + 2] * (float)q2;
            yp[l + 64] = d * (float)sc[is + 4] * (float)q3;
            yp[l + 96] = d * (float)sc[is + 6] * (float)q4;
        }
    }
}
/* quant.c:435-458: scale from the low byte of each u32, dl = d/2*(2s+1),
 * four 7-bit sign groups from bit 8, two grid entries per 8 outputs. */
static void blk_iq3_xxs(const uint8_t *b, float *y) {
    float d = rd_f16(b) * 0.5f;
    const uint8_t *qs = b + 2;
    for (int g = 0; g < 8; g++) {
        uint32_t gas = rd_u32(b + 66 + 4 * g);
        float dl = d * (float)(2 * (int)(gas & 0xFF) + 1);
        for (int k = 0; k < 4; k++) {
            int signs = lmc_ksigns_iq2xs[(gas >> (8 + 7 * k)) & 0x7F];
            for (int i = 0; i < 8; i++) {
                uint32_t ent = lmc_iq3xxs_grid[qs[8 * g + 2 * k + (i >> 2)]];
                float v = (float)(int8_t)((ent >> (8 * (i & 3))) & 0xFF);
                y[32 * g + 8 * k + i] = dl * (((signs >> i) & 1) ? -v : v);
            }
        }
    }
}
/* quant.c:464-487: one 9-bit grid index per 8 outputs, unsigned bytes. */
static void blk_iq3_s(const uint8_t *b, float *y) {
    float d = rd_f16(b);
    const uint8_t *qs = b + 2, *qh = b + 66, *sg = b + 74, *scl = b + 106;
    for (int g = 0; g < 8; g++) {
        float dl = d * (float)(2 * ((scl[g >> 1] >> (4 * (g & 1))) & 0x0F) + 1);
        for (int i = 0; i < 32; i++) {
            int i8 = 4 * g + (i >> 3);
            int hb = (qh[i8 >> 3] >> (i8 & 7)) & 1;
            uint32_t ent = lmc_iq3s_grid[qs[i8] | (hb << 8)];
            float v = (float)((ent >> (8 * (i & 3))) & 0xFF);
            int sgn = (sg[i8] >> (i & 7)) & 1;
            y[32 * g + i] = dl * (sgn ? -v : v);
        }
    }
}
/* quant.c:499-521: scales_h u32 @2, scales_l @6, codes @10 (the last two
 * code bytes are the next block's first two bytes). */
static void blk_iq4_xs(const uint8_t *b, float *y) {
    float d = rd_f16(b);
    uint32_t sh = rd_u32(b + 2);
    const uint8_t *sl = b + 6, *qs = b + 10;
    for (int g = 0; g < 8; g++) {
        int lo = (g & 1) ? (sl[g >> 1] >> 4) : (sl[g >> 1] & 0x0F);
        int sc = (lo | (((sh >> (2 * g)) & 3) << 4));
        sc = (sc - 32) * 2 + 1;
        float dl = d * (float)sc;
        for (int i = 0; i < 32; i++) {
            int byte = qs[16 * g + i / 2];
            int n = (i & 1) ? (byte >> 4) : (byte & 0x0F);
            y[32 * g + i] = dl * (float)lmc_iq4nl_table[n];
        }
    }
}

typedef void (*blk_fn)(const uint8_t *, float *);

static blk_fn blk_decoder(uint32_t type) {
    switch (type) {
    case ORC_Q4_0: return blk_q4_0;
    case ORC_Q4_1: return blk_q4_1;
    case ORC_Q5_0: return blk_q5_0;
    case ORC_Q5_1: return blk_q5_1;
    case ORC_Q8_0: return blk_q8_0;
    case ORC_Q2_K: return blk_q2_k;
    case ORC_Q3_K: return blk_q3_k;
    case ORC_Q4_K: return blk_q4_k;
    case ORC_Q5_K: return blk_q5_k;
    case ORC_Q6_K: return blk_q6_k;
    case ORC_IQ3_XXS: return blk_iq3_xxs;
    case ORC_IQ3_S: return blk_iq3_s;
    case ORC_IQ4_XS: return blk_iq4_xs;
    default: return NULL;
    }
}

/* quant.c dequant_* and the F32/F16 cases of gguf.c:317-327. */
int orc_dequant(uint32_t type, const uint8_t *src, float *dst, size_t n) {
    int be, bb;
    if (orc_block_geometry(type, &be, &bb)) return -1;
    if (n % (size_t)be) return -1;
    if (type == ORC_F32) { memcpy(dst, src, n * 4); return 0; }
    if (type == ORC_F16) {
        for (size_t i = 0; i < n; i++) dst[i] = rd_f16(src + 2 * i);
        return 0;
    }
    blk_fn f = blk_decoder(type);
    size_t nb = n / (size_t)be;
    for (size_t i = 0; i < nb; i++) f(src + i * (size_t)bb, dst + i * (size_t)be);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Ops                                                                        */
/* ------------------------------------------------------------------------ */
void orc_matmul_vec(float *out, const float *w, const float *bias,
                    const float *in, int M, int K) {
    for (int m = 0; m < M; m++) {
        const float *r = w + (size_t)m * K;
        double acc = bias ? (double)bias[m] : 0.0;
        for (int k = 0; k < K; k++) acc += (double)r[k] * (double)in[k];
        out[m] = (float)acc;
    }
}

float orc_gelu(float x) { return x * (1.0f / (1.0f + expf(-1.702f * x))); }
float orc_silu(float x) { return x * (1.0f / (1.0f + expf(-x))); }

void orc_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    if (sum < 1e-30f) {
        for (int i = 0; i < n; i++) x[i] = 1.0f / (float)n;
        return;
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

void orc_layer_norm(float *out, const float *x, const float *w, const float *b, int dim) {
    double mean = 0.0, var = 0.0;
    for (int i = 0; i < dim; i++) mean += x[i];
    mean /= dim;
    for (int i = 0; i < dim; i++) { double d = x[i] - mean; var += d * d; }
    float inv_std = (float)(1.0 / sqrt(var / dim + 1e-5));
    for (int i = 0; i < dim; i++) out[i] = (float)((x[i] - mean) * inv_std) * w[i] + b[i];
}

void orc_rms_norm(float *out, const float *x, const float *w, int dim, float eps) {
    double ss = 0.0;
    for (int i = 0; i < dim; i++) ss += (double)x[i] * x[i];
    float r = (float)(1.0 / sqrt(ss / dim + eps));
    for (int i = 0; i < dim; i++) out[i] = w[i] * r * x[i];
}

void orc_rope_apply(float *v, const float *c, const float *s, int Dh) {
    for (int d = 0; d < Dh / 2; d++) {
        float v0 = v[2 * d], v1 = v[2 * d + 1];
        v[2 * d] = v0 * c[d] - v1 * s[d];
        v[2 * d + 1] = v0 * s[d] + v1 * c[d];
    }
}

void orc_rope_cache(float *ct, float *st, int S, int Dh, float theta) {
    if (!(theta > 0.0f)) theta = 10000.0f;
    for (int p = 0; p < S; p++)
        for (int d = 0; d < Dh / 2; d++) {
            float a = (float)p / powf(theta, 2.0f * (float)d / (float)Dh);
            ct[(size_t)p * (Dh / 2) + d] = cosf(a);
            st[(size_t)p * (Dh / 2) + d] = sinf(a);
        }
}

void orc_attention(float *out, const float *q, const float *kc, const float *vc,
                   int H, int Hkv, int Dh, int S, int pos) {
    int G = H / Hkv, ctx = pos + 1;
    float scale = 1.0f / sqrtf((float)Dh);
    float *sc = (float *)malloc(sizeof(float) * (size_t)ctx);
    for (int h = 0; h < H; h++) {
        const float *kb = kc + (size_t)(h / G) * S * Dh;
        const float *vb = vc + (size_t)(h / G) * S * Dh;
        for (int t = 0; t < ctx; t++) {
            double dot = 0.0;
            for (int d = 0; d < Dh; d++) dot += (double)q[h * Dh + d] * kb[(size_t)t * Dh + d];
            sc[t] = (float)dot * scale;
        }
        orc_softmax(sc, ctx);
        for (int d = 0; d < Dh; d++) {
            double acc = 0.0;
            for (int t = 0; t < ctx; t++) acc += (double)sc[t] * vb[(size_t)t * Dh + d];
            out[h * Dh + d] = (float)acc;
        }
    }
    free(sc);
}

int orc_argmax(const float *x, int n) {
    int best = 0;
    for (int i = 1; i < n; i++) if (x[i] > x[best]) best = i;
    return best;
}

/* lmc.c:29-59: xorshift64 (shifts 13, 7, 17), a draw = top 53 bits / 2^53 in
 * float; greedy below temperature 1e-6; otherwise scale, softmax, sort
 * descending (qsort with the same comparison), nucleus = shortest prefix
 * whose running sum reaches top_p, renormalised walk until r < cdf. */
typedef struct { float prob; int idx; } OrcProbIdx;
static int orc_cmp_desc(const void *a, const void *b) {
    const OrcProbIdx *pa = (const OrcProbIdx *)a, *pb = (const OrcProbIdx *)b;
    return (pb->prob > pa->prob) ? 1 : (pb->prob < pa->prob) ? -1 : 0;
}
int orc_sample_top_p(float *logits, int V, float temperature, float top_p, uint64_t *rng, double *margin) {
    if (margin) *margin = 1.0;
    if (temperature < 1e-6f) return orc_argmax(logits, V);
    const float inv_temp = 1.0f / temperature;
    for (int i = 0; i < V; i++) logits[i] *= inv_temp;
    orc_softmax(logits, V);
    OrcProbIdx *srt = (OrcProbIdx *)malloc(sizeof(OrcProbIdx) * (size_t)V);
    if (!srt) return -1;
    for (int i = 0; i < V; i++) { srt[i].prob = logits[i]; srt[i].idx = i; }
    qsort(srt, (size_t)V, sizeof(OrcProbIdx), orc_cmp_desc);
    float cumsum = 0.0f;
    int nucleus = 0;
    for (int i = 0; i < V; i++) { cumsum += srt[i].prob; nucleus = i + 1; if (cumsum >= top_p) break; }
    float ns = 0.0f;
    for (int i = 0; i < nucleus; i++) ns += srt[i].prob;
    uint64_t st = *rng;
    st ^= st << 13; st ^= st >> 7; st ^= st << 17;
    *rng = st;
    const float inv_ns = 1.0f / ns, r = (float)(st >> 11) / (float)(1ULL << 53);
    float cdf = 0.0f;
    int pick = srt[nucleus - 1].idx;
    double m = 1.0;
    for (int i = 0; i < nucleus; i++) {
        cdf += srt[i].prob * inv_ns;
        const double d = fabs((double)cdf - (double)r);
        if (d < m) m = d;
        if (r < cdf) { pick = srt[i].idx; break; }
    }
    /* the nucleus boundary: how close the running sum came to top_p */
    double c2 = 0.0;
    for (int i = 0; i < nucleus; i++) c2 += srt[i].prob;
    if (fabs(c2 - top_p) < m) m = fabs(c2 - top_p);
    if (nucleus >= 1) {
        double c1 = c2 - srt[nucleus - 1].prob;
        if (fabs(c1 - top_p) < m) m = fabs(c1 - top_p);
    }
    if (margin) *margin = m;
    free(srt);
    return pick;
}

/* ------------------------------------------------------------------------ */
/* Whole model: GGUF parse (gguf.c:114-353) + forward (ops.c, ops_llama.c)    */
/* ------------------------------------------------------------------------ */
typedef struct {
    float *ln1_w, *ln1_b, *ln2_w, *ln2_b, *qkv_w, *qkv_b, *proj_w, *proj_b;
    float *fc_w, *fc_b, *fc2_w, *fc2_b;                       /* GPT-2 */
    float *rms_attn, *rms_ffn, *q_w, *k_w, *v_w, *o_w, *gate_w, *up_w, *down_w; /* LLaMA */
} OrcLayer;

struct OrcModel {
    int arch, V, S, L, H, Hkv, D, F, Dh, kv_mode;
    float theta, eps;
    float *wte, *wpe, *lnf_w, *lnf_b, *rmsf, *lm_head;
    float *rope_cos, *rope_sin;
    OrcLayer *layers;
    float *kc, *vc;
    float *x, *xn, *qkv, *q, *k, *v, *att, *proj, *h1, *h2, *ffo;
};

typedef struct { const uint8_t *p, *end; int err; } Rd;
static int rd_need(Rd *r, size_t n) { if ((size_t)(r->end - r->p) < n) { r->err = 1; return 0; } return 1; }
static uint32_t g_u32(Rd *r) { uint32_t v = 0; if (rd_need(r, 4)) { memcpy(&v, r->p, 4); r->p += 4; } return v; }
static uint64_t g_u64(Rd *r) { uint64_t v = 0; if (rd_need(r, 8)) { memcpy(&v, r->p, 8); r->p += 8; } return v; }
static float g_f32(Rd *r) { float v = 0; if (rd_need(r, 4)) { memcpy(&v, r->p, 4); r->p += 4; } return v; }
static const char *g_str(Rd *r, uint64_t *len) {
    *len = g_u64(r);
    if (!rd_need(r, *len)) return "";
    const char *s = (const char *)r->p; r->p += *len; return s;
}
static int streq(const char *s, uint64_t n, const char *lit) { return strlen(lit) == n && !memcmp(s, lit, n); }
static void skip_val(Rd *r, uint32_t t);
static void skip_val(Rd *r, uint32_t t) {
    static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (t == 8) { uint64_t n; g_str(r, &n); return; }
    if (t == 9) { uint32_t et = g_u32(r); uint64_t c = g_u64(r); for (uint64_t i = 0; i < c && !r->err; i++) skip_val(r, et); return; }
    if (t > 12) { r->err = 1; return; }
    if (rd_need(r, (size_t)sz[t])) r->p += sz[t];
}

static float **name_slot(OrcModel *m, const char *nm) {
    int ll = m->arch == 2;
    if (!strcmp(nm, "token_embd.weight")) return &m->wte;
    if (!strcmp(nm, "position_embd.weight")) return &m->wpe;
    if (!strcmp(nm, "output.weight")) return &m->lm_head;
    if (!strcmp(nm, "output_norm.weight")) return ll ? &m->rmsf : &m->lnf_w;
    if (!strcmp(nm, "output_norm.bias")) return &m->lnf_b;
    if (strncmp(nm, "blk.", 4)) return NULL;
    int l = atoi(nm + 4);
    if (l < 0 || l >= m->L) return NULL;
    const char *r = strchr(nm + 4, '.');
    if (!r) return NULL;
    r++;
    OrcLayer *w = &m->layers[l];
    if (!strcmp(r, "attn_norm.weight")) return ll ? &w->rms_attn : &w->ln1_w;
    if (!strcmp(r, "attn_norm.bias")) return &w->ln1_b;
    if (!strcmp(r, "attn_qkv.weight")) return &w->qkv_w;
    if (!strcmp(r, "attn_qkv.bias")) return &w->qkv_b;
    if (!strcmp(r, "attn_q.weight")) return &w->q_w;
    if (!strcmp(r, "attn_k.weight")) return &w->k_w;
    if (!strcmp(r, "attn_v.weight")) return &w->v_w;
    if (!strcmp(r, "attn_output.weight")) return ll ? &w->o_w : &w->proj_w;
    if (!strcmp(r, "attn_output.bias")) return &w->proj_b;
    if (!strcmp(r, "ffn_norm.weight")) return ll ? &w->rms_ffn : &w->ln2_w;
    if (!strcmp(r, "ffn_norm.bias")) return &w->ln2_b;
    if (!strcmp(r, "ffn_up.weight")) return ll ? &w->up_w : &w->fc_w;
    if (!strcmp(r, "ffn_up.bias")) return &w->fc_b;
    if (!strcmp(r, "ffn_down.weight")) return ll ? &w->down_w : &w->fc2_w;
    if (!strcmp(r, "ffn_down.bias")) return &w->fc2_b;
    if (!strcmp(r, "ffn_gate.weight")) return &w->gate_w;
    return NULL;
}

OrcModel *orc_model_load(const char *path) {
    FILE *f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    long fsz = ftell(f);
    fseek(f, 0, SEEK_SET);
    uint8_t *buf = (uint8_t *)malloc((size_t)fsz + 64);
    if (!buf || fread(buf, 1, (size_t)fsz, f) != (size_t)fsz) { fclose(f); free(buf); return NULL; }
    fclose(f);
    memset(buf + fsz, 0, 64);
    Rd r = {buf, buf + fsz, 0};
    OrcModel *m = (OrcModel *)calloc(1, sizeof(OrcModel));
    uint32_t magic = g_u32(&r), ver = g_u32(&r);
    if (magic != 0x46554747u || ver < 1 || ver > 3) goto fail;
    uint64_t nt = g_u64(&r), nkv = g_u64(&r);
    m->V = 128256; m->S = 8192; m->theta = 10000.0f; m->eps = 1e-5f;
    int vocab_key = 0, tok_count = 0;
    for (uint64_t i = 0; i < nkv && !r.err; i++) {
        uint64_t kl; const char *k = g_str(&r, &kl);
        uint32_t t = g_u32(&r);
        if (t == 4) {
            int v = (int)g_u32(&r);
            if (streq(k, kl, "gpt2.block_count") || streq(k, kl, "llama.block_count")) m->L = v;
            else if (streq(k, kl, "gpt2.attention.head_count") || streq(k, kl, "llama.attention.head_count")) m->H = v;
            else if (streq(k, kl, "gpt2.embedding_length") || streq(k, kl, "llama.embedding_length")) m->D = v;
            else if (streq(k, kl, "gpt2.feed_forward_length") || streq(k, kl, "llama.feed_forward_length")) m->F = v;
            else if (streq(k, kl, "gpt2.context_length") || streq(k, kl, "llama.context_length")) m->S = v;
            else if (streq(k, kl, "gpt2.vocab_size")) m->V = v;
            else if (streq(k, kl, "llama.vocab_size")) { m->V = v; vocab_key = v; }
            else if (streq(k, kl, "llama.attention.head_count_kv")) m->Hkv = v;
        } else if (t == 6) {
            float v = g_f32(&r);
            if (streq(k, kl, "llama.rope.freq_base")) m->theta = v;
            else if (streq(k, kl, "llama.attention.layer_norm_rms_epsilon")) m->eps = v;
        } else if (t == 8) {
            uint64_t vl; const char *v = g_str(&r, &vl);
            if (streq(k, kl, "general.architecture")) {
                if (streq(v, vl, "llama")) m->arch = 2;
                else if (streq(v, vl, "gpt2")) m->arch = 1;
            }
        } else if (t == 9 && streq(k, kl, "tokenizer.ggml.tokens")) {
            uint32_t et = g_u32(&r); uint64_t c = g_u64(&r);
            if (c <= 32768) tok_count = (int)c;
            for (uint64_t j = 0; j < c && !r.err; j++) skip_val(&r, et);
        } else {
            skip_val(&r, t);
        }
    }
    if (r.err) goto fail;
    /* gguf.c:218-244 */
    if (m->arch == 0) m->arch = m->Hkv > 0 ? 2 : 1;
    if (m->arch == 2 && m->Hkv == 0) m->Hkv = m->H;
    if (m->arch == 1) m->Hkv = m->H;
    if (m->arch == 1 && m->V == 128256) m->V = 50257;
    {
        int vn = tok_count ? tok_count : vocab_key;
        if (m->arch == 2 && vn > 0 && vn < m->V) m->V = vn;
    }
    if (!m->L || !m->H || !m->D) goto fail;
    if (!m->F) m->F = 4 * m->D;
    m->Dh = m->D / m->H;
    m->layers = (OrcLayer *)calloc((size_t)m->L, sizeof(OrcLayer));
    typedef struct { char name[256]; uint32_t type; uint64_t n, off; } TI;
    TI *ti = (TI *)calloc((size_t)nt, sizeof(TI));
    for (uint64_t i = 0; i < nt && !r.err; i++) {
        uint64_t nl; const char *nm = g_str(&r, &nl);
        if (nl > 255) nl = 255;
        memcpy(ti[i].name, nm, nl);
        uint32_t nd = g_u32(&r);
        ti[i].n = 1;
        for (uint32_t d = 0; d < nd; d++) ti[i].n *= g_u64(&r);
        ti[i].type = g_u32(&r);
        ti[i].off = g_u64(&r);
    }
    if (r.err) { free(ti); goto fail; }
    size_t data = (((size_t)(r.p - buf)) + 31) / 32 * 32;   /* gguf.c:285-287 */
    for (uint64_t i = 0; i < nt; i++) {
        float **slot = name_slot(m, ti[i].name);
        if (!slot) continue;
        int be, bb;
        if (orc_block_geometry(ti[i].type, &be, &bb) || ti[i].n % (uint64_t)be) { free(ti); goto fail; }
        size_t bytes = (size_t)(ti[i].n / (uint64_t)be) * (size_t)bb;
        if (data + ti[i].off + bytes > (size_t)fsz) { free(ti); goto fail; }
        free(*slot);
        *slot = (float *)malloc(sizeof(float) * (size_t)ti[i].n);
        orc_dequant(ti[i].type, buf + data + ti[i].off, *slot, (size_t)ti[i].n);
    }
    free(ti);
    free(buf);
    buf = NULL;
    if (m->arch == 2) {
        m->rope_cos = (float *)malloc(sizeof(float) * (size_t)m->S * (m->Dh / 2));
        m->rope_sin = (float *)malloc(sizeof(float) * (size_t)m->S * (m->Dh / 2));
        orc_rope_cache(m->rope_cos, m->rope_sin, m->S, m->Dh, m->theta);
    }
    {
        size_t kv = (size_t)m->L * m->Hkv * m->S * m->Dh;
        m->kc = (float *)calloc(kv, sizeof(float));
        m->vc = (float *)calloc(kv, sizeof(float));
        int D = m->D, F = m->F, H = m->H, Dh = m->Dh;
        m->x = calloc((size_t)D, 4); m->xn = calloc((size_t)D, 4); m->qkv = calloc((size_t)3 * D, 4);
        m->q = calloc((size_t)H * Dh, 4); m->k = calloc((size_t)m->Hkv * Dh, 4); m->v = calloc((size_t)m->Hkv * Dh, 4);
        m->att = calloc((size_t)D, 4); m->proj = calloc((size_t)D, 4);
        m->h1 = calloc((size_t)F, 4); m->h2 = calloc((size_t)F, 4); m->ffo = calloc((size_t)D, 4);
    }
    if (!m->lm_head) goto fail;   /* the synthetic files always carry output.weight */
    return m;
fail:
    free(buf);
    orc_model_free(m);
    return NULL;
}

void orc_model_free(OrcModel *m) {
    if (!m) return;
    if (m->layers) {
        for (int l = 0; l < m->L; l++) {
            float **p = (float **)&m->layers[l];
            for (size_t i = 0; i < sizeof(OrcLayer) / sizeof(float *); i++) free(p[i]);
        }
    }
    free(m->layers);
    free(m->wte); free(m->wpe); free(m->lnf_w); free(m->lnf_b); free(m->rmsf); free(m->lm_head);
    free(m->rope_cos); free(m->rope_sin); free(m->kc); free(m->vc);
    free(m->x); free(m->xn); free(m->qkv); free(m->q); free(m->k); free(m->v);
    free(m->att); free(m->proj); free(m->h1); free(m->h2); free(m->ffo);
    free(m);
}

void orc_model_set_kv(OrcModel *m, int mode) { m->kv_mode = mode; }

void orc_model_config(const OrcModel *m, int *c) {
    c[0] = m->arch; c[1] = m->V; c[2] = m->S; c[3] = m->L; c[4] = m->H; c[5] = m->Hkv;
    c[6] = m->D; c[7] = m->F; c[8] = m->Dh; c[9] = (int)(m->theta * 1000.0f); c[10] = (int)(m->eps * 1e9f);
}

int orc_model_forward(OrcModel *m, int tok, int pos, float *logits) {
    int D = m->D, F = m->F, H = m->H, Hkv = m->Hkv, Dh = m->Dh, S = m->S;
    if (tok < 0 || tok >= m->V || pos < 0 || pos >= S) return -1;
    if (m->arch == 1) {   /* ops.c:212-237 */
        for (int i = 0; i < D; i++) m->x[i] = m->wte[(size_t)tok * D + i] + m->wpe[(size_t)pos * D + i];
        for (int l = 0; l < m->L; l++) {
            OrcLayer *w = &m->layers[l];
            float *kc = m->kc + (size_t)l * H * S * Dh, *vc = m->vc + (size_t)l * H * S * Dh;
            orc_layer_norm(m->xn, m->x, w->ln1_w, w->ln1_b, D);
            orc_matmul_vec(m->qkv, w->qkv_w, w->qkv_b, m->xn, 3 * D, D);
            for (int h = 0; h < H; h++) {
                memcpy(kc + ((size_t)h * S + pos) * Dh, m->qkv + D + h * Dh, (size_t)Dh * 4);
                memcpy(vc + ((size_t)h * S + pos) * Dh, m->qkv + 2 * D + h * Dh, (size_t)Dh * 4);
                orc_kv_round_row(kc + ((size_t)h * S + pos) * Dh, Dh, m->kv_mode);
                orc_kv_round_row(vc + ((size_t)h * S + pos) * Dh, Dh, m->kv_mode);
            }
            orc_attention(m->att, m->qkv, kc, vc, H, H, Dh, S, pos);
            orc_matmul_vec(m->proj, w->proj_w, w->proj_b, m->att, D, D);
            for (int i = 0; i < D; i++) m->x[i] += m->proj[i];
            orc_layer_norm(m->xn, m->x, w->ln2_w, w->ln2_b, D);
            orc_matmul_vec(m->h1, w->fc_w, w->fc_b, m->xn, F, D);
            for (int i = 0; i < F; i++) m->h1[i] = orc_gelu(m->h1[i]);
            orc_matmul_vec(m->ffo, w->fc2_w, w->fc2_b, m->h1, D, F);
            for (int i = 0; i < D; i++) m->x[i] += m->ffo[i];
        }
        orc_layer_norm(m->xn, m->x, m->lnf_w, m->lnf_b, D);
    } else {              /* ops_llama.c:157-192 */
        memcpy(m->x, m->wte + (size_t)tok * D, (size_t)D * 4);
        const float *cr = m->rope_cos + (size_t)pos * (Dh / 2), *sr = m->rope_sin + (size_t)pos * (Dh / 2);
        for (int l = 0; l < m->L; l++) {
            OrcLayer *w = &m->layers[l];
            float *kc = m->kc + (size_t)l * Hkv * S * Dh, *vc = m->vc + (size_t)l * Hkv * S * Dh;
            orc_rms_norm(m->xn, m->x, w->rms_attn, D, m->eps);
            orc_matmul_vec(m->q, w->q_w, NULL, m->xn, H * Dh, D);
            orc_matmul_vec(m->k, w->k_w, NULL, m->xn, Hkv * Dh, D);
            orc_matmul_vec(m->v, w->v_w, NULL, m->xn, Hkv * Dh, D);
            for (int h = 0; h < H; h++) orc_rope_apply(m->q + h * Dh, cr, sr, Dh);
            for (int h = 0; h < Hkv; h++) orc_rope_apply(m->k + h * Dh, cr, sr, Dh);
            for (int h = 0; h < Hkv; h++) {
                memcpy(kc + ((size_t)h * S + pos) * Dh, m->k + h * Dh, (size_t)Dh * 4);
                memcpy(vc + ((size_t)h * S + pos) * Dh, m->v + h * Dh, (size_t)Dh * 4);
                orc_kv_round_row(kc + ((size_t)h * S + pos) * Dh, Dh, m->kv_mode);
                orc_kv_round_row(vc + ((size_t)h * S + pos) * Dh, Dh, m->kv_mode);
            }
            orc_attention(m->att, m->q, kc, vc, H, Hkv, Dh, S, pos);
            orc_matmul_vec(m->proj, w->o_w, NULL, m->att, D, D);
            for (int i = 0; i < D; i++) m->x[i] += m->proj[i];
            orc_rms_norm(m->xn, m->x, w->rms_ffn, D, m->eps);
            orc_matmul_vec(m->h1, w->gate_w, NULL, m->xn, F, D);
            orc_matmul_vec(m->h2, w->up_w, NULL, m->xn, F, D);
            for (int i = 0; i < F; i++) m->h1[i] = orc_silu(m->h1[i]) * m->h2[i];
            orc_matmul_vec(m->ffo, w->down_w, NULL, m->h1, D, F);
            for (int i = 0; i < D; i++) m->x[i] += m->ffo[i];
        }
        orc_rms_norm(m->xn, m->x, m->rmsf, D, m->eps);
    }
    orc_matmul_vec(logits, m->lm_head, NULL, m->xn, m->V, D);
    return 0;
}
