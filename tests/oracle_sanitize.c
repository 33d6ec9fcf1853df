/* oracle_sanitize.c - drives every entry point of the C oracle
 * (oracle/lmc_oracle.c) once, for a build under AddressSanitizer and
 * UndefinedBehaviorSanitizer (tests/test_oracle_sanitize.py): buffers are
 * allocated to their exact sizes, so a read or write past any of them
 * stops the run.  The one over-read LMc itself makes (IQ4_XS reads two
 * bytes past its last block, src/quant.c:506,515) is given exactly those two
 * bytes.  argv: GGUF files to load and run a few positions of, in every
 * K/V row form, then files that must fail to load (truncated). */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../oracle/lmc_oracle.h"

static uint64_t rng = 0x9E3779B97F4A7C15ull;
static uint32_t next_u32(void) {
    rng ^= rng << 13;
    rng ^= rng >> 7;
    rng ^= rng << 17;
    return (uint32_t)(rng >> 16);
}
static float next_f(void) { return (float)((int)(next_u32() % 20001) - 10000) / 2500.0f; }
static float *farr(size_t n) {
    float *p = (float *)malloc(n * sizeof(float));
    for (size_t i = 0; i < n; i++) p[i] = next_f();
    return p;
}

#define CHECK(c)                                                         \
    do {                                                                 \
        if (!(c)) {                                                      \
            fprintf(stderr, "check failed: %s (line %d)\n", #c, __LINE__); \
            return 1;                                                    \
        }                                                                \
    } while (0)

static int dequant_all(void) {
    const uint32_t types[] = {ORC_F32, ORC_F16, ORC_Q4_0, ORC_Q4_1, ORC_Q5_0, ORC_Q5_1, ORC_Q8_0, ORC_Q2_K,
                              ORC_Q3_K, ORC_Q4_K, ORC_Q5_K, ORC_Q6_K, ORC_IQ3_XXS, ORC_IQ3_S, ORC_IQ4_XS};
    for (size_t i = 0; i < sizeof types / sizeof types[0]; i++) {
        int be = 0, bb = 0;
        CHECK(orc_block_geometry(types[i], &be, &bb) == 0);
        const size_t nb = 3, n = nb * (size_t)be, bytes = nb * (size_t)bb + (types[i] == ORC_IQ4_XS ? 2 : 0);
        uint8_t *src = (uint8_t *)malloc(bytes);
        for (size_t k = 0; k < bytes; k++) src[k] = (uint8_t)next_u32();
        if (types[i] == ORC_F32) /* finite floats only (the bytes are read as IEEE values) */
            for (size_t k = 0; k < n; k++) {
                const float f = next_f();
                memcpy(src + 4 * k, &f, 4);
            }
        float *dst = (float *)malloc(n * sizeof(float));
        CHECK(orc_dequant(types[i], src, dst, n) == 0);
        if (be > 1) CHECK(orc_dequant(types[i], src, dst, n + 1) != 0); /* not a whole block: refused */
        free(src);
        free(dst);
    }
    for (uint32_t h = 0; h < 65536; h++) (void)orc_f16_to_f32((uint16_t)h);
    return 0;
}

static int small_ops(void) {
    const int M = 37, K = 96;
    float *w = farr((size_t)M * K), *x = farr(K), *b = farr(M), *out = (float *)malloc(M * sizeof(float));
    orc_matmul_vec(out, w, b, x, M, K);
    orc_matmul_vec(out, w, NULL, x, M, K);
    for (int i = -40; i <= 40; i++) {
        (void)orc_gelu((float)i * 0.5f);
        (void)orc_silu((float)i * 0.5f);
    }
    float one[1] = {3.0f};
    orc_softmax(one, 1);
    CHECK(one[0] == 1.0f);
    float big[4] = {1e30f, -1e30f, 1e30f, 0.0f};
    orc_softmax(big, 4);
    float ninf[3] = {-INFINITY, -INFINITY, -INFINITY}; /* the sum < 1e-30 branch: uniform */
    orc_softmax(ninf, 3);
    float *ln = (float *)malloc(K * sizeof(float)), *lw = farr(K), *lb = farr(K);
    orc_layer_norm(ln, x, lw, lb, K);
    orc_rms_norm(ln, x, lw, K, 1e-5f);
    const int S = 16, Dh = 32, H = 4, Hkv = 2;
    float *cs = (float *)malloc(sizeof(float) * S * (Dh / 2)), *sn = (float *)malloc(sizeof(float) * S * (Dh / 2));
    orc_rope_cache(cs, sn, S, Dh, 10000.0f);
    float *q = farr((size_t)H * Dh);
    orc_rope_apply(q, cs + (S - 1) * (Dh / 2), sn + (S - 1) * (Dh / 2), Dh);
    float *kc = farr((size_t)Hkv * S * Dh), *vc = farr((size_t)Hkv * S * Dh), *ao = (float *)malloc(sizeof(float) * H * Dh);
    orc_attention(ao, q, kc, vc, H, Hkv, Dh, S, 0);
    orc_attention(ao, q, kc, vc, H, Hkv, Dh, S, S - 1);
    int8_t codes[64];
    float scale = 0.0f, zero[64] = {0};
    orc_kv_q8_row(x, 64, codes, &scale);
    orc_kv_q8_row(zero, 64, codes, &scale);
    CHECK(scale == 0.0f);
    for (int mode = 0; mode < 3; mode++) {
        float *row = farr(64);
        orc_kv_round_row(row, 64, mode);
        free(row);
    }
    (void)orc_f32_to_f16_to_f32(65519.0f);
    (void)orc_f32_to_f16_to_f32(1e-8f);
    CHECK(orc_argmax(x, K) >= 0);
    const int V = 300;
    const float temps[] = {0.7f, 1.0f, 1e-7f}, tops[] = {0.9f, 1.5f, 1e-6f};
    uint64_t st = 0x1234567ull;
    for (int t = 0; t < 3; t++)
        for (int p = 0; p < 3; p++) {
            float *lg = farr(V);
            double margin = 0.0;
            const int tok = orc_sample_top_p(lg, V, temps[t], tops[p], &st, &margin);
            CHECK(tok >= 0 && tok < V);
            free(lg);
        }
    free(w); free(x); free(b); free(out); free(ln); free(lw); free(lb); free(cs); free(sn); free(q);
    free(kc); free(vc); free(ao);
    return 0;
}

int main(int argc, char **argv) {
    if (dequant_all() || small_ops()) return 1;
    int i = 1;
    for (; i < argc && strcmp(argv[i], "--bad"); i++) {
        for (int mode = 0; mode < 3; mode++) {
            OrcModel *m = orc_model_load(argv[i]);
            CHECK(m != NULL);
            orc_model_set_kv(m, mode);
            int cfg[11];
            orc_model_config(m, cfg);
            float *lg = (float *)malloc(sizeof(float) * (size_t)cfg[1]);
            for (int pos = 0; pos < 5 && pos < cfg[2]; pos++)
                CHECK(orc_model_forward(m, (int)(next_u32() % (uint32_t)cfg[1]), pos, lg) == 0);
            free(lg);
            orc_model_free(m);
        }
    }
    for (i++; i < argc; i++) CHECK(orc_model_load(argv[i]) == NULL);
    puts("ok");
    return 0;
}
