/* example_main.c - an LMc-side program written against LMc's headers only
 * (models.h, ops.h, gguf.h): the generate() loop of LMc's lmc.c
 * (src/lmc.c:86-133) without a tokenizer - token ids in, greedy ids out - and
 * a walk through the ops.h kernels on the loaded weights.
 *
 * The same source is linked two ways: with LMc's own gguf.c, ops.c and
 * ops_llama.c (the reference build of the test oracle), and with the drop-in
 * layer lmc_b200/dropin/lmc_ops.c, which runs every op on the B200.  Nothing
 * here changes between the two; the outputs are compared by the tests.
 *
 *   example_main MODEL.gguf gen N ID [ID ...]   prints "ids n id id ..."
 *   example_main MODEL.gguf ops                 prints "name n v v ..." lines
 *   example_main format PATH [PATH ...]         prints "format f PATH" per path
 *                                               (detect_format; no model)
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "gguf.h"
#include "models.h"
#include "ops.h"
#include "utils.h"

/* greedy pick as src/lmc.c:45-47: strict >, so the first maximum wins */
static int argmax_first(const float *x, int n) {
    int best = 0;
    for (int i = 1; i < n; i++)
        if (x[i] > x[best]) best = i;
    return best;
}

static void put(const char *name, const float *v, int n) {
    printf("%s %d", name, n);
    for (int i = 0; i < n; i++) printf(" %.9g", v[i]);
    printf("\n");
}

/* deterministic inputs (no RNG state shared with anything) */
static void fill(float *v, int n, float a, float b) {
    for (int i = 0; i < n; i++) v[i] = sinf(a * (float)i + b) * (1.0f + 0.25f * cosf(0.11f * (float)i));
}

static int gen(int n_new, const int *prompt, int n_prompt) {
    const float *lg = NULL;
    g_kv_cache.seq_len = 0;
    for (int i = 0; i < n_prompt; i++) {
        lg = model_forward(prompt[i], i);
        g_kv_cache.seq_len = i + 1;
    }
    int pos = n_prompt;
    printf("ids %d", n_new);
    for (int s = 0; s < n_new; s++) {
        const int nxt = argmax_first(lg, CFG_V);
        printf(" %d", nxt);
        if (s + 1 < n_new) {
            lg = model_forward(nxt, pos);
            g_kv_cache.seq_len = pos + 1;
            pos++;
        }
    }
    printf("\n");
    return 0;
}

static int ops(void) {
    const int D = CFG_D, F = CFG_F, H = CFG_H, Dh = CFG_Dh, S = CFG_S, V = CFG_V;
    const int Hkv = CFG_Hkv > 0 ? CFG_Hkv : H; /* as init_kv_cache (src/models.c:123) */
    const LayerWeights *lw = &g_weights.layers[0];
    const size_t cache = (size_t)Hkv * S * Dh;
    float *x = malloc(sizeof(float) * D), *xn = malloc(sizeof(float) * D), *y = malloc(sizeof(float) * 4 * D);
    float *h1 = malloc(sizeof(float) * F), *h2 = malloc(sizeof(float) * F), *lg = malloc(sizeof(float) * V);
    float *q = malloc(sizeof(float) * H * Dh), *k = malloc(sizeof(float) * Hkv * Dh);
    float *v = malloc(sizeof(float) * Hkv * Dh), *sc = malloc(sizeof(float) * H * S);
    float *qkv = malloc(sizeof(float) * 3 * D), *att = malloc(sizeof(float) * H * Dh);
    float *s1 = malloc(sizeof(float) * 4 * D), *s2 = malloc(sizeof(float) * 4 * D), *s3 = malloc(sizeof(float) * F);
    float *kc = calloc(cache, sizeof(float)), *vc = calloc(cache, sizeof(float));
    float *kc2 = calloc(cache, sizeof(float)), *vc2 = calloc(cache, sizeof(float));
    if (!x || !xn || !y || !h1 || !h2 || !lg || !q || !k || !v || !sc || !qkv || !att || !s1 || !s2 || !s3 || !kc ||
        !vc || !kc2 || !vc2)
        LMC_FATAL("out of memory");
    char name[64];

    fill(x, D, 0.37f, 0.1f);
    float sv[7] = {-9.0f, -1.5f, -0.25f, 0.0f, 0.3f, 2.0f, 11.0f}, g[7], si[7];
    for (int i = 0; i < 7; i++) { g[i] = gelu(sv[i]); si[i] = silu(sv[i]); }
    put("gelu", g, 7);
    put("silu", si, 7);
    memcpy(y, x, sizeof(float) * D);
    softmax(y, D);
    put("softmax", y, D);
    if (CFG_ARCH == ARCH_GPT2) {
        layer_norm(xn, x, lw->ln1_weight, lw->ln1_bias, D);
        put("layer_norm", xn, D);
        matmul_vec(y, lw->qkv_weight, lw->qkv_bias, xn, 3 * D, D);
        put("matmul_vec_qkv", y, 3 * D);
        for (int pos = 0; pos < 3; pos++) {
            fill(xn, D, 0.21f + 0.05f * pos, 0.3f);
            attention_forward(att, xn, lw, kc, vc, pos, qkv, sc);
            snprintf(name, sizeof name, "attention_forward_%d", pos);
            put(name, att, D);
        }
        put("k_cache_row2", kc + 2 * Dh, Dh);
        layer_norm(xn, x, g_weights.ln_f_weight, g_weights.ln_f_bias, D);
    } else {
        rms_norm(xn, x, lw->rms_attn_weight, D, CFG_EPS);
        put("rms_norm", xn, D);
        matmul_vec(q, lw->q_weight, NULL, xn, H * Dh, D);
        put("matmul_vec_q", q, H * Dh);
        rope_apply(q, g_weights.rope_cos + 3 * (Dh / 2), g_weights.rope_sin + 3 * (Dh / 2), Dh);
        put("rope_apply", q, Dh);
        for (int pos = 0; pos < 3; pos++) {
            fill(xn, D, 0.21f + 0.05f * pos, 0.3f);
            llama_attention_forward(att, xn, lw, kc, vc, pos, q, k, v, sc);
            snprintf(name, sizeof name, "llama_attention_forward_%d", pos);
            put(name, att, H * Dh);
        }
        put("k_cache_row2", kc + 2 * Dh, Dh);
        fill(xn, D, 0.13f, 0.7f);
        swiglu_ffn_forward(y, xn, lw, h1, h2);
        put("swiglu_ffn_forward", y, D);
        rms_norm(xn, x, g_weights.rms_f_weight, D, CFG_EPS);
    }
    matmul_vec(lg, g_weights.lm_head, NULL, xn, V, D);
    put("matmul_vec_lm_head", lg, V);
    /* LMc's transformer_block_forward runs the GPT-2 block (src/ops.c:182-206);
     * its LLaMA block is inline in llama_model_forward */
    fill(x, D, 0.05f, 0.9f);
    for (int pos = 0; pos < 3 && CFG_ARCH == ARCH_GPT2; pos++) {
        transformer_block_forward(x, lw, kc2, vc2, pos, s1, s2, att, sc, s3, y, s1 + D);
        snprintf(name, sizeof name, "transformer_block_forward_%d", pos);
        put(name, x, D);
    }
    return 0;
}

int main(int argc, char **argv) {
    if (argc < 3) {
        fprintf(stderr, "usage: %s MODEL.gguf gen N ID... | ops, or %s format PATH...\n", argv[0], argv[0]);
        return 2;
    }
    if (!strcmp(argv[1], "format")) {
        for (int i = 2; i < argc; i++) printf("format %d %s\n", (int)detect_format(argv[i]), argv[i]);
        return 0;
    }
    load_model(argv[1]);
    init_kv_cache();
    init_activations();
    int rc;
    if (!strcmp(argv[2], "gen") && argc >= 5) {
        const int n_new = atoi(argv[3]), n_prompt = argc - 4;
        int *prompt = malloc(sizeof(int) * n_prompt);
        for (int i = 0; i < n_prompt; i++) prompt[i] = atoi(argv[4 + i]);
        rc = gen(n_new, prompt, n_prompt);
        free(prompt);
    } else if (!strcmp(argv[2], "ops")) {
        rc = ops();
    } else {
        fprintf(stderr, "unknown mode %s\n", argv[2]);
        rc = 2;
    }
    fflush(stdout);
    return rc;
}
