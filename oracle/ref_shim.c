/* ref_shim.c - ctypes-friendly entry points around LMc's own compiled
 * sources (nile-agi/LMc src/*.c, built from where they lie by
 * oracle/Makefile into oracle/_ref/).  TEST INFRASTRUCTURE ONLY: a
 * parity reference and the CPU baseline, never the product.
 *
 * LMc's lmc.c (CLI, tokenizer, sampling) is not linked; this file takes its
 * place as the driver.  Greedy selection restates lmc.c:45-47 (strict '>'),
 * and timing uses CLOCK_MONOTONIC wall time, not lmc.c's clock() CPU time.
 */
#define _POSIX_C_SOURCE 200809L
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <time.h>
#include <unistd.h>
#include <fcntl.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#include "models.h"
#include "ops.h"
#include "gguf.h"
#include "quant.h"

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

double refshim_now(void) { return now_s(); }

void refshim_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int refshim_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Dispatch to LMc's dequant_* (quant.c:178-521) and the F32/F16 cases of
 * the loader (gguf.c:317-327). */
int refshim_dequant(uint32_t type, const uint8_t *src, float *dst, size_t n) {
    switch (type) {
    case GGUF_TYPE_F32: memcpy(dst, src, n * 4); return 0;
    case GGUF_TYPE_F16:
        for (size_t i = 0; i < n; i++) { uint16_t h; memcpy(&h, src + 2 * i, 2); dst[i] = f16_to_f32(h); }
        return 0;
    case GGUF_TYPE_Q4_0: dequant_q4_0(src, dst, n); return 0;
    case GGUF_TYPE_Q4_1: dequant_q4_1(src, dst, n); return 0;
    case GGUF_TYPE_Q5_0: dequant_q5_0(src, dst, n); return 0;
    case GGUF_TYPE_Q5_1: dequant_q5_1(src, dst, n); return 0;
    case GGUF_TYPE_Q8_0: dequant_q8_0(src, dst, n); return 0;
    case GGUF_TYPE_Q2_K: dequant_q2k(src, dst, n); return 0;
    case GGUF_TYPE_Q3_K: dequant_q3k(src, dst, n); return 0;
    case GGUF_TYPE_Q4_K: dequant_q4k(src, dst, n); return 0;
    case GGUF_TYPE_Q5_K: dequant_q5k(src, dst, n); return 0;
    case GGUF_TYPE_Q6_K: dequant_q6k(src, dst, n); return 0;
    case GGUF_TYPE_IQ3_XXS: dequant_iq3xxs(src, dst, n); return 0;
    case GGUF_TYPE_IQ3_S: dequant_iq3s(src, dst, n); return 0;
    case GGUF_TYPE_IQ4_XS: dequant_iq4_xs(src, dst, n); return 0;
    default: return -1;
    }
}

/* load_model (gguf.c:422) + init_kv_cache + init_activations
 * (models.c:122-164), with LMc's [INFO] chatter on stdout silenced. */
/* LMc's own cleanup (lmc.c:320-324), so a process can load one model
 * after another without keeping the previous arena. */
static int g_loaded = 0;
void refshim_free(void) {
    if (!g_loaded) return;
    arena_free();
    free(g_weights.layers);
    g_weights.layers = NULL;
    free(g_kv_cache.k_cache);
    free(g_kv_cache.v_cache);
    g_kv_cache.k_cache = g_kv_cache.v_cache = NULL;
    free_activations();
    g_loaded = 0;
}

int refshim_load(const char *path) {
    refshim_free();
    fflush(stdout);
    int saved = dup(1), devnull = open("/dev/null", O_WRONLY);
    if (devnull >= 0) dup2(devnull, 1);
    load_model(path);
    init_kv_cache();
    init_activations();
    g_loaded = 1;
    fflush(stdout);
    if (saved >= 0) { dup2(saved, 1); close(saved); }
    if (devnull >= 0) close(devnull);
    return 0;
}

void refshim_config(int *c) {
    c[0] = g_cfg.arch; c[1] = g_cfg.vocab_size; c[2] = g_cfg.seq_len; c[3] = g_cfg.n_layers;
    c[4] = g_cfg.n_heads; c[5] = g_cfg.n_kv_heads; c[6] = g_cfg.embed_dim; c[7] = g_cfg.ffn_dim;
    c[8] = g_cfg.head_dim;
}

/* model_forward (ops.c:212) with the logits copied out. */
int refshim_forward(int tok, int pos, float *logits_out) {
    const float *lg = model_forward(tok, pos);
    g_kv_cache.seq_len = pos + 1;
    if (logits_out) memcpy(logits_out, lg, sizeof(float) * (size_t)g_cfg.vocab_size);
    return 0;
}

static int argmax_first(const float *x, int n) {
    int best = 0;
    for (int i = 1; i < n; i++) if (x[i] > x[best]) best = i;
    return best;
}

/* The generate() loop of lmc.c:108-132 without tokenizer / EOS: feed the
 * prompt token by token, then n_new greedy steps.  out_ids gets the n_new
 * generated ids; times are wall seconds for the prefill and decode parts. */
int refshim_generate(const int *prompt, int n_prompt, int n_new, int *out_ids,
                     double *t_prefill, double *t_decode) {
    const float *lg = NULL;
    double t0 = now_s();
    for (int i = 0; i < n_prompt; i++) { lg = model_forward(prompt[i], i); g_kv_cache.seq_len = i + 1; }
    double t1 = now_s();
    int pos = n_prompt;
    for (int s = 0; s < n_new; s++) {
        if (pos >= g_cfg.seq_len) return -1;
        int nxt = argmax_first(lg, g_cfg.vocab_size);
        out_ids[s] = nxt;
        if (s + 1 < n_new) { lg = model_forward(nxt, pos); g_kv_cache.seq_len = pos + 1; pos++; }
    }
    double t2 = now_s();
    if (t_prefill) *t_prefill = t1 - t0;
    if (t_decode) *t_decode = t2 - t1;
    return 0;
}

/* matmul_vec (ops.c:69) called `reps` times; returns wall seconds. */
double refshim_time_matmul(float *out, const float *w, const float *bias, const float *in,
                           int M, int K, int reps) {
    double t0 = now_s();
    for (int r = 0; r < reps; r++) matmul_vec(out, w, bias, in, M, K);
    return now_s() - t0;
}

/* LMc's own sample_top_p and RNG (lmc.c:29-59) are file-static in lmc.c, so
 * lmc.c itself is compiled into this file, its main renamed out of the way.
 * refshim_sample_top_p seeds the RNG state directly and runs LMc's function
 * on a logits row (scaled and softmaxed in place, as LMc does); vocab_size
 * and the sort buffer are set for the call and restored after it. */
#define main lmc_cli_main_unused
#include "lmc.c"
#undef main

int refshim_sample_top_p(float *logits, int V, float temperature, float top_p, uint64_t *state) {
    const int saved_v = g_cfg.vocab_size;
    void *saved_buf = g_act.sorted_buf;
    void *buf = malloc((size_t)V * (sizeof(float) + sizeof(int)));
    if (!buf) return -1;
    g_cfg.vocab_size = V;
    g_act.sorted_buf = buf;
    g_rng_state = *state;
    const int tok = sample_top_p(logits, temperature, top_p);
    *state = g_rng_state;
    g_cfg.vocab_size = saved_v;
    g_act.sorted_buf = saved_buf;
    free(buf);
    return tok;
}
