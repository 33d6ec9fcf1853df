/* lmc_ops.c - the C99 drop-in layer (include/lmc_ops.h): LMc's load_model,
 * model_forward and ops.h kernels on the B200.
 *
 * Compiled against LMc's own headers (utils.h, models.h, ops.h, gguf.h) in
 * place of LMc's gguf.c, ops.c and ops_llama.c, and linked with LMc's
 * utils.c and models.c (the arena, g_cfg / g_weights / g_kv_cache / g_act
 * and their init functions) and liblmc_b200.so.  Every op runs on the device;
 * a failing call ends the process through LMC_FATAL as LMc's errors do.
 */
#include <limits.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "gguf.h"
#include "llama_tok.h"
#include "models.h"
#include "ops.h"
#include "utils.h"

#include "lmc_cuda.h"
#include "lmc_ops.h"

#define CHECK(expr)                                                                   \
    do {                                                                              \
        if ((expr) != LMC_OK) LMC_FATAL("%s: %s", #expr, lmc_last_error());          \
    } while (0)

static lmc_model *g_dev;

lmc_model *lmcdrop_model(void) { return g_dev; }

/* ---- registry: host address -> device object ------------------------------ */
typedef struct {
    const void *host;
    const lmc_qtensor *q; /* matrix */
    const float *d;       /* vector */
    int n;
    int owned; /* uploaded here (a caller's unregistered fp32 matrix) */
} Reg;
static Reg *g_reg;
static int g_nreg, g_capreg;

static Reg *reg_find(const void *host) {
    for (int i = g_nreg - 1; i >= 0; i--)
        if (g_reg[i].host == host) return &g_reg[i];
    return NULL;
}
static Reg *reg_add(const void *host) {
    Reg *r = reg_find(host);
    if (r) return r;
    if (g_nreg == g_capreg) {
        g_capreg = g_capreg ? 2 * g_capreg : 256;
        g_reg = (Reg *)realloc(g_reg, sizeof(Reg) * (size_t)g_capreg);
        if (!g_reg) LMC_FATAL("drop-in: out of host memory");
    }
    r = &g_reg[g_nreg++];
    memset(r, 0, sizeof *r);
    r->host = host;
    return r;
}
void lmcdrop_register_matrix(const float *host, const lmc_qtensor *t) { reg_add(host)->q = t; }
void lmcdrop_register_vector(const float *host, const float *d_vec, int n) {
    Reg *r = reg_add(host);
    r->d = d_vec;
    r->n = n;
}
const lmc_qtensor *lmcdrop_lookup_matrix(const float *host) {
    const Reg *r = reg_find(host);
    return r ? r->q : NULL;
}

/* ---- device scratch ---------------------------------------------------------- */
enum { S_X, S_Y, S_Z, S_W, S_B, S_POS, S_COS, S_SIN, S_WS, S_N };
static void *g_s[S_N];
static size_t g_sz[S_N];
static void *scratch(int i, size_t bytes) {
    if (bytes > g_sz[i]) {
        if (g_s[i]) CHECK(lmc_buffer_free(g_s[i]));
        g_s[i] = NULL;
        CHECK(lmc_buffer_alloc(bytes, &g_s[i]));
        g_sz[i] = bytes;
    }
    return g_s[i];
}
static void h2d(void *d, const void *h, size_t n) { CHECK(lmc_copy(d, h, n, LMC_H2D, NULL)); }
static void d2h(void *h, const void *d, size_t n) { CHECK(lmc_copy(h, d, n, LMC_D2H, NULL)); }
static void sync0(void) { CHECK(lmc_stream_sync(NULL)); }

/* A host fp32 vector on the device: its registered copy, else uploaded into
 * scratch slot `slot` (caller data that may change between calls). */
static const float *dvec(const float *h, int n, int slot) {
    if (!h) return NULL;
    const Reg *r = reg_find(h);
    if (r && r->d && r->n >= n) return r->d;
    float *d = (float *)scratch(slot, sizeof(float) * (size_t)n);
    h2d(d, h, sizeof(float) * (size_t)n);
    return d;
}

/* The device tensor for a weight pointer LMc passes: the registered one, or
 * the caller's fp32 matrix uploaded once (cached by address). */
static const lmc_qtensor *dmat(const float *w, int M, int K) {
    Reg *r = reg_find(w);
    if (!r || !r->q) {
        lmc_qtensor *t = NULL;
        CHECK(lmc_qtensor_upload(LMC_TYPE_F32, M, K, w, sizeof(float) * (size_t)M * K, &t));
        r = reg_add(w);
        r->q = t;
        r->owned = 1;
    }
    int rows = 0, cols = 0;
    CHECK(lmc_qtensor_shape(r->q, NULL, &rows, &cols));
    if (rows != M || cols != K) LMC_FATAL("drop-in matmul_vec: weight is %dx%d, called as %dx%d", rows, cols, M, K);
    return r->q;
}

/* ---- the tokenizer vocabulary LMc's llama_tok.c reads --------------------------
 * LMc's loader fills g_llama_vocab from the GGUF arrays tokenizer.ggml.tokens
 * and tokenizer.ggml.scores while it parses the header (src/gguf.c:181-205),
 * when the vocabulary fits LLAMA_TOK_MAX_VOCAB.  The device loader does not
 * keep strings, so this reads the two arrays again from the file header. */
typedef struct {
    FILE *f;
    int v1; /* GGUF v1: 32-bit lengths and counts */
    int bad;
} Hdr;
static uint64_t rd(Hdr *h, int bytes) {
    uint64_t v = 0;
    if (fread(&v, 1, (size_t)bytes, h->f) != (size_t)bytes) h->bad = 1;
    return v;
}
static uint64_t rd_len(Hdr *h) { return rd(h, h->v1 ? 4 : 8); }
/* Forward only: a length from the file beyond what a long holds would turn
 * into a backward seek (and the header would be read again, without end). */
static void skip_bytes(Hdr *h, uint64_t n) {
    if (n > (uint64_t)LONG_MAX || fseek(h->f, (long)n, SEEK_CUR)) h->bad = 1;
}
/* Arrays of arrays deeper than any real file are refused instead of
 * recursing without bound. */
#define GGUF_MAX_NESTING 16
static void skip_value_at(Hdr *h, uint32_t type, int depth) {
    static const int size[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (type == 8) {
        skip_bytes(h, rd_len(h));
    } else if (type == 9) {
        if (depth >= GGUF_MAX_NESTING) {
            h->bad = 1;
            return;
        }
        const uint32_t et = (uint32_t)rd(h, 4);
        const uint64_t n = rd_len(h);
        for (uint64_t i = 0; i < n && !h->bad; i++) skip_value_at(h, et, depth + 1);
    } else if (type < 13) {
        skip_bytes(h, (uint64_t)size[type]);
    } else {
        h->bad = 1;
    }
}
static void skip_value(Hdr *h, uint32_t type) { skip_value_at(h, type, 0); }
static void read_llama_vocab(const char *path) {
    Hdr h = {fopen(path, "rb"), 0, 0};
    if (!h.f) return;
    const uint32_t magic = (uint32_t)rd(&h, 4), version = (uint32_t)rd(&h, 4);
    h.v1 = version == 1;
    (void)rd_len(&h); /* tensor count */
    const uint64_t n_kv = rd_len(&h);
    if (magic != 0x46554747u || h.bad) { fclose(h.f); return; }
    for (uint64_t i = 0; i < n_kv && !h.bad; i++) {
        char key[128] = {0};
        const uint64_t kl = rd_len(&h);
        if (kl < sizeof key) { if (fread(key, 1, (size_t)kl, h.f) != (size_t)kl) h.bad = 1; }
        else skip_bytes(&h, kl);
        const uint32_t type = (uint32_t)rd(&h, 4);
        if (type != 9) { skip_value(&h, type); continue; }
        const uint32_t et = (uint32_t)rd(&h, 4);
        const uint64_t n = rd_len(&h);
        if (!strcmp(key, "tokenizer.ggml.tokens") && et == 8 && n <= LLAMA_TOK_MAX_VOCAB) {
            g_llama_vocab_n = (int)n;
            for (uint64_t j = 0; j < n && !h.bad; j++) {
                const uint64_t sl = rd_len(&h);
                char *t = g_llama_vocab[j].text;
                const uint64_t keep = sl < LLAMA_TOK_MAX_PIECE - 1 ? sl : LLAMA_TOK_MAX_PIECE - 1;
                if (fread(t, 1, (size_t)keep, h.f) != (size_t)keep) h.bad = 1;
                t[keep] = '\0';
                skip_bytes(&h, sl - keep);
            }
        } else if (!strcmp(key, "tokenizer.ggml.scores") && et == 6) {
            for (uint64_t j = 0; j < n && !h.bad; j++) {
                float sc;
                uint32_t bits = (uint32_t)rd(&h, 4);
                memcpy(&sc, &bits, 4);
                if (g_llama_vocab_n > 0 && j < (uint64_t)g_llama_vocab_n) g_llama_vocab[j].score = sc;
            }
        } else {
            for (uint64_t j = 0; j < n && !h.bad; j++) skip_value(&h, et);
        }
    }
    fclose(h.f);
}

/* gguf.h's detect_format (src/gguf.c:394-403), kept alike because callers
 * branch on it: a name ending in .gguf or .bin decides; otherwise the first
 * four bytes of the file, GGUF's magic or that of LMc's .bin format; a file
 * that cannot be read is FORMAT_UNKNOWN.  (This layer's load_model reads
 * GGUF only; the .bin loader is not part of the device path.) */
ModelFormat detect_format(const char *path) {
    const size_t n = strlen(path);
    if (n >= 5 && !strcmp(path + n - 5, ".gguf")) return FORMAT_GGUF;
    if (n >= 4 && !strcmp(path + n - 4, ".bin")) return FORMAT_BIN;
    FILE *f = fopen(path, "rb");
    if (!f) return FORMAT_UNKNOWN;
    uint32_t magic = 0;
    if (fread(&magic, sizeof magic, 1, f) != 1) magic = 0;
    fclose(f);
    return magic == GGUF_MAGIC ? FORMAT_GGUF : magic == MODEL_MAGIC ? FORMAT_BIN : FORMAT_UNKNOWN;
}

/* LMc's CLI falls back to a model file at a default location when --model is
 * not given (src/gguf.c:414-420): the first of these that opens. */
const char *find_default_model(void) {
    static const char *const names[] = {"model.gguf", "models/model.gguf", "models/gpt2.gguf",
                                        "models/gpt2-small.gguf", "models/tinyllama.gguf", NULL};
    for (int i = 0; names[i]; i++) {
        FILE *f = fopen(names[i], "rb");
        if (f) {
            fclose(f);
            return names[i];
        }
    }
    return NULL;
}

/* ---- load_model (src/gguf.c:114-353) ---------------------------------------- */
static float *placeholder(const lmc_qtensor *t) {
    if (!t) return NULL;
    float *h = arena_alloc(4); /* a unique host address; no weights behind it */
    lmcdrop_register_matrix(h, t);
    return h;
}
static float *host_vector(int layer, int which) {
    int n = 0;
    const float *d = lmc_model_vector(g_dev, layer, which, &n);
    if (!d) return NULL;
    float *h = arena_alloc((size_t)n);
    d2h(h, d, sizeof(float) * (size_t)n);
    lmcdrop_register_vector(h, d, n);
    return h;
}

void load_model(const char *path) {
    CHECK(lmc_init(0));
    CHECK(lmc_model_load(path, 1, LMC_KV_F32, &g_dev));
    lmc_model_config c;
    CHECK(lmc_model_get_config(g_dev, &c));
    memset(&g_cfg, 0, sizeof g_cfg);
    g_cfg.arch = c.arch == 1 ? ARCH_GPT2 : ARCH_LLAMA;
    g_cfg.vocab_size = c.vocab_size;
    g_cfg.seq_len = c.seq_len;
    g_cfg.n_layers = c.n_layers;
    g_cfg.n_heads = c.n_heads;
    g_cfg.embed_dim = c.embed_dim;
    g_cfg.ffn_dim = c.ffn_dim;
    g_cfg.head_dim = c.head_dim;
    g_cfg.n_kv_heads = c.n_kv_heads;
    g_cfg.n_kv_groups = c.n_heads / c.n_kv_heads;
    g_cfg.rope_theta = c.rope_theta;
    g_cfg.norm_eps = c.norm_eps;
    g_cfg.rope_dim = c.head_dim;
    /* the arena holds the vector copies, the RoPE tables and the placeholders */
    const size_t D = (size_t)c.embed_dim, F = (size_t)c.ffn_dim, L = (size_t)c.n_layers;
    size_t floats = L * (8 * D + 3 * D + F + 64) + 4 * D + 64;
    if (g_cfg.arch == ARCH_GPT2) floats += (size_t)c.seq_len * D;
    else floats += (size_t)c.seq_len * (size_t)c.head_dim;
    arena_init(floats);
    memset(&g_weights, 0, sizeof g_weights);
    g_weights.layers = (LayerWeights *)calloc(L, sizeof(LayerWeights));
    if (!g_weights.layers) LMC_FATAL("drop-in: out of host memory");
    g_weights.wte = placeholder(lmc_model_matrix(g_dev, 0, LMC_W_TOKEN_EMBD));
    g_weights.lm_head = placeholder(lmc_model_matrix(g_dev, 0, LMC_W_OUTPUT));
    for (int l = 0; l < (int)L; l++) {
        LayerWeights *w = &g_weights.layers[l];
        w->attn_proj_weight = placeholder(lmc_model_matrix(g_dev, l, LMC_W_ATTN_OUT));
        if (g_cfg.arch == ARCH_GPT2) {
            w->ln1_weight = host_vector(l, LMC_V_ATTN_NORM);
            w->ln1_bias = host_vector(l, LMC_V_ATTN_NORM_B);
            w->ln2_weight = host_vector(l, LMC_V_FFN_NORM);
            w->ln2_bias = host_vector(l, LMC_V_FFN_NORM_B);
            w->qkv_weight = placeholder(lmc_model_matrix(g_dev, l, LMC_W_QKV));
            w->qkv_bias = host_vector(l, LMC_V_QKV_B);
            w->attn_proj_bias = host_vector(l, LMC_V_ATTN_OUT_B);
            w->ffn_fc_weight = placeholder(lmc_model_matrix(g_dev, l, LMC_W_FFN_UP));
            w->ffn_fc_bias = host_vector(l, LMC_V_FFN_UP_B);
            w->ffn_proj_weight = placeholder(lmc_model_matrix(g_dev, l, LMC_W_FFN_DOWN));
            w->ffn_proj_bias = host_vector(l, LMC_V_FFN_DOWN_B);
        } else {
            w->rms_attn_weight = host_vector(l, LMC_V_ATTN_NORM);
            w->rms_ffn_weight = host_vector(l, LMC_V_FFN_NORM);
            w->q_weight = placeholder(lmc_model_matrix(g_dev, l, LMC_W_Q));
            w->k_weight = placeholder(lmc_model_matrix(g_dev, l, LMC_W_K));
            w->v_weight = placeholder(lmc_model_matrix(g_dev, l, LMC_W_V));
            w->gate_weight = placeholder(lmc_model_matrix(g_dev, l, LMC_W_GATE));
            w->up_weight = placeholder(lmc_model_matrix(g_dev, l, LMC_W_FFN_UP));
            w->down_weight = placeholder(lmc_model_matrix(g_dev, l, LMC_W_FFN_DOWN));
        }
    }
    if (g_cfg.arch == ARCH_GPT2) {
        g_weights.wpe = host_vector(0, LMC_V_POS_EMBD);
        g_weights.ln_f_weight = host_vector(0, LMC_V_OUTPUT_NORM);
        g_weights.ln_f_bias = host_vector(0, LMC_V_OUTPUT_NORM_B);
    } else {
        g_weights.rms_f_weight = host_vector(0, LMC_V_OUTPUT_NORM);
        g_weights.rope_cos = host_vector(0, LMC_V_ROPE_COS);
        g_weights.rope_sin = host_vector(0, LMC_V_ROPE_SIN);
    }
    sync0();
    read_llama_vocab(path);
    LMC_INFO("Loaded on the B200 (GGUF blocks kept on the device): %s", path);
}

/* ---- model_forward (src/ops.c:212-237, src/ops_llama.c:157-192) ---------------- */
float *model_forward(int token_id, int pos) {
    if (!g_dev) LMC_FATAL("model_forward before load_model");
    int next = 0;
    CHECK(lmc_model_forward(g_dev, &token_id, &pos, 1, g_act.logits, &next));
    return g_act.logits;
}

/* ---- small ops ------------------------------------------------------------- */
static float scalar_op(float x, int silu_op) {
    float *d = (float *)scratch(S_Z, sizeof(float));
    h2d(d, &x, sizeof x);
    if (silu_op) CHECK(lmc_silu(d, 1, NULL));
    else CHECK(lmc_gelu(d, 1, NULL));
    d2h(&x, d, sizeof x);
    sync0();
    return x;
}
float gelu(float x) { return scalar_op(x, 0); }
float silu(float x) { return scalar_op(x, 1); }

void softmax(float *x, int n) {
    float *d = (float *)scratch(S_X, sizeof(float) * (size_t)n);
    h2d(d, x, sizeof(float) * (size_t)n);
    CHECK(lmc_softmax(d, n, 1, NULL));
    d2h(x, d, sizeof(float) * (size_t)n);
    sync0();
}

void layer_norm(float *restrict out, const float *restrict x, const float *restrict weight,
                const float *restrict bias, int dim) {
    float *dx = (float *)scratch(S_X, sizeof(float) * (size_t)dim);
    float *dy = (float *)scratch(S_Y, sizeof(float) * (size_t)dim);
    h2d(dx, x, sizeof(float) * (size_t)dim);
    CHECK(lmc_layer_norm(dy, dx, dvec(weight, dim, S_W), dvec(bias, dim, S_B), dim, 1, NULL));
    d2h(out, dy, sizeof(float) * (size_t)dim);
    sync0();
}

void rms_norm(float *restrict out, const float *restrict x, const float *restrict weight, int dim, float eps) {
    float *dx = (float *)scratch(S_X, sizeof(float) * (size_t)dim);
    float *dy = (float *)scratch(S_Y, sizeof(float) * (size_t)dim);
    h2d(dx, x, sizeof(float) * (size_t)dim);
    CHECK(lmc_rms_norm(dy, dx, dvec(weight, dim, S_W), dim, 1, eps, NULL));
    d2h(out, dy, sizeof(float) * (size_t)dim);
    sync0();
}

void matmul_vec(float *restrict out, const float *restrict weight, const float *restrict bias,
                const float *restrict in, int M, int K) {
    const lmc_qtensor *t = dmat(weight, M, K);
    float *dx = (float *)scratch(S_X, sizeof(float) * (size_t)K);
    float *dy = (float *)scratch(S_Y, sizeof(float) * (size_t)M);
    h2d(dx, in, sizeof(float) * (size_t)K);
    CHECK(lmc_matmul(t, dx, K, dvec(bias, M, S_B), dy, M, 1, LMC_EPI_NONE, NULL));
    d2h(out, dy, sizeof(float) * (size_t)M);
    sync0();
}

/* A RoPE row (Dh/2 floats) on the device: inside the registered table when
 * it comes from g_weights.rope_cos / rope_sin, else uploaded. */
static const float *drope_row(const float *row, int half, int slot) {
    for (int i = 0; i < g_nreg; i++) {
        const Reg *r = &g_reg[i];
        if (!r->d || !r->host) continue;
        const float *h = (const float *)r->host;
        if (row >= h && row + half <= h + r->n) return r->d + (row - h);
    }
    return dvec(row, half, slot);
}

void rope_apply(float *vec, const float *cos_row, const float *sin_row, int head_dim) {
    float *d = (float *)scratch(S_X, sizeof(float) * (size_t)head_dim);
    h2d(d, vec, sizeof(float) * (size_t)head_dim);
    CHECK(lmc_rope_apply(d, drope_row(cos_row, head_dim / 2, S_COS), drope_row(sin_row, head_dim / 2, S_SIN),
                         head_dim, 1, NULL));
    d2h(vec, d, sizeof(float) * (size_t)head_dim);
    sync0();
}

/* ---- attention over LMc's host KV cache ----------------------------------------- */
/* Device copy of a host cache [Hkv][S][Dh] of one layer (by address). */
static void *dcache(float *host, int Hkv) {
    Reg *r = reg_find(host);
    if (r && r->d) return (void *)r->d;
    const size_t n = (size_t)Hkv * CFG_S * CFG_Dh;
    void *d = NULL;
    CHECK(lmc_buffer_alloc(sizeof(float) * n, &d));
    h2d(d, host, sizeof(float) * n);
    r = reg_add(host);
    r->d = (const float *)d;
    r->n = (int)n;
    r->owned = 1;
    return d;
}

/* attention on the device: q [H Dh] (rotated), k/v new rows [Hkv Dh] (k
 * rotated), appended at pos to both the device and the host caches; out
 * [H Dh] on the device */
static void attend(float *d_out, const float *d_q, const float *d_k, const float *d_v, float *k_cache,
                   float *v_cache, int pos, int H, int Hkv) {
    const int Dh = CFG_Dh, S = CFG_S;
    void *dk = dcache(k_cache, Hkv), *dv = dcache(v_cache, Hkv);
    int *dp = (int *)scratch(S_POS, sizeof(int));
    h2d(dp, &pos, sizeof pos);
    const size_t wsb = lmc_attention_workspace_bytes(1, H, Dh, S);
    void *ws = wsb ? scratch(S_WS, wsb) : NULL;
    CHECK(lmc_attention_decode(d_out, d_q, d_k, d_v, dk, dv, LMC_KV_F32, dp, 1, H, Hkv, Dh, S, ws, wsb, NULL));
    for (int h = 0; h < Hkv; h++) { /* the host cache gets the same rows (src/ops.c:122-125) */
        const size_t off = ((size_t)h * S + pos) * Dh;
        d2h(k_cache + off, (const float *)dk + off, sizeof(float) * (size_t)Dh);
        d2h(v_cache + off, (const float *)dv + off, sizeof(float) * (size_t)Dh);
    }
}

void attention_forward(float *restrict out, const float *restrict x_norm, const LayerWeights *lw,
                       float *restrict k_cache, float *restrict v_cache, int pos, float *restrict qkv_buf,
                       float *restrict scores_buf) {
    (void)scores_buf;
    const int D = CFG_D, H = CFG_H;
    float *dx = (float *)scratch(S_X, sizeof(float) * (size_t)D);
    float *dqkv = (float *)scratch(S_Y, sizeof(float) * 3 * (size_t)D);
    float *dout = (float *)scratch(S_Z, sizeof(float) * (size_t)D);
    h2d(dx, x_norm, sizeof(float) * (size_t)D);
    CHECK(lmc_matmul(dmat(lw->qkv_weight, 3 * D, D), dx, D, dvec(lw->qkv_bias, 3 * D, S_B), dqkv, 3 * D, 1,
                     LMC_EPI_NONE, NULL));
    attend(dout, dqkv, dqkv + D, dqkv + 2 * D, k_cache, v_cache, pos, H, H);
    d2h(qkv_buf, dqkv, sizeof(float) * 3 * (size_t)D);
    d2h(out, dout, sizeof(float) * (size_t)D);
    sync0();
}

/* q, k, v projections and RoPE of one position on the device (src/ops_llama.c:66-78) */
static void llama_qkv(float *dq, float *dk, float *dv, const float *dx, const LayerWeights *lw, int pos) {
    const int D = CFG_D, H = CFG_H, Hkv = CFG_Hkv, Dh = CFG_Dh;
    CHECK(lmc_matmul(dmat(lw->q_weight, H * Dh, D), dx, D, NULL, dq, H * Dh, 1, LMC_EPI_NONE, NULL));
    CHECK(lmc_matmul(dmat(lw->k_weight, Hkv * Dh, D), dx, D, NULL, dk, Hkv * Dh, 1, LMC_EPI_NONE, NULL));
    CHECK(lmc_matmul(dmat(lw->v_weight, Hkv * Dh, D), dx, D, NULL, dv, Hkv * Dh, 1, LMC_EPI_NONE, NULL));
    const float *c = drope_row(g_weights.rope_cos + (size_t)pos * (Dh / 2), Dh / 2, S_COS);
    const float *s = drope_row(g_weights.rope_sin + (size_t)pos * (Dh / 2), Dh / 2, S_SIN);
    CHECK(lmc_rope_apply(dq, c, s, Dh, H, NULL));
    CHECK(lmc_rope_apply(dk, c, s, Dh, Hkv, NULL));
}

void llama_attention_forward(float *restrict out, const float *restrict x_norm, const LayerWeights *lw,
                             float *restrict k_cache, float *restrict v_cache, int pos, float *restrict q_buf,
                             float *restrict k_buf, float *restrict v_buf, float *restrict scores_buf) {
    (void)scores_buf;
    const int D = CFG_D, H = CFG_H, Hkv = CFG_Hkv, Dh = CFG_Dh;
    float *dx = (float *)scratch(S_X, sizeof(float) * (size_t)D);
    float *dqkv = (float *)scratch(S_Y, sizeof(float) * (size_t)(H + 2 * Hkv) * Dh);
    float *dout = (float *)scratch(S_Z, sizeof(float) * (size_t)H * Dh);
    float *dq = dqkv, *dk = dqkv + (size_t)H * Dh, *dv = dk + (size_t)Hkv * Dh;
    h2d(dx, x_norm, sizeof(float) * (size_t)D);
    llama_qkv(dq, dk, dv, dx, lw, pos);
    attend(dout, dq, dk, dv, k_cache, v_cache, pos, H, Hkv);
    d2h(q_buf, dq, sizeof(float) * (size_t)H * Dh);
    d2h(k_buf, dk, sizeof(float) * (size_t)Hkv * Dh);
    d2h(v_buf, dv, sizeof(float) * (size_t)Hkv * Dh);
    d2h(out, dout, sizeof(float) * (size_t)H * Dh);
    sync0();
}

void swiglu_ffn_forward(float *restrict out, const float *restrict x, const LayerWeights *lw,
                        float *restrict gate_buf, float *restrict up_buf) {
    const int D = CFG_D, F = CFG_F;
    float *dx = (float *)scratch(S_X, sizeof(float) * (size_t)D);
    float *dg = (float *)scratch(S_Y, sizeof(float) * 2 * (size_t)F);
    float *du = dg + F;
    float *dout = (float *)scratch(S_Z, sizeof(float) * (size_t)D);
    h2d(dx, x, sizeof(float) * (size_t)D);
    CHECK(lmc_matmul(dmat(lw->gate_weight, F, D), dx, D, NULL, dg, F, 1, LMC_EPI_NONE, NULL));
    CHECK(lmc_matmul(dmat(lw->up_weight, F, D), dx, D, NULL, du, F, 1, LMC_EPI_NONE, NULL));
    CHECK(lmc_swiglu(dg, du, (size_t)F, NULL));
    CHECK(lmc_matmul(dmat(lw->down_weight, D, F), dg, F, NULL, dout, D, 1, LMC_EPI_NONE, NULL));
    d2h(gate_buf, dg, sizeof(float) * (size_t)F); /* silu(gate) * up, as LMc leaves it */
    d2h(up_buf, du, sizeof(float) * (size_t)F);
    d2h(out, dout, sizeof(float) * (size_t)D);
    sync0();
}

/* One block with the residual stream kept on the device between its ops
 * (src/ops.c:182-206).  LMc's own version runs the GPT-2 block only (its
 * LLaMA block is inline in llama_model_forward); for a LLaMA model this one
 * runs that block (src/ops_llama.c:165-187). */
void transformer_block_forward(float *x, const LayerWeights *lw, float *k_cache, float *v_cache, int pos,
                               float *scratch_norm, float *scratch_qkv, float *scratch_attn, float *scratch_scores,
                               float *scratch_ffn, float *scratch_proj, float *scratch_ffnout) {
    (void)scratch_norm; (void)scratch_qkv; (void)scratch_attn; (void)scratch_scores;
    (void)scratch_ffn; (void)scratch_proj; (void)scratch_ffnout;
    const int D = CFG_D, F = CFG_F, H = CFG_H, Hkv = CFG_Hkv, Dh = CFG_Dh;
    const size_t QKV = (size_t)(H + 2 * Hkv) * Dh > 3 * (size_t)D ? (size_t)(H + 2 * Hkv) * Dh : 3 * (size_t)D;
    float *dx = (float *)scratch(S_X, sizeof(float) * (size_t)D);
    float *dn = (float *)scratch(S_W, sizeof(float) * (size_t)D);
    float *dqkv = (float *)scratch(S_Y, sizeof(float) * QKV);
    float *dh = (float *)scratch(S_Z, sizeof(float) * (2 * (size_t)F + (size_t)H * Dh));
    float *datt = dh + 2 * (size_t)F;
    h2d(dx, x, sizeof(float) * (size_t)D);
    if (g_cfg.arch == ARCH_GPT2) {
        CHECK(lmc_layer_norm(dn, dx, dvec(lw->ln1_weight, D, S_COS), dvec(lw->ln1_bias, D, S_SIN), D, 1, NULL));
        CHECK(lmc_matmul(dmat(lw->qkv_weight, 3 * D, D), dn, D, dvec(lw->qkv_bias, 3 * D, S_B), dqkv, 3 * D, 1,
                         LMC_EPI_NONE, NULL));
        attend(datt, dqkv, dqkv + D, dqkv + 2 * D, k_cache, v_cache, pos, H, H);
        CHECK(lmc_matmul(dmat(lw->attn_proj_weight, D, D), datt, D, dvec(lw->attn_proj_bias, D, S_B), dx, D, 1,
                         LMC_EPI_ACCUM, NULL));
        CHECK(lmc_layer_norm(dn, dx, dvec(lw->ln2_weight, D, S_COS), dvec(lw->ln2_bias, D, S_SIN), D, 1, NULL));
        CHECK(lmc_matmul(dmat(lw->ffn_fc_weight, F, D), dn, D, dvec(lw->ffn_fc_bias, F, S_B), dh, F, 1, LMC_EPI_GELU,
                         NULL));
        CHECK(lmc_matmul(dmat(lw->ffn_proj_weight, D, F), dh, F, dvec(lw->ffn_proj_bias, D, S_B), dx, D, 1,
                         LMC_EPI_ACCUM, NULL));
    } else {
        float *dq = dqkv, *dk = dqkv + (size_t)H * Dh, *dv = dk + (size_t)Hkv * Dh;
        CHECK(lmc_rms_norm(dn, dx, dvec(lw->rms_attn_weight, D, S_B), D, 1, CFG_EPS, NULL));
        llama_qkv(dq, dk, dv, dn, lw, pos);
        attend(datt, dq, dk, dv, k_cache, v_cache, pos, H, Hkv);
        CHECK(lmc_matmul(dmat(lw->attn_proj_weight, D, H * Dh), datt, H * Dh, NULL, dx, D, 1, LMC_EPI_ACCUM, NULL));
        CHECK(lmc_rms_norm(dn, dx, dvec(lw->rms_ffn_weight, D, S_B), D, 1, CFG_EPS, NULL));
        CHECK(lmc_matmul(dmat(lw->gate_weight, F, D), dn, D, NULL, dh, F, 1, LMC_EPI_NONE, NULL));
        CHECK(lmc_matmul(dmat(lw->up_weight, F, D), dn, D, NULL, dh + F, F, 1, LMC_EPI_NONE, NULL));
        CHECK(lmc_swiglu(dh, dh + F, (size_t)F, NULL));
        CHECK(lmc_matmul(dmat(lw->down_weight, D, F), dh, F, NULL, dx, D, 1, LMC_EPI_ACCUM, NULL));
    }
    d2h(x, dx, sizeof(float) * (size_t)D);
    sync0();
}
