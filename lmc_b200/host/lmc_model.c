/* lmc_model.c - C99 host runtime: GGUF load onto the device and the
 * decode-step driver (LMc load_model + model_forward + generate, on B200).
 *
 * LMc parses the GGUF header (src/gguf.c:114-282), dequantizes every tensor
 * into an fp32 arena (src/gguf.c:290-347) and runs model_forward on the CPU
 * (src/ops.c:212-237, src/ops_llama.c:157-192).  Here the same header rules
 * pick the configuration, the raw blocks go to the device as qtensors, and a
 * step is a fixed sequence of kernel launches on one stream that reads the
 * token and position of each sequence from device memory - so a step can be
 * captured once as a CUDA graph and replayed for every position, and greedy
 * generation runs without the host waiting between tokens.
 */
#define _DEFAULT_SOURCE
#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <nccl.h>

#include "../csrc/lmc_internal.h"

typedef struct {
    /* GPT-2 (src/models.h:79-117) */
    lmc_qtensor *qkv, *proj, *fc, *fc2;
    float *ln1_w, *ln1_b, *ln2_w, *ln2_b, *qkv_b, *proj_b, *fc_b, *fc2_b;
    /* LLaMA */
    lmc_qtensor *q, *k, *v, *o, *gate, *up, *down;
    float *rms_attn, *rms_ffn;
    /* q|k|v and gate|up concatenated by rows (same type and width), so each
     * pair of projections is one launch; NULL when they cannot be fused */
    lmc_qtensor *qkv_cat, *gateup_cat;
    /* gate and up with their 16-row tiles interleaved, built for the
     * persistent step (whose gate|up GEMV then finishes silu(gate) * up) */
    lmc_qtensor *gateup_il;
} Layer;

struct lmc_model {
    lmc_model_config cfg;
    int max_batch, kv_dtype;
    /* rows per step (>= max_batch): a prompt chunk of one sequence runs one
     * position per row (lmc_model_prefill); d_seq[row] = its cache sequence */
    int max_rows, prefill, prefill_head; /* prefill_head: this chunk is the prompt's last */
    int *d_seq;
    lmc_qtensor *wte, *lm_head;
    float *wpe, *lnf_w, *lnf_b, *rmsf, *rope_cos, *rope_sin;
    Layer *layers;
    void *kc, *vc;
    size_t kv_layer_bytes;
    /* paged KV cache (page_size 0: contiguous [seq][kv head][seq_len][row]).
     * Each layer's cache is a pool of n_pages pages [page][kv head][page_size]
     * [row]; position t of sequence s lives in page
     * d_pages[s * max_pages + t / page_size] (the same page id in every
     * layer's pool).  The host hands pages out before the step that first
     * writes them: h_pages mirrors the table (-1: none), seq_np[s] = pages
     * sequence s holds (always its first seq_np[s] table entries), free_ids
     * the n_free ids not held. */
    int page_size, page_shift, max_pages, n_pages, n_free;
    int *d_pages, *h_pages, *seq_np, *free_ids;
    int g_pos; /* next position of the last generation's step loop (lmc_model_replay) */
    float *x, *xn, *qkv, *att, *h, *h2, *logits;
    void *ws;
    size_t ws_bytes;
    int *d_tok, *d_pos, *d_next, *d_step, *d_prompt, *d_ids;
    unsigned long long *d_keys; /* per sequence greedy-pick key of the step */
    int *d_attn_cnt;            /* attention split arrival counters [batch][kv heads] */
    int *h_stage; /* pinned: tokens, positions, next ids */
    int *h_next_map; /* mapped pinned: the persistent forward step writes its picks here */
    /* tensor parallel: the residual sums over peer memory (peer_allreduce.cu);
     * peer_base[p] = rank p's region mapped here (CUDA IPC) */
    void *peer_base[LMC_PEER_MAX];
    int peer_on;
    int prompt_cap, ids_cap;
    cudaStream_t stream;
    cudaGraphExec_t gexec;
    int g_batch, g_nprompt, g_nnew; /* shape the captured graph was built for */
    int g_kernels;                  /* kernel nodes in the captured step graph */
    /* tensor-parallel shard (tp_size 1: the whole model on this GPU).  This
     * rank holds heads [rank hl, +hl) with their kv heads, ffn rows
     * [rank fl, +fl) of gate / up (columns of down), attn_output columns of
     * its heads, and lm_head rows [v0, v0 + vl). */
    int tp_rank, tp_size, hl, hkvl, fl, vl, v0;
    ncclComm_t comm;
    /* the step as one persistent launch (lmc_step_prog), built on first use:
     * per batch size for lmc_model_forward, and one for the generate loop
     * (with the arguments it was built for); no_persist: it cannot be built */
    lmc_step_prog *pfwd[3], *pgen;
    int no_persist[3], gen_persist_failed;
    int pg_batch, pg_nprompt, pg_nnew, pg_smp;
    float pg_t, pg_p;
    /* top-p sampling in the generate loop (lmc_model_generate_sample):
     * smp = 1 while such a loop runs; one xorshift64 state per sequence */
    int smp;
    float smp_t, smp_p;
    unsigned long long *d_rng;
    int g_smp;
    float g_t, g_p;
    const int *pg_prompt;
    const int *pg_ids;
};

#define TRY(expr)                     \
    do {                              \
        int _rc = (expr);             \
        if (_rc) return _rc;          \
    } while (0)
#define CUTRY(expr)                                                                              \
    do {                                                                                         \
        cudaError_t _e = (expr);                                                                 \
        if (_e != cudaSuccess)                                                                   \
            return lmc_set_error(LMC_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e));        \
    } while (0)

/* ------------------------------------------------------------------------ */
/* GGUF reading (layout per src/gguf.c:114-287)                               */
/* ------------------------------------------------------------------------ */
typedef struct { const unsigned char *p, *end; int err; } Rd;
static int need(Rd *r, size_t n) { if ((size_t)(r->end - r->p) < n) { r->err = 1; return 0; } return 1; }
static uint32_t u32(Rd *r) { uint32_t v = 0; if (need(r, 4)) { memcpy(&v, r->p, 4); r->p += 4; } return v; }
static uint64_t u64(Rd *r) { uint64_t v = 0; if (need(r, 8)) { memcpy(&v, r->p, 8); r->p += 8; } return v; }
static float f32(Rd *r) { float v = 0; if (need(r, 4)) { memcpy(&v, r->p, 4); r->p += 4; } return v; }
static const char *str(Rd *r, uint64_t *n) {
    *n = u64(r);
    if (!need(r, *n)) { *n = 0; return ""; }
    const char *s = (const char *)r->p;
    r->p += *n;
    return s;
}
static int is(const char *s, uint64_t n, const char *lit) { return strlen(lit) == n && !memcmp(s, lit, n); }
/* Skips one metadata value of type t.  Arrays may nest (arrays of arrays);
 * a file nesting them deeper than any real one does is refused instead of
 * recursing without bound. */
#define GGUF_MAX_NESTING 16
static void skip_at(Rd *r, uint32_t t, int depth) {
    static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (t == 8) { uint64_t n; str(r, &n); return; }
    if (t == 9) {
        if (depth >= GGUF_MAX_NESTING) { r->err = 1; return; }
        uint32_t et = u32(r);
        uint64_t c = u64(r);
        for (uint64_t i = 0; i < c && !r->err; i++) skip_at(r, et, depth + 1);
        return;
    }
    if (t > 12) { r->err = 1; return; }
    if (need(r, (size_t)sz[t])) r->p += sz[t];
}
static void skip(Rd *r, uint32_t t) { skip_at(r, t, 0); }

typedef struct { char name[96]; uint32_t type; uint64_t dims[4]; uint32_t nd; uint64_t n, off; } TInfo;

/* The tensor's bytes do not lie inside the fsz bytes of tensor data (the
 * offset comes from the file: compared without forming off + bytes, which
 * a crafted offset could wrap around). */
static int past_end(const TInfo *t, size_t bytes, size_t fsz) { return t->off > fsz || bytes > fsz - t->off; }

/* ------------------------------------------------------------------------ */
static int upload_vec(const TInfo *t, const unsigned char *data, size_t fsz, int want, float **out) {
    size_t bytes;
    TRY(lmc_tensor_bytes(t->type, (size_t)t->n, &bytes));
    if ((int64_t)t->n != want) return lmc_set_error(LMC_ERR_IO, "tensor %s: %llu elements, expected %d", t->name,
                                                    (unsigned long long)t->n, want);
    if (past_end(t, bytes, fsz)) return lmc_set_error(LMC_ERR_IO, "tensor %s: data past end of file", t->name);
    CUTRY(cudaMalloc((void **)out, sizeof(float) * (size_t)want + 16));
    if (t->type == LMC_TYPE_F32) {
        CUTRY(cudaMemcpy(*out, data + t->off, bytes, cudaMemcpyHostToDevice));
        return LMC_OK;
    }
    void *tmp = NULL;
    CUTRY(cudaMalloc(&tmp, bytes + LMC_BLOCK_PAD));
    cudaMemset(tmp, 0, bytes + LMC_BLOCK_PAD);
    cudaMemcpy(tmp, data + t->off, bytes, cudaMemcpyHostToDevice);
    int rc = lmc_dequant(t->type, tmp, (size_t)t->n, *out, NULL);
    cudaDeviceSynchronize();
    cudaFree(tmp);
    return rc;
}

static int upload_mat(const TInfo *t, const unsigned char *data, size_t fsz, int rows, int cols, lmc_qtensor **out) {
    size_t bytes;
    TRY(lmc_tensor_bytes(t->type, (size_t)t->n, &bytes));
    if ((int64_t)t->n != (int64_t)rows * cols || (t->nd >= 2 && (t->dims[0] != (uint64_t)cols || t->dims[1] != (uint64_t)rows)))
        return lmc_set_error(LMC_ERR_IO, "tensor %s: shape mismatch (expected %d x %d)", t->name, rows, cols);
    if (past_end(t, bytes, fsz)) return lmc_set_error(LMC_ERR_IO, "tensor %s: data past end of file", t->name);
    return lmc_qtensor_upload(t->type, rows, cols, data + t->off, bytes, out);
}

/* Rows [r0, r0 + nr) of a row-major block matrix (rows must not share blocks). */
static int upload_rows(const TInfo *t, const unsigned char *data, size_t fsz, int rows, int cols, int r0, int nr,
                       lmc_qtensor **out) {
    size_t bytes, rb;
    TRY(lmc_tensor_bytes(t->type, (size_t)t->n, &bytes));
    if ((int64_t)t->n != (int64_t)rows * cols || (t->nd >= 2 && (t->dims[0] != (uint64_t)cols || t->dims[1] != (uint64_t)rows)))
        return lmc_set_error(LMC_ERR_IO, "tensor %s: shape mismatch (expected %d x %d)", t->name, rows, cols);
    if (past_end(t, bytes, fsz)) return lmc_set_error(LMC_ERR_IO, "tensor %s: data past end of file", t->name);
    if (lmc_tensor_bytes(t->type, (size_t)cols, &rb))
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "tensor %s: rows share blocks, cannot shard by rows", t->name);
    return lmc_qtensor_upload(t->type, nr, cols, data + t->off + (size_t)r0 * rb, (size_t)nr * rb, out);
}

/* Columns [c0, c0 + nc) of every row (block-aligned). */
static int upload_cols(const TInfo *t, const unsigned char *data, size_t fsz, int rows, int cols, int c0, int nc,
                       lmc_qtensor **out) {
    size_t bytes, rb, cb0, cbn;
    TRY(lmc_tensor_bytes(t->type, (size_t)t->n, &bytes));
    if ((int64_t)t->n != (int64_t)rows * cols || (t->nd >= 2 && (t->dims[0] != (uint64_t)cols || t->dims[1] != (uint64_t)rows)))
        return lmc_set_error(LMC_ERR_IO, "tensor %s: shape mismatch (expected %d x %d)", t->name, rows, cols);
    if (past_end(t, bytes, fsz)) return lmc_set_error(LMC_ERR_IO, "tensor %s: data past end of file", t->name);
    if (lmc_tensor_bytes(t->type, (size_t)cols, &rb) || lmc_tensor_bytes(t->type, (size_t)c0, &cb0) ||
        lmc_tensor_bytes(t->type, (size_t)nc, &cbn))
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "tensor %s: column shard [%d, %d) is not block-aligned", t->name, c0,
                             c0 + nc);
    unsigned char *buf = (unsigned char *)malloc((size_t)rows * cbn + 1);
    if (!buf) return lmc_set_error(LMC_ERR_OOM, "column shard of %s", t->name);
    for (int r = 0; r < rows; r++) memcpy(buf + (size_t)r * cbn, data + t->off + (size_t)r * rb + cb0, cbn);
    int rc = lmc_qtensor_upload(t->type, rows, nc, buf, (size_t)rows * cbn, out);
    free(buf);
    return rc;
}

static int dev_alloc(void **p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) return lmc_set_error(LMC_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    return cudaMemset(*p, 0, bytes ? bytes : 16) == cudaSuccess ? LMC_OK : lmc_set_error(LMC_ERR_CUDA, "memset");
}

/* Slot lookup for a tensor name (src/gguf.c:62-97). */
static int bind_tensor(lmc_model *m, const TInfo *t, const unsigned char *data, size_t fsz) {
    const lmc_model_config *c = &m->cfg;
    const int D = c->embed_dim, F = c->ffn_dim, V = c->vocab_size, S = c->seq_len;
    const int ll = c->arch == 2, KV = c->n_kv_heads * c->head_dim, QD = c->n_heads * c->head_dim;
    const char *nm = t->name;
    if (!strcmp(nm, "token_embd.weight")) return upload_mat(t, data, fsz, V, D, &m->wte);
    if (!strcmp(nm, "position_embd.weight")) return ll ? 0 : upload_vec(t, data, fsz, S * D, &m->wpe);
    if (!strcmp(nm, "output.weight"))
        return m->tp_size > 1 ? upload_rows(t, data, fsz, V, D, m->v0, m->vl, &m->lm_head)
                              : upload_mat(t, data, fsz, V, D, &m->lm_head);
    if (!strcmp(nm, "output_norm.weight")) return upload_vec(t, data, fsz, D, ll ? &m->rmsf : &m->lnf_w);
    if (!strcmp(nm, "output_norm.bias")) return ll ? 0 : upload_vec(t, data, fsz, D, &m->lnf_b);
    if (strncmp(nm, "blk.", 4)) return 0;
    int l = atoi(nm + 4);
    if (l < 0 || l >= c->n_layers) return 0;
    const char *r = strchr(nm + 4, '.');
    if (!r) return 0;
    r++;
    Layer *w = &m->layers[l];
    if (!ll) {
        if (!strcmp(r, "attn_norm.weight")) return upload_vec(t, data, fsz, D, &w->ln1_w);
        if (!strcmp(r, "attn_norm.bias")) return upload_vec(t, data, fsz, D, &w->ln1_b);
        if (!strcmp(r, "attn_qkv.weight")) return upload_mat(t, data, fsz, 3 * D, D, &w->qkv);
        if (!strcmp(r, "attn_qkv.bias")) return upload_vec(t, data, fsz, 3 * D, &w->qkv_b);
        if (!strcmp(r, "attn_output.weight")) return upload_mat(t, data, fsz, D, D, &w->proj);
        if (!strcmp(r, "attn_output.bias")) return upload_vec(t, data, fsz, D, &w->proj_b);
        if (!strcmp(r, "ffn_norm.weight")) return upload_vec(t, data, fsz, D, &w->ln2_w);
        if (!strcmp(r, "ffn_norm.bias")) return upload_vec(t, data, fsz, D, &w->ln2_b);
        if (!strcmp(r, "ffn_up.weight")) return upload_mat(t, data, fsz, F, D, &w->fc);
        if (!strcmp(r, "ffn_up.bias")) return upload_vec(t, data, fsz, F, &w->fc_b);
        if (!strcmp(r, "ffn_down.weight")) return upload_mat(t, data, fsz, D, F, &w->fc2);
        if (!strcmp(r, "ffn_down.bias")) return upload_vec(t, data, fsz, D, &w->fc2_b);
    } else {
        const int Dh = c->head_dim, tr = m->tp_rank;
        if (!strcmp(r, "attn_norm.weight")) return upload_vec(t, data, fsz, D, &w->rms_attn);
        if (!strcmp(r, "ffn_norm.weight")) return upload_vec(t, data, fsz, D, &w->rms_ffn);
        if (m->tp_size > 1) { /* this rank's shard (see struct lmc_model) */
            if (!strcmp(r, "attn_q.weight")) return upload_rows(t, data, fsz, QD, D, tr * m->hl * Dh, m->hl * Dh, &w->q);
            if (!strcmp(r, "attn_k.weight"))
                return upload_rows(t, data, fsz, KV, D, tr * m->hkvl * Dh, m->hkvl * Dh, &w->k);
            if (!strcmp(r, "attn_v.weight"))
                return upload_rows(t, data, fsz, KV, D, tr * m->hkvl * Dh, m->hkvl * Dh, &w->v);
            if (!strcmp(r, "attn_output.weight"))
                return upload_cols(t, data, fsz, D, QD, tr * m->hl * Dh, m->hl * Dh, &w->o);
            if (!strcmp(r, "ffn_gate.weight")) return upload_rows(t, data, fsz, F, D, tr * m->fl, m->fl, &w->gate);
            if (!strcmp(r, "ffn_up.weight")) return upload_rows(t, data, fsz, F, D, tr * m->fl, m->fl, &w->up);
            if (!strcmp(r, "ffn_down.weight")) return upload_cols(t, data, fsz, D, F, tr * m->fl, m->fl, &w->down);
            return 0;
        }
        if (!strcmp(r, "attn_q.weight")) return upload_mat(t, data, fsz, QD, D, &w->q);
        if (!strcmp(r, "attn_k.weight")) return upload_mat(t, data, fsz, KV, D, &w->k);
        if (!strcmp(r, "attn_v.weight")) return upload_mat(t, data, fsz, KV, D, &w->v);
        if (!strcmp(r, "attn_output.weight")) return upload_mat(t, data, fsz, D, QD, &w->o);
        if (!strcmp(r, "ffn_gate.weight")) return upload_mat(t, data, fsz, F, D, &w->gate);
        if (!strcmp(r, "ffn_up.weight")) return upload_mat(t, data, fsz, F, D, &w->up);
        if (!strcmp(r, "ffn_down.weight")) return upload_mat(t, data, fsz, D, F, &w->down);
    }
    return 0;
}

static int check_complete(const lmc_model *m) {
    const lmc_model_config *c = &m->cfg;
    if (!m->wte || !m->lm_head) return lmc_set_error(LMC_ERR_IO, "GGUF lacks token_embd.weight or output.weight");
    for (int l = 0; l < c->n_layers; l++) {
        const Layer *w = &m->layers[l];
        int ok = c->arch == 1 ? (w->qkv && w->proj && w->fc && w->fc2 && w->ln1_w && w->ln1_b && w->ln2_w &&
                                 w->ln2_b && w->qkv_b && w->proj_b && w->fc_b && w->fc2_b)
                              : (w->q && w->k && w->v && w->o && w->gate && w->up && w->down && w->rms_attn &&
                                 w->rms_ffn);
        if (!ok) return lmc_set_error(LMC_ERR_IO, "GGUF lacks tensors of layer %d", l);
    }
    if (c->arch == 1 && (!m->wpe || !m->lnf_w || !m->lnf_b))
        return lmc_set_error(LMC_ERR_IO, "GGUF lacks position_embd or output_norm");
    if (c->arch == 2 && !m->rmsf) return lmc_set_error(LMC_ERR_IO, "GGUF lacks output_norm.weight");
    return LMC_OK;
}

/* The GGUF file mapped read-only (pages are read from the file as the
 * parser and the staged uploads touch them: no whole-file copy in host
 * memory); a plain read into a heap buffer when mapping fails. */
typedef struct {
    unsigned char *p;
    size_t n;
    int mapped;
} FileView;
static int file_open(const char *path, FileView *v) {
    v->p = NULL;
    v->n = 0;
    v->mapped = 0;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return lmc_set_error(LMC_ERR_IO, "cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) || st.st_size <= 0) {
        close(fd);
        return lmc_set_error(LMC_ERR_IO, "cannot stat %s", path);
    }
    v->n = (size_t)st.st_size;
    void *p = mmap(NULL, v->n, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p != MAP_FAILED) {
        madvise(p, v->n, MADV_SEQUENTIAL);
        close(fd);
        v->p = (unsigned char *)p;
        v->mapped = 1;
        return LMC_OK;
    }
    v->p = (unsigned char *)malloc(v->n);
    if (!v->p) {
        close(fd);
        return lmc_set_error(LMC_ERR_OOM, "host buffer for %s", path);
    }
    size_t got = 0;
    while (got < v->n) {
        const ssize_t k = read(fd, v->p + got, v->n - got);
        if (k <= 0) break;
        got += (size_t)k;
    }
    close(fd);
    if (got != v->n) {
        free(v->p);
        v->p = NULL;
        return lmc_set_error(LMC_ERR_IO, "short read of %s", path);
    }
    return LMC_OK;
}
static void file_close(FileView *v) {
    if (!v->p) return;
    if (v->mapped) munmap(v->p, v->n);
    else free(v->p);
    v->p = NULL;
}

static int load(lmc_model *m, const char *path) {
    FileView fv;
    TRY(file_open(path, &fv));
    unsigned char *buf = fv.p;
    const size_t fsz = fv.n;
    Rd r = {buf, buf + fsz, 0};
    lmc_model_config *c = &m->cfg;
    int rc = LMC_OK;
    TInfo *ti = NULL;
    uint32_t magic = u32(&r), ver = u32(&r);
    if (magic != 0x46554747u || ver < 1 || ver > 3) { rc = lmc_set_error(LMC_ERR_IO, "%s: not a GGUF v1-3 file", path); goto done; }
    uint64_t nt = u64(&r), nkv = u64(&r);
    /* defaults, src/gguf.c:131-140 */
    c->arch = 0; c->vocab_size = 128256; c->seq_len = 8192; c->rope_theta = 10000.0f; c->norm_eps = 1e-5f;
    int vocab_key = 0, tok_count = 0;
    for (uint64_t i = 0; i < nkv && !r.err; i++) {
        uint64_t kl;
        const char *k = str(&r, &kl);
        uint32_t t = u32(&r);
        if (t == 4) { /* src/gguf.c:146-164 */
            int v = (int)u32(&r);
            if (is(k, kl, "gpt2.block_count") || is(k, kl, "llama.block_count")) c->n_layers = v;
            else if (is(k, kl, "gpt2.attention.head_count") || is(k, kl, "llama.attention.head_count")) c->n_heads = v;
            else if (is(k, kl, "gpt2.embedding_length") || is(k, kl, "llama.embedding_length")) c->embed_dim = v;
            else if (is(k, kl, "gpt2.feed_forward_length") || is(k, kl, "llama.feed_forward_length")) c->ffn_dim = v;
            else if (is(k, kl, "gpt2.context_length") || is(k, kl, "llama.context_length")) c->seq_len = v;
            else if (is(k, kl, "gpt2.vocab_size")) c->vocab_size = v;
            else if (is(k, kl, "llama.vocab_size")) { c->vocab_size = v; vocab_key = v; }
            else if (is(k, kl, "llama.attention.head_count_kv")) c->n_kv_heads = v;
        } else if (t == 6) { /* src/gguf.c:166-172 */
            float v = f32(&r);
            if (is(k, kl, "llama.rope.freq_base")) c->rope_theta = v;
            else if (is(k, kl, "llama.attention.layer_norm_rms_epsilon")) c->norm_eps = v;
        } else if (t == 8) { /* src/gguf.c:173-179 */
            uint64_t vl;
            const char *v = str(&r, &vl);
            if (is(k, kl, "general.architecture")) {
                if (is(v, vl, "llama")) c->arch = 2;
                else if (is(v, vl, "gpt2")) c->arch = 1;
            }
        } else if (t == 9 && is(k, kl, "tokenizer.ggml.tokens")) { /* src/gguf.c:184-199 */
            uint32_t et = u32(&r);
            uint64_t cnt = u64(&r);
            if (cnt <= 32768) tok_count = (int)cnt;
            for (uint64_t j = 0; j < cnt && !r.err; j++) skip(&r, et);
        } else {
            skip(&r, t);
        }
    }
    if (r.err) { rc = lmc_set_error(LMC_ERR_IO, "%s: truncated metadata", path); goto done; }
    /* src/gguf.c:218-244 */
    if (c->arch == 0) c->arch = c->n_kv_heads > 0 ? 2 : 1;
    if (c->arch == 2 && c->n_kv_heads == 0) c->n_kv_heads = c->n_heads;
    if (c->arch == 1) c->n_kv_heads = c->n_heads;
    if (c->arch == 1 && c->vocab_size == 128256) c->vocab_size = 50257;
    {
        int vn = tok_count ? tok_count : vocab_key;
        if (c->arch == 2 && vn > 0 && vn < c->vocab_size) c->vocab_size = vn;
    }
    if (!c->n_layers || !c->n_heads || !c->embed_dim) { rc = lmc_set_error(LMC_ERR_IO, "%s: missing L/H/D metadata", path); goto done; }
    {   /* the values are u32 in the file: none may be negative as an int or
         * so large that products of them overflow before any allocation */
        const int64_t lim = 1 << 24, f = c->ffn_dim ? c->ffn_dim : 4 * (int64_t)c->embed_dim;
        const int64_t dims[7] = {c->n_layers, c->n_heads, c->n_kv_heads, c->embed_dim, f, c->seq_len,
                                 c->vocab_size};
        for (int i = 0; i < 7; i++)
            if (dims[i] <= 0 || dims[i] > lim) {
                rc = lmc_set_error(LMC_ERR_IO, "%s: model dimension %lld outside [1, %lld] (L, H, Hkv, D, F, S, V = "
                                   "%d, %d, %d, %d, %lld, %d, %d)", path, (long long)dims[i], (long long)lim,
                                   c->n_layers, c->n_heads, c->n_kv_heads, c->embed_dim, (long long)f, c->seq_len,
                                   c->vocab_size);
                goto done;
            }
    }
    if (!c->ffn_dim) c->ffn_dim = 4 * c->embed_dim;
    c->head_dim = c->embed_dim / c->n_heads;
    if (c->n_heads % c->n_kv_heads) { rc = lmc_set_error(LMC_ERR_IO, "%s: heads %d not a multiple of kv heads %d", path, c->n_heads, c->n_kv_heads); goto done; }
    /* shard geometry (tensor parallel: LLaMA only, whole heads per rank) */
    m->hl = c->n_heads; m->hkvl = c->n_kv_heads; m->fl = c->ffn_dim; m->vl = c->vocab_size; m->v0 = 0;
    if (m->tp_size > 1) {
        const int N = m->tp_size;
        if (c->arch != 2) { rc = lmc_set_error(LMC_ERR_UNSUPPORTED, "tensor parallel: LLaMA models only"); goto done; }
        if (c->n_heads % N || c->n_kv_heads % N || c->ffn_dim % N) {
            rc = lmc_set_error(LMC_ERR_UNSUPPORTED, "tensor parallel: heads %d / kv heads %d / ffn %d not divisible by %d",
                               c->n_heads, c->n_kv_heads, c->ffn_dim, N);
            goto done;
        }
        m->hl = c->n_heads / N; m->hkvl = c->n_kv_heads / N; m->fl = c->ffn_dim / N;
        const int vr = (c->vocab_size + N - 1) / N;
        m->v0 = m->tp_rank * vr;
        m->vl = c->vocab_size - m->v0 < vr ? c->vocab_size - m->v0 : vr;
    }
    m->layers = (Layer *)calloc((size_t)c->n_layers, sizeof(Layer));
    ti = (TInfo *)calloc((size_t)nt ? (size_t)nt : 1, sizeof(TInfo));
    if (!m->layers || !ti) { rc = lmc_set_error(LMC_ERR_OOM, "host tables"); goto done; }
    for (uint64_t i = 0; i < nt && !r.err; i++) {
        uint64_t nl;
        const char *nm = str(&r, &nl);
        if (nl >= sizeof ti[i].name) nl = sizeof ti[i].name - 1;
        memcpy(ti[i].name, nm, nl);
        ti[i].nd = u32(&r);
        ti[i].n = 1;
        for (uint32_t d = 0; d < ti[i].nd; d++) {
            uint64_t v = u64(&r);
            if (d < 4) ti[i].dims[d] = v;
            ti[i].n *= v;
        }
        ti[i].type = u32(&r);
        ti[i].off = u64(&r);
    }
    if (r.err) { rc = lmc_set_error(LMC_ERR_IO, "%s: truncated tensor table", path); goto done; }
    {
        size_t data = ((size_t)(r.p - buf) + 31) / 32 * 32; /* src/gguf.c:285-287 */
        if (data > (size_t)fsz) { rc = lmc_set_error(LMC_ERR_IO, "%s: no tensor data after the header", path); goto done; }
        for (uint64_t i = 0; i < nt && !rc; i++) rc = bind_tensor(m, &ti[i], buf + data, (size_t)fsz - data);
    }
    if (!rc) rc = check_complete(m);
    if (!rc && c->arch == 2) { /* fuse q|k|v and gate|up (LMc keeps them separate, ops_llama.c:70-72,148-149) */
        for (int l = 0; l < c->n_layers && !rc; l++) {
            Layer *w = &m->layers[l];
            const lmc_qtensor *qkv[3] = {w->q, w->k, w->v}, *gu[2] = {w->gate, w->up};
            rc = lmc_qtensor_concat(qkv, 3, &w->qkv_cat);
            if (!rc) rc = lmc_qtensor_concat(gu, 2, &w->gateup_cat);
        }
    }
done:
    free(ti);
    file_close(&fv);
    return rc;
}

/* RoPE table with LMc's expression (src/models.c:101-117). */
static int build_rope(lmc_model *m) {
    const int S = m->cfg.seq_len, half = m->cfg.head_dim / 2;
    const float theta = m->cfg.rope_theta > 0.0f ? m->cfg.rope_theta : 10000.0f;
    float *c = (float *)malloc(sizeof(float) * (size_t)S * half), *s = (float *)malloc(sizeof(float) * (size_t)S * half);
    if (!c || !s) { free(c); free(s); return lmc_set_error(LMC_ERR_OOM, "rope table"); }
    for (int p = 0; p < S; p++)
        for (int d = 0; d < half; d++) {
            float a = (float)p / powf(theta, 2.0f * (float)d / (float)m->cfg.head_dim);
            c[(size_t)p * half + d] = cosf(a);
            s[(size_t)p * half + d] = sinf(a);
        }
    int rc = dev_alloc((void **)&m->rope_cos, sizeof(float) * (size_t)S * half);
    if (!rc) rc = dev_alloc((void **)&m->rope_sin, sizeof(float) * (size_t)S * half);
    if (!rc && (cudaMemcpy(m->rope_cos, c, sizeof(float) * (size_t)S * half, cudaMemcpyHostToDevice) != cudaSuccess ||
                cudaMemcpy(m->rope_sin, s, sizeof(float) * (size_t)S * half, cudaMemcpyHostToDevice) != cudaSuccess))
        rc = lmc_set_error(LMC_ERR_CUDA, "rope upload");
    free(c);
    free(s);
    return rc;
}

static int alloc_state(lmc_model *m) {
    const lmc_model_config *c = &m->cfg;
    /* KV cache: max_batch sequences; everything per row: max_rows rows */
    const size_t NS = (size_t)m->max_batch, B = (size_t)m->max_rows, D = c->embed_dim, F = c->ffn_dim,
                 V = c->vocab_size;
    const size_t QD = (size_t)c->n_heads * c->head_dim, KV = (size_t)c->n_kv_heads * c->head_dim;
    if (m->kv_dtype == LMC_KV_Q8 && (c->head_dim % 16 || c->head_dim > 512))
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "int8 KV rows need a head size that is a multiple of 16, <= 512");
    /* this rank's kv heads, rows of LMC_KV_ROW_BYTES */
    const size_t row_bytes = LMC_KV_ROW_BYTES(m->kv_dtype, c->head_dim);
    if (m->page_size) {
        if (c->seq_len % m->page_size)
            return lmc_set_error(LMC_ERR_INVALID, "KV page size %d does not divide the context %d", m->page_size,
                                 c->seq_len);
        m->max_pages = c->seq_len / m->page_size;
        const size_t table = NS * (size_t)m->max_pages;
        if ((size_t)m->n_pages > table) m->n_pages = (int)table; /* every sequence's whole context */
        m->kv_layer_bytes = (size_t)m->n_pages * m->hkvl * (size_t)m->page_size * row_bytes;
        TRY(dev_alloc((void **)&m->d_pages, sizeof(int) * table));
        CUTRY(cudaMemset(m->d_pages, 0xff, sizeof(int) * table)); /* -1: no page */
        m->h_pages = (int *)malloc(sizeof(int) * table);
        m->seq_np = (int *)calloc(NS, sizeof(int));
        m->free_ids = (int *)malloc(sizeof(int) * (size_t)m->n_pages);
        if (!m->h_pages || !m->seq_np || !m->free_ids) return lmc_set_error(LMC_ERR_OOM, "KV page table");
        for (size_t i = 0; i < table; i++) m->h_pages[i] = -1;
        for (int k = 0; k < m->n_pages; k++) m->free_ids[k] = m->n_pages - 1 - k; /* handed out as 0, 1, 2, ... */
        m->n_free = m->n_pages;
    } else {
        m->kv_layer_bytes = NS * (size_t)m->hkvl * (size_t)c->seq_len * row_bytes;
    }
    TRY(dev_alloc(&m->kc, m->kv_layer_bytes * c->n_layers));
    TRY(dev_alloc(&m->vc, m->kv_layer_bytes * c->n_layers));
    TRY(dev_alloc((void **)&m->x, 4 * B * D));
    TRY(dev_alloc((void **)&m->xn, 4 * B * D));
    TRY(dev_alloc((void **)&m->qkv, 4 * B * (QD + 2 * KV + 3 * D)));
    TRY(dev_alloc((void **)&m->att, 4 * B * (QD > D ? QD : D)));
    TRY(dev_alloc((void **)&m->h, 4 * B * 2 * F)); /* gate | up rows */
    TRY(dev_alloc((void **)&m->h2, 4 * B * F));
    TRY(dev_alloc((void **)&m->d_keys, 8 * B));
    {   /* LMC_ATTN_FUSED=0: merge the attention splits in a separate kernel
         * instead of in the last split CTA (same result, one launch more) */
        const char *f = getenv("LMC_ATTN_FUSED");
        if (!(f && f[0] == '0')) TRY(dev_alloc((void **)&m->d_attn_cnt, 4 * B * (size_t)m->hkvl));
    }
    TRY(dev_alloc((void **)&m->logits, 4 * B * V));
    /* attention split scratch: the split count depends on batch x heads, and a
     * step may run any batch up to B with this rank's heads */
    m->ws_bytes = 0;
    for (int b = 1; b <= (int)B; b++) {
        const size_t need = lmc_attention_workspace_bytes(b, m->hl, c->head_dim, c->seq_len);
        if (need > m->ws_bytes) m->ws_bytes = need;
    }
    TRY(dev_alloc(&m->ws, m->ws_bytes));
    TRY(dev_alloc((void **)&m->d_tok, 4 * B));
    TRY(dev_alloc((void **)&m->d_pos, 4 * B));
    TRY(dev_alloc((void **)&m->d_seq, 4 * B));
    TRY(dev_alloc((void **)&m->d_next, 4 * B));
    TRY(dev_alloc((void **)&m->d_step, 16));
    TRY(dev_alloc((void **)&m->d_rng, 8 * B));
    CUTRY(cudaMallocHost((void **)&m->h_stage, 3 * sizeof(int) * B));
    CUTRY(cudaHostAlloc((void **)&m->h_next_map, sizeof(int) * B, cudaHostAllocMapped));
    CUTRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    if (B > 8) { /* the batched GEMM's activation workspace, sized before any graph capture */
        const size_t kmax = D > F ? (D > QD ? D : QD) : (F > QD ? F : QD);
        TRY(lmc_gemm_reserve((int)B, (int)kmax, m->stream));
    }
    if (c->arch == 2) TRY(build_rope(m));
    return LMC_OK;
}

int lmc_nccl_unique_id(void *id) {
    if (!id) return lmc_set_error(LMC_ERR_INVALID, "nccl_unique_id: null");
    ncclUniqueId u;
    ncclResult_t r = ncclGetUniqueId(&u);
    if (r != ncclSuccess) return lmc_set_error(LMC_ERR_NCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
    memcpy(id, &u, sizeof u);
    return LMC_OK;
}

static int setup_peer(lmc_model *m);

static int model_load(const char *path, int max_batch, int max_rows, int kv_dtype, int page_size, int n_pages,
                      int tp_rank, int tp_size, const void *nccl_id, lmc_model **out) {
    if (!path || !out || max_batch <= 0) return lmc_set_error(LMC_ERR_INVALID, "model_load: args");
    if (page_size && (page_size < 16 || page_size > (1 << 16) || (page_size & (page_size - 1)) || n_pages <= 0))
        return lmc_set_error(LMC_ERR_INVALID, "model_load: KV pages of %d positions, %d pages (need a power of two "
                             "in [16, 65536] and at least one page)", page_size, n_pages);
    if (kv_dtype != LMC_KV_F32 && kv_dtype != LMC_KV_F16 && kv_dtype != LMC_KV_Q8)
        return lmc_set_error(LMC_ERR_INVALID, "model_load: kv dtype");
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size || (tp_size > 1 && !nccl_id))
        return lmc_set_error(LMC_ERR_INVALID, "model_load: shard %d of %d", tp_rank, tp_size);
    *out = NULL;
    lmc_model *m = (lmc_model *)calloc(1, sizeof(lmc_model));
    if (!m) return lmc_set_error(LMC_ERR_OOM, "model struct");
    m->max_batch = max_batch;
    m->max_rows = max_rows > max_batch ? max_rows : max_batch;
    m->kv_dtype = kv_dtype;
    m->page_size = page_size;
    while (page_size && (1 << m->page_shift) < page_size) m->page_shift++;
    m->n_pages = page_size ? n_pages : 0;
    m->tp_rank = tp_rank;
    m->tp_size = tp_size;
    int rc = load(m, path);
    if (!rc) rc = alloc_state(m);
    if (!rc && tp_size > 1) { /* every rank of the group calls this (collective) */
        ncclUniqueId u;
        memcpy(&u, nccl_id, sizeof u);
        ncclResult_t r = ncclCommInitRank(&m->comm, tp_size, u, tp_rank);
        if (r != ncclSuccess) { m->comm = NULL; rc = lmc_set_error(LMC_ERR_NCCL, "ncclCommInitRank: %s", ncclGetErrorString(r)); }
        const char *pe = getenv("LMC_TP_PEER"); /* 0: the residual sums through NCCL */
        if (!rc && !(pe && pe[0] == '0')) rc = setup_peer(m);
    }
    if (!rc && cudaDeviceSynchronize() != cudaSuccess) rc = lmc_set_error(LMC_ERR_CUDA, "load sync");
    if (rc) {
        char msg[1024];
        snprintf(msg, sizeof msg, "%s", lmc_last_error());
        lmc_model_free(m);
        return lmc_set_error(rc, "%s", msg);
    }
    *out = m;
    return LMC_OK;
}

int lmc_model_load(const char *path, int max_batch, int kv_dtype, lmc_model **out) {
    return model_load(path, max_batch, max_batch, kv_dtype, 0, 0, 0, 1, NULL, out);
}

int lmc_model_load_ex(const char *path, int max_batch, int max_rows, int kv_dtype, int tp_rank, int tp_size,
                      const void *nccl_id, lmc_model **out) {
    return model_load(path, max_batch, max_rows, kv_dtype, 0, 0, tp_rank, tp_size, nccl_id, out);
}

int lmc_model_load_tp(const char *path, int max_batch, int kv_dtype, int tp_rank, int tp_size, const void *nccl_id,
                      lmc_model **out) {
    return model_load(path, max_batch, max_batch, kv_dtype, 0, 0, tp_rank, tp_size, nccl_id, out);
}

int lmc_model_load_paged(const char *path, int max_batch, int max_rows, int kv_dtype, int page_size, int n_pages,
                         int tp_rank, int tp_size, const void *nccl_id, lmc_model **out) {
    if (page_size <= 0) return lmc_set_error(LMC_ERR_INVALID, "model_load_paged: page size %d", page_size);
    return model_load(path, max_batch, max_rows, kv_dtype, page_size, n_pages, tp_rank, tp_size, nccl_id, out);
}

/* Pages for positions [0, npos[i]) of sequence seqs[i], i < n (distinct
 * sequences), taken from the free ids before the step that writes them; the
 * changed table entries are copied to the device on the model's stream, so
 * they land after every step already queued.  All or nothing: with too few
 * free pages nothing changes and the call fails with LMC_ERR_OOM. */
static int pages_reserve(lmc_model *m, int n, const int *seqs, const int *npos) {
    if (!m->page_size) return LMC_OK;
    long long want = 0;
    for (int i = 0; i < n; i++) {
        const int need = (npos[i] + m->page_size - 1) >> m->page_shift;
        if (need > m->seq_np[seqs[i]]) want += need - m->seq_np[seqs[i]];
    }
    if (want > m->n_free)
        return lmc_set_error(LMC_ERR_OOM, "KV pages: %lld more needed, %d of %d free", want, m->n_free, m->n_pages);
    for (int i = 0; i < n; i++) {
        const int sq = seqs[i], need = (npos[i] + m->page_size - 1) >> m->page_shift, first = m->seq_np[sq];
        if (need <= first) continue;
        int *row = m->h_pages + (size_t)sq * m->max_pages;
        for (int k = first; k < need; k++) row[k] = m->free_ids[--m->n_free];
        m->seq_np[sq] = need;
        /* pageable source: the copy has taken the entries when the call returns */
        CUTRY(cudaMemcpyAsync(m->d_pages + (size_t)sq * m->max_pages + first, row + first,
                              sizeof(int) * (size_t)(need - first), cudaMemcpyHostToDevice, m->stream));
    }
    return LMC_OK;
}

/* The same pages for one position count shared by sequences 0 .. B-1. */
static int pages_reserve_all(lmc_model *m, int B, int npos) {
    if (!m->page_size) return LMC_OK;
    int rc = LMC_OK;
    int *seqs = (int *)malloc(sizeof(int) * 2 * (size_t)B);
    if (!seqs) return lmc_set_error(LMC_ERR_OOM, "KV pages: host");
    for (int b = 0; b < B; b++) { seqs[b] = b; seqs[B + b] = npos; }
    rc = pages_reserve(m, B, seqs, seqs + B);
    free(seqs);
    return rc;
}

int lmc_model_release_seq(lmc_model *m, int seq) {
    if (!m || seq < 0 || seq >= m->max_batch)
        return lmc_set_error(LMC_ERR_INVALID, "model_release_seq: sequence %d (of %d)", seq, m ? m->max_batch : 0);
    if (!m->page_size) return LMC_OK; /* the contiguous cache keeps every sequence's rows */
    const int np = m->seq_np[seq];
    int *row = m->h_pages + (size_t)seq * m->max_pages;
    for (int k = np - 1; k >= 0; k--) {
        m->free_ids[m->n_free++] = row[k];
        row[k] = -1;
    }
    m->seq_np[seq] = 0;
    if (np)
        CUTRY(cudaMemcpyAsync(m->d_pages + (size_t)seq * m->max_pages, row, sizeof(int) * (size_t)np,
                              cudaMemcpyHostToDevice, m->stream));
    return LMC_OK;
}

int lmc_model_kv_pages(const lmc_model *m, int *page_size, int *n_pages, int *n_free) {
    if (!m) return lmc_set_error(LMC_ERR_INVALID, "model_kv_pages: null");
    if (page_size) *page_size = m->page_size;
    if (n_pages) *n_pages = m->n_pages;
    if (n_free) *n_free = m->n_free;
    return LMC_OK;
}

int lmc_model_shard(const lmc_model *m, int *tp_rank, int *tp_size, int *vocab_begin, int *vocab_rows) {
    if (!m) return lmc_set_error(LMC_ERR_INVALID, "model_shard: null");
    if (tp_rank) *tp_rank = m->tp_rank;
    if (tp_size) *tp_size = m->tp_size;
    if (vocab_begin) *vocab_begin = m->v0;
    if (vocab_rows) *vocab_rows = m->vl;
    return LMC_OK;
}

int lmc_model_get_config(const lmc_model *m, lmc_model_config *c) {
    if (!m || !c) return lmc_set_error(LMC_ERR_INVALID, "model_get_config: null");
    *c = m->cfg;
    return LMC_OK;
}

void *lmc_model_device_buffer(lmc_model *m, int which) { return m && which == 0 ? m->logits : NULL; }

int lmc_model_free(lmc_model *m) {
    if (!m) return LMC_OK;
    if (m->gexec) cudaGraphExecDestroy(m->gexec); /* (it may hold the communicator's calls) */
    for (int b = 0; b < 3; b++) lmc_step_prog_free(m->pfwd[b]);
    lmc_step_prog_free(m->pgen);
    for (int p = 0; p < LMC_PEER_MAX; p++) {
        if (!m->peer_base[p]) continue;
        if (p == m->tp_rank) cudaFree(m->peer_base[p]);
        else cudaIpcCloseMemHandle(m->peer_base[p]);
    }
    if (m->comm) ncclCommDestroy(m->comm);
    if (m->layers) {
        for (int l = 0; l < m->cfg.n_layers; l++) {
            Layer *w = &m->layers[l];
            lmc_qtensor *qs[] = {w->qkv, w->proj, w->fc, w->fc2, w->q, w->k, w->v, w->o, w->gate, w->up, w->down,
                                 w->qkv_cat, w->gateup_cat, w->gateup_il};
            for (size_t i = 0; i < sizeof qs / sizeof qs[0]; i++) lmc_qtensor_free(qs[i]);
            float *vs[] = {w->ln1_w, w->ln1_b, w->ln2_w, w->ln2_b, w->qkv_b, w->proj_b, w->fc_b, w->fc2_b, w->rms_attn, w->rms_ffn};
            for (size_t i = 0; i < sizeof vs / sizeof vs[0]; i++) if (vs[i]) cudaFree(vs[i]);
        }
        free(m->layers);
    }
    lmc_qtensor_free(m->wte);
    lmc_qtensor_free(m->lm_head);
    void *ps[] = {m->wpe, m->lnf_w, m->lnf_b, m->rmsf, m->rope_cos, m->rope_sin, m->kc, m->vc, m->x, m->xn, m->qkv,
                  m->att, m->h, m->h2, m->logits, m->ws, m->d_tok, m->d_pos, m->d_next, m->d_step, m->d_prompt, m->d_ids,
                  m->d_keys, m->d_attn_cnt, m->d_seq, m->d_rng};
    for (size_t i = 0; i < sizeof ps / sizeof ps[0]; i++) if (ps[i]) cudaFree(ps[i]);
    if (m->d_pages) cudaFree(m->d_pages);
    free(m->h_pages);
    free(m->seq_np);
    free(m->free_ids);
    if (m->h_stage) cudaFreeHost(m->h_stage);
    if (m->h_next_map) cudaFreeHost(m->h_next_map);
    if (m->stream) cudaStreamDestroy(m->stream);
    free(m);
    return LMC_OK;
}

/* ------------------------------------------------------------------------ */
/* One decode step for B sequences: tokens d_tok, positions d_pos -> logits   */
/* and greedy ids in d_next.  Only kernel launches on m->stream (capturable). */
/* ------------------------------------------------------------------------ */
/* x -> norm -> W, as one tensor-core launch with the norm as its prologue
 * when W has the tiled layout (batch <= 8: the GEMV) or the batched GEMM
 * applies (batch > 8), else a norm kernel and a plain matmul. */
static int norm_matmul_in(lmc_model *m, const float *xin, const lmc_qtensor *W, int pro, const float *nw,
                          const float *nb, float eps, const float *bias, float *y, int ldy, int B, int epi,
                          unsigned long long *keys) {
    const int D = m->cfg.embed_dim;
    cudaStream_t s = m->stream;
    if ((B > 8 && W->gemm_wscale > 0.0f) || (lmc_qtensor_has_tiled(W) && (keys == NULL || B <= 8))) {
        lmc_gemv_extra ex = {pro, nw, nb, NULL, eps, keys, keys ? m->v0 : 0};
        return lmc_tiled_gemv_ex(W, xin, D, bias, y, ldy, B, epi, &ex, s);
    }
    if (keys && m->v0) return lmc_set_error(LMC_ERR_UNSUPPORTED, "sharded lm_head needs the tensor-core layout");
    if (pro == LMC_PRO_LAYERNORM) TRY(lmc_layer_norm(m->xn, xin, nw, nb, D, B, s));
    else TRY(lmc_rms_norm(m->xn, xin, nw, D, B, eps, s));
    TRY(lmc_matmul(W, m->xn, D, bias, y, ldy, B, epi, s));
    if (keys) TRY(lmc_argmax_keys_launch(y, W->rows, B, keys, s));
    return LMC_OK;
}
static int norm_matmul(lmc_model *m, const lmc_qtensor *W, int pro, const float *nw, const float *nb, float eps,
                       const float *bias, float *y, int ldy, int B, int epi, unsigned long long *keys) {
    return norm_matmul_in(m, m->x, W, pro, nw, nb, eps, bias, y, ldy, B, epi, keys);
}

/* Waits for the model's stream.  In a tensor-parallel group a step's NCCL
 * kernels wait for every rank, so a rank that left or failed would stall the
 * stream for good: the wait polls the stream, checks NCCL's asynchronous
 * error between polls, and on an error, or after LMC_NCCL_WAIT_S seconds
 * (default 300), aborts the communicator (which ends its kernels) and
 * returns LMC_ERR_NCCL or LMC_ERR_TIMEOUT.  The model then has no
 * communicator and its tensor-parallel calls fail. */
static int model_sync(lmc_model *m) {
    if (m->tp_size <= 1 || !m->comm) {
        CUTRY(cudaStreamSynchronize(m->stream));
        return LMC_OK;
    }
    const char *e = getenv("LMC_NCCL_WAIT_S");
    const double limit = e && atof(e) > 0 ? atof(e) : 300.0;
    struct timespec t0, t, nap = {0, 50000};
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (;;) {
        const cudaError_t q = cudaStreamQuery(m->stream);
        if (q == cudaSuccess) return LMC_OK;
        if (q != cudaErrorNotReady) return lmc_set_error(LMC_ERR_CUDA, "stream: %s", cudaGetErrorString(q));
        ncclResult_t ae = ncclSuccess;
        if (ncclCommGetAsyncError(m->comm, &ae) == ncclSuccess && ae != ncclSuccess && ae != ncclInProgress) {
            ncclCommAbort(m->comm);
            m->comm = NULL;
            return lmc_set_error(LMC_ERR_NCCL, "NCCL error in a step: %s (communicator aborted)",
                                 ncclGetErrorString(ae));
        }
        clock_gettime(CLOCK_MONOTONIC, &t);
        if ((double)(t.tv_sec - t0.tv_sec) + 1e-9 * (double)(t.tv_nsec - t0.tv_nsec) > limit) {
            ncclCommAbort(m->comm);
            m->comm = NULL;
            return lmc_set_error(LMC_ERR_TIMEOUT, "a step's collectives did not finish in %.0f s "
                                 "(a rank left?); communicator aborted", limit);
        }
        nanosleep(&nap, NULL);
    }
}

/* Sum of the ranks' partial x (tensor parallel): rank 0 added its partial to
 * the residual, the others wrote theirs over it, so the in-place sum is the
 * next residual on every rank. */
/* The regions of the peer sums: allocated and zeroed here, their IPC
 * handles exchanged over NCCL (all-gather), every peer's opened.  Collective. */
static int setup_peer(lmc_model *m) {
    const int R = m->tp_rank, N = m->tp_size;
    if (N > LMC_PEER_MAX) return LMC_OK;
    const size_t bytes = lmc_peer_region_bytes();
    CUTRY(cudaMalloc(&m->peer_base[R], bytes));
    CUTRY(cudaMemset(m->peer_base[R], 0, bytes));
    CUTRY(cudaDeviceSynchronize()); /* zeroed before any peer can write into it (the all-gather below) */
    cudaIpcMemHandle_t h;
    CUTRY(cudaIpcGetMemHandle(&h, m->peer_base[R]));
    char *dh = NULL, hs[LMC_PEER_MAX * sizeof(cudaIpcMemHandle_t)];
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    CUTRY(cudaMalloc((void **)&dh, hb * N));
    int rc = LMC_OK;
    if (cudaMemcpy(dh + hb * R, &h, hb, cudaMemcpyHostToDevice) != cudaSuccess) rc = lmc_set_error(LMC_ERR_CUDA, "peer handles");
    if (!rc && ncclAllGather(dh + hb * R, dh, hb, ncclChar, m->comm, m->stream) != ncclSuccess)
        rc = lmc_set_error(LMC_ERR_NCCL, "peer handles: all-gather");
    if (!rc) rc = model_sync(m);
    if (!rc && cudaMemcpy(hs, dh, hb * N, cudaMemcpyDeviceToHost) != cudaSuccess) rc = lmc_set_error(LMC_ERR_CUDA, "peer handles");
    cudaFree(dh);
    for (int p = 0; p < N && !rc; p++) {
        if (p == R) continue;
        cudaIpcMemHandle_t hp;
        memcpy(&hp, hs + hb * p, hb);
        if (cudaIpcOpenMemHandle(&m->peer_base[p], hp, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            m->peer_base[p] = NULL;
            rc = lmc_set_error(LMC_ERR_CUDA, "peer region of rank %d: cudaIpcOpenMemHandle", p);
        }
    }
    /* every rank must take the same path: peer sums only if every rank mapped every region */
    int *dok = NULL, ok = rc == LMC_OK;
    if (cudaMalloc((void **)&dok, sizeof(int)) == cudaSuccess) {
        if (cudaMemcpy(dok, &ok, sizeof(int), cudaMemcpyHostToDevice) == cudaSuccess &&
            ncclAllReduce(dok, dok, 1, ncclInt32, ncclMin, m->comm, m->stream) == ncclSuccess && model_sync(m) == LMC_OK)
            (void)cudaMemcpy(&ok, dok, sizeof(int), cudaMemcpyDeviceToHost);
        else
            ok = 0;
        cudaFree(dok);
    } else {
        ok = 0;
    }
    m->peer_on = ok;
    return m->comm ? LMC_OK : rc; /* without peer sums the NCCL path still works */
}

static int tp_sum_x(lmc_model *m, int B) {
    if (m->tp_size <= 1) return LMC_OK;
    const int n = B * m->cfg.embed_dim;
    if (m->peer_on && n <= lmc_peer_max_floats() && n % 4 == 0)
        return lmc_peer_allreduce(m->x, n, m->tp_rank, m->tp_size, m->peer_base, m->stream);
    if (!m->comm) return lmc_set_error(LMC_ERR_NCCL, "the tensor-parallel communicator was aborted");
    ncclResult_t r = ncclAllReduce(m->x, m->x, (size_t)B * m->cfg.embed_dim, ncclFloat32, ncclSum, m->comm, m->stream);
    return r == ncclSuccess ? LMC_OK : lmc_set_error(LMC_ERR_NCCL, "ncclAllReduce: %s", ncclGetErrorString(r));
}

/* The attention of one layer over its cache (contiguous or paged): q of
 * each row against the cached rows of its sequence, the new K/V rows
 * appended, output into m->att (row stride ldo). */
static int attn_rows(lmc_model *m, int ldo, const float *q, int ldq, const float *k, const float *v, int ldkv,
                     void *kc, void *vc, int B, int H, int Hkv, const float *rc, const float *rs) {
    const lmc_model_config *c = &m->cfg;
    const int *seq = m->prefill ? m->d_seq : NULL;
    if (m->page_size)
        return lmc_attention_rows_paged_launch(m->att, ldo, q, ldq, k, v, ldkv, kc, vc, m->kv_dtype, m->d_pos, seq, B,
                                               H, Hkv, c->head_dim, m->d_pages, m->max_pages, m->page_shift,
                                               m->n_pages, m->ws, m->ws_bytes, rc, rs, m->d_attn_cnt, m->stream);
    return lmc_attention_rows_launch(m->att, ldo, q, ldq, k, v, ldkv, kc, vc, m->kv_dtype, m->d_pos, seq, B, H, Hkv,
                                     c->head_dim, c->seq_len, m->ws, m->ws_bytes, rc, rs, m->d_attn_cnt, m->stream);
}

/* One decode step for B sequences: tokens d_tok, positions d_pos -> logits
 * and each sequence's greedy-pick key in d_keys.  Only kernel launches on
 * m->stream, so it can be captured as a graph.  LayerNorm / RMSNorm run as
 * the prologue of the projection that follows them, SwiGLU as the prologue
 * of ffn_down, and the greedy argmax as the epilogue of lm_head, whenever the
 * weights have the tensor-core layout. */
static int step(lmc_model *m, int B) {
    const lmc_model_config *c = &m->cfg;
    const int D = c->embed_dim, F = c->ffn_dim, V = c->vocab_size, H = c->n_heads;
    const int Dh = c->head_dim, S = c->seq_len;
    cudaStream_t s = m->stream;
    TRY(lmc_embed_launch(m->wte->type, m->wte->blocks, c->arch == 1 ? m->wpe : NULL, m->d_tok, m->d_pos, D, V, S, B,
                         m->x, s));
    for (int l = 0; l < c->n_layers; l++) {
        const Layer *w = &m->layers[l];
        char *kc = (char *)m->kc + m->kv_layer_bytes * l, *vc = (char *)m->vc + m->kv_layer_bytes * l;
        if (c->arch == 1) { /* src/ops.c:182-206 */
            TRY(norm_matmul(m, w->qkv, LMC_PRO_LAYERNORM, w->ln1_w, w->ln1_b, 1e-5f, w->qkv_b, m->qkv, 3 * D, B,
                            LMC_EPI_NONE, NULL));
            TRY(attn_rows(m, D, m->qkv, 3 * D, m->qkv + D, m->qkv + 2 * D, 3 * D, kc, vc, B, H, H, NULL, NULL));
            TRY(lmc_matmul(w->proj, m->att, D, w->proj_b, m->x, D, B, LMC_EPI_ACCUM, s));
            TRY(norm_matmul(m, w->fc, LMC_PRO_LAYERNORM, w->ln2_w, w->ln2_b, 1e-5f, w->fc_b, m->h, F, B, LMC_EPI_GELU,
                            NULL));
            TRY(lmc_matmul(w->fc2, m->h, F, w->fc2_b, m->x, D, B, LMC_EPI_ACCUM, s));
        } else { /* src/ops_llama.c:165-187 (this rank's heads and ffn rows when sharded) */
            const int QD = m->hl * Dh, KVD = m->hkvl * Dh, F = m->fl, H = m->hl, Hkv = m->hkvl;
            const int rp = m->tp_size > 1 && m->tp_rank > 0 ? LMC_EPI_NONE : LMC_EPI_ACCUM; /* residual add */
            const int LQ = QD + 2 * KVD;
            float *q = m->qkv, *k, *v;
            int ld;
            if (w->qkv_cat) {
                TRY(norm_matmul(m, w->qkv_cat, LMC_PRO_RMSNORM, w->rms_attn, NULL, c->norm_eps, NULL, q, LQ, B,
                                LMC_EPI_NONE, NULL));
                k = q + QD;
                v = q + QD + KVD;
                ld = LQ;
            } else {
                k = m->qkv + (size_t)B * QD;
                v = k + (size_t)B * KVD;
                TRY(lmc_rms_norm(m->xn, m->x, w->rms_attn, D, B, c->norm_eps, s));
                TRY(lmc_matmul(w->q, m->xn, D, NULL, q, QD, B, LMC_EPI_NONE, s));
                TRY(lmc_matmul(w->k, m->xn, D, NULL, k, KVD, B, LMC_EPI_NONE, s));
                TRY(lmc_matmul(w->v, m->xn, D, NULL, v, KVD, B, LMC_EPI_NONE, s));
                ld = 0;
            }
            /* RoPE on q and the new K row happens inside the attention kernel */
            TRY(attn_rows(m, QD, q, ld ? ld : QD, k, v, ld ? ld : KVD, kc, vc, B, H, Hkv, m->rope_cos, m->rope_sin));
            TRY(lmc_matmul(w->o, m->att, QD, NULL, m->x, D, B, rp, s));
            TRY(tp_sum_x(m, B));
            if (w->gateup_cat && (lmc_qtensor_has_tiled(w->down) || (B > 8 && w->down->gemm_wscale > 0.0f))) {
                TRY(norm_matmul(m, w->gateup_cat, LMC_PRO_RMSNORM, w->rms_ffn, NULL, c->norm_eps, NULL, m->h, 2 * F,
                                B, LMC_EPI_NONE, NULL));
                lmc_gemv_extra ex = {LMC_PRO_SWIGLU, NULL, NULL, m->h + F, 0.0f, NULL, 0};
                TRY(lmc_tiled_gemv_ex(w->down, m->h, 2 * F, NULL, m->x, D, B, rp, &ex, s));
            } else {
                TRY(lmc_rms_norm(m->xn, m->x, w->rms_ffn, D, B, c->norm_eps, s));
                TRY(lmc_matmul(w->gate, m->xn, D, NULL, m->h, F, B, LMC_EPI_NONE, s));
                TRY(lmc_matmul(w->up, m->xn, D, NULL, m->h2, F, B, LMC_EPI_NONE, s));
                TRY(lmc_swiglu(m->h, m->h2, (size_t)B * F, s));
                TRY(lmc_matmul(w->down, m->h, F, NULL, m->x, D, B, rp, s));
            }
            TRY(tp_sum_x(m, B));
        }
    }
    /* a prompt needs the logits of its last row only (the next token): the
     * head runs for the last chunk's last row and not at all for the others */
    if (m->prefill && !m->prefill_head) return LMC_OK;
    const float *xl = m->prefill ? m->x + (size_t)(B - 1) * D : m->x;
    const int BL = m->prefill ? 1 : B;
    if (c->arch == 1)
        TRY(norm_matmul_in(m, xl, m->lm_head, LMC_PRO_LAYERNORM, m->lnf_w, m->lnf_b, 1e-5f, NULL, m->logits, V, BL,
                           LMC_EPI_NONE, m->d_keys));
    else
        TRY(norm_matmul_in(m, xl, m->lm_head, LMC_PRO_RMSNORM, m->rmsf, NULL, c->norm_eps, NULL, m->logits, m->vl, BL,
                           LMC_EPI_NONE, m->d_keys));
    if (m->tp_size > 1) { /* greedy pick over the vocabulary shards: max of the 64-bit keys */
        if (!m->comm) return lmc_set_error(LMC_ERR_NCCL, "the tensor-parallel communicator was aborted");
        ncclResult_t r = ncclAllReduce(m->d_keys, m->d_keys, (size_t)BL, ncclUint64, ncclMax, m->comm, m->stream);
        if (r != ncclSuccess) return lmc_set_error(LMC_ERR_NCCL, "ncclAllReduce(keys): %s", ncclGetErrorString(r));
    }
    return LMC_OK;
}

/* ------------------------------------------------------------------------ */
/* The same step as one persistent launch (step_kernel.cu)                    */
/* ------------------------------------------------------------------------ */
/* The persistent step pays off where a step is many small ops (GPT-2 Small:
 * 87 MB of weights, ~5 us of weights per op).  For larger models each op
 * streams tens of MB and the kernel-by-kernel path, whose launches overlap
 * the next kernel's weight streaming with the current one (programmatic
 * dependent launch) and whose GEMVs keep long activation rows in registers,
 * measured faster (TinyLlama shape 901 vs 811 tokens/s, 8B shape 286 vs 267
 * at batch 1).  LMC_PERSISTENT=0 / 1 forces either path (same results). */
#define PERSIST_MAX_WEIGHT_BYTES (256ull << 20)
static size_t qt_bytes(const lmc_qtensor *t) { return t ? t->bytes : 0; }
static int persist_enabled(const lmc_model *m) {
    const char *e = getenv("LMC_PERSISTENT");
    if (e && e[0] == '0') return 0;
    if (e && e[0] == '1') return 1;
    size_t w = qt_bytes(m->wte) + qt_bytes(m->lm_head);
    for (int l = 0; l < m->cfg.n_layers; l++) {
        const Layer *y = &m->layers[l];
        w += qt_bytes(y->qkv) + qt_bytes(y->proj) + qt_bytes(y->fc) + qt_bytes(y->fc2) + qt_bytes(y->q) +
             qt_bytes(y->k) + qt_bytes(y->v) + qt_bytes(y->o) + qt_bytes(y->gate) + qt_bytes(y->up) +
             qt_bytes(y->down);
    }
    return w <= PERSIST_MAX_WEIGHT_BYTES;
}

static lmc_step_op *add_op(lmc_step_op *ops, int *n, int kind, int B) {
    lmc_step_op *o = &ops[(*n)++];
    memset(o, 0, sizeof *o);
    o->kind = kind;
    o->batch = B;
    return o;
}
static void add_gemv(lmc_step_op *ops, int *n, int B, const lmc_qtensor *w, const float *x, int ldx, const float *bias,
                     float *y, int ldy, int epi, int pro, const float *nw, const float *nb, float eps,
                     const float *x2) {
    lmc_step_op *o = add_op(ops, n, LMC_OP_GEMV, B);
    o->w = w;
    o->x = x;
    o->ldx = ldx;
    o->bias = bias;
    o->y = y;
    o->ldy = ldy;
    o->epi = epi;
    o->ex.pro = pro;
    o->ex.w = nw;
    o->ex.b = nb;
    o->ex.eps = eps;
    o->ex.x2 = x2;
}
static void add_attn(lmc_step_op *ops, int *n, lmc_model *m, int B, float *out, int ldo, const float *q, int ldq,
                     const float *k, const float *v, int ldkv, void *kc, void *vc, int H, int Hkv, const float *rc,
                     const float *rs) {
    const lmc_model_config *c = &m->cfg;
    lmc_step_op *o = add_op(ops, n, LMC_OP_ATTN, B);
    o->out = out;
    o->ldo = ldo;
    o->q = q;
    o->ldq = ldq;
    o->k_new = k;
    o->v_new = v;
    o->ldkv = ldkv;
    o->k_cache = kc;
    o->v_cache = vc;
    o->kv_dtype = m->kv_dtype;
    o->H = H;
    o->Hkv = Hkv;
    o->Dh = c->head_dim;
    o->S = c->seq_len;
    o->rope_cos = rc;
    o->rope_sin = rs;
    o->ws = m->ws;
    o->ws_bytes = m->ws_bytes;
    o->cnt = m->d_attn_cnt;
    o->pos = m->d_pos;
}

/* step() (and the greedy pick, or with gen the generate bookkeeping) as a
 * persistent program: the whole model on one GPU, batch <= 2, every
 * projection on the tiled layout; else LMC_ERR_UNSUPPORTED. */
static int build_prog(lmc_model *m, int B, int gen, int n_prompt, int n_new, lmc_step_prog **out) {
    const lmc_model_config *c = &m->cfg;
    *out = NULL;
    if (!persist_enabled(m) || m->tp_size > 1 || B > 2 || !m->d_attn_cnt || m->page_size)
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "persistent step: not for this model or batch");
    const int D = c->embed_dim, F = c->ffn_dim, V = c->vocab_size, H = c->n_heads, Dh = c->head_dim;
    lmc_step_op *ops = (lmc_step_op *)calloc((size_t)(5 * c->n_layers + 5), sizeof(lmc_step_op));
    if (!ops) return lmc_set_error(LMC_ERR_OOM, "persistent step: host");
    int n = 0, rc = LMC_OK;
    lmc_step_op *e = add_op(ops, &n, LMC_OP_EMBED, B);
    e->wte_type = m->wte->type;
    e->wte = m->wte->blocks;
    e->wpe = c->arch == 1 ? m->wpe : NULL;
    e->D = D;
    e->V = V;
    e->S = c->seq_len;
    e->tok = m->d_tok;
    e->pos = m->d_pos;
    e->y = m->x;
    /* norm statistics: slot 1 = x after the embedding, 2 + 2l = x after layer
     * l's attention output, 3 + 2l = x after layer l's FFN (see lmc_step_op) */
    e->stats_out = 1;
    for (int l = 0; l < c->n_layers && !rc; l++) {
        const int s_in = l == 0 ? 1 : 3 + 2 * (l - 1), s_mid = 2 + 2 * l, s_out = 3 + 2 * l;
        const int n0 = n;
        Layer *w = &m->layers[l];
        char *kc = (char *)m->kc + m->kv_layer_bytes * l, *vc = (char *)m->vc + m->kv_layer_bytes * l;
        if (c->arch == 1) { /* src/ops.c:182-206 */
            add_gemv(ops, &n, B, w->qkv, m->x, D, w->qkv_b, m->qkv, 3 * D, LMC_EPI_NONE, LMC_PRO_LAYERNORM, w->ln1_w,
                     w->ln1_b, 1e-5f, NULL);
            add_attn(ops, &n, m, B, m->att, D, m->qkv, 3 * D, m->qkv + D, m->qkv + 2 * D, 3 * D, kc, vc, H, H, NULL,
                     NULL);
            add_gemv(ops, &n, B, w->proj, m->att, D, w->proj_b, m->x, D, LMC_EPI_ACCUM, LMC_PRO_NONE, NULL, NULL, 0.0f,
                     NULL);
            add_gemv(ops, &n, B, w->fc, m->x, D, w->fc_b, m->h, F, LMC_EPI_GELU, LMC_PRO_LAYERNORM, w->ln2_w, w->ln2_b,
                     1e-5f, NULL);
            add_gemv(ops, &n, B, w->fc2, m->h, F, w->fc2_b, m->x, D, LMC_EPI_ACCUM, LMC_PRO_NONE, NULL, NULL, 0.0f,
                     NULL);
        } else { /* src/ops_llama.c:165-187 */
            if (!w->qkv_cat || !w->gateup_cat) {
                rc = lmc_set_error(LMC_ERR_UNSUPPORTED, "persistent step: q/k/v or gate/up not fused");
                break;
            }
            const int QD = H * Dh, KVD = c->n_kv_heads * Dh, LQ = QD + 2 * KVD;
            add_gemv(ops, &n, B, w->qkv_cat, m->x, D, NULL, m->qkv, LQ, LMC_EPI_NONE, LMC_PRO_RMSNORM, w->rms_attn,
                     NULL, c->norm_eps, NULL);
            add_attn(ops, &n, m, B, m->att, QD, m->qkv, LQ, m->qkv + QD, m->qkv + QD + KVD, LQ, kc, vc, H,
                     c->n_kv_heads, m->rope_cos, m->rope_sin);
            add_gemv(ops, &n, B, w->o, m->att, QD, NULL, m->x, D, LMC_EPI_ACCUM, LMC_PRO_NONE, NULL, NULL, 0.0f, NULL);
            /* gate and up interleaved by row tile: the gate|up GEMV finishes
             * h = silu(gate) * up itself, so the down projection reads h as
             * it is instead of every CTA redoing the SwiGLU on its input */
            if (!w->gateup_il && F % 16 == 0 && lmc_qtensor_has_tiled(w->gate) && lmc_qtensor_has_tiled(w->up)) {
                rc = lmc_qtensor_interleave(w->gate, w->up, 16, &w->gateup_il);
                if (rc) break;
            }
            if (w->gateup_il && w->gateup_il->tiled) {
                add_gemv(ops, &n, B, w->gateup_il, m->x, D, NULL, m->h, 2 * F, LMC_EPI_GLU_PAIRS, LMC_PRO_RMSNORM,
                         w->rms_ffn, NULL, c->norm_eps, NULL);
                add_gemv(ops, &n, B, w->down, m->h, 2 * F, NULL, m->x, D, LMC_EPI_ACCUM, LMC_PRO_NONE, NULL, NULL, 0.0f,
                         NULL);
            } else {
                add_gemv(ops, &n, B, w->gateup_cat, m->x, D, NULL, m->h, 2 * F, LMC_EPI_NONE, LMC_PRO_RMSNORM,
                         w->rms_ffn, NULL, c->norm_eps, NULL);
                add_gemv(ops, &n, B, w->down, m->h, 2 * F, NULL, m->x, D, LMC_EPI_ACCUM, LMC_PRO_SWIGLU, NULL, NULL,
                         0.0f, m->h + F);
            }
        }
        /* this layer's five ops: norm-in, attention, residual, norm-in, residual */
        ops[n0].stats_in = s_in;
        ops[n0 + 2].stats_out = s_mid;
        ops[n0 + 3].stats_in = s_mid;
        ops[n0 + 4].stats_out = s_out;
    }
    if (!rc) {
        if (c->arch == 1)
            add_gemv(ops, &n, B, m->lm_head, m->x, D, NULL, m->logits, V, LMC_EPI_NONE, LMC_PRO_LAYERNORM, m->lnf_w,
                     m->lnf_b, 1e-5f, NULL);
        else
            add_gemv(ops, &n, B, m->lm_head, m->x, D, NULL, m->logits, m->vl, LMC_EPI_NONE, LMC_PRO_RMSNORM, m->rmsf,
                     NULL, c->norm_eps, NULL);
        ops[n - 1].ex.keys = m->d_keys;
        ops[n - 1].ex.key_base = m->v0;
        ops[n - 1].stats_in = 3 + 2 * (c->n_layers - 1);
        if (gen && m->smp) { /* the top-p draw replaces the greedy pick */
            lmc_step_op *sp = add_op(ops, &n, LMC_OP_SAMPLE, B);
            sp->y = m->logits;
            sp->V = V;
            sp->temperature = m->smp_t;
            sp->top_p = m->smp_p;
            sp->rng = m->d_rng;
            sp->next = m->d_next;
            sp->step = m->d_step;
            sp->n_prompt = n_prompt;
        }
        lmc_step_op *k = add_op(ops, &n, gen ? LMC_OP_ADVANCE : LMC_OP_KEYS, B);
        k->from_next = gen && m->smp;
        if (!gen && cudaHostGetDevicePointer((void **)&k->next_host, m->h_next_map, 0) != cudaSuccess) {
            (void)cudaGetLastError(); /* lmc_model_forward reads the picks there: no persistent step without it */
            free(ops);
            return lmc_set_error(LMC_ERR_CUDA, "persistent step: no device address for the mapped picks");
        }
        k->keys = m->d_keys;
        k->next = m->d_next;
        k->tok = m->d_tok;
        k->pos = m->d_pos;
        k->step = m->d_step;
        k->prompt = m->d_prompt;
        k->ids = m->d_ids;
        k->n_prompt = n_prompt;
        k->n_new = n_new;
        rc = lmc_step_prog_build(ops, n, out);
    }
    free(ops);
    return rc;
}

/* The forward program for batch B, built on first use (NULL: not possible) */
static lmc_step_prog *fwd_prog(lmc_model *m, int B) {
    if (B > 2 || m->no_persist[B]) return NULL;
    if (!m->pfwd[B] && build_prog(m, B, 0, 0, 0, &m->pfwd[B]) != LMC_OK) m->no_persist[B] = 1;
    return m->pfwd[B];
}

int lmc_model_forward(lmc_model *m, const int *h_tokens, const int *h_pos, int B, float *h_logits, int *h_next) {
    if (!m || !h_tokens || !h_pos || B <= 0 || B > m->max_batch)
        return lmc_set_error(LMC_ERR_INVALID, "model_forward: args (batch %d, max %d)", B, m ? m->max_batch : 0);
    for (int b = 0; b < B; b++) {
        if (h_tokens[b] < 0 || h_tokens[b] >= m->cfg.vocab_size)
            return lmc_set_error(LMC_ERR_INVALID, "model_forward: token %d outside [0, %d)", h_tokens[b], m->cfg.vocab_size);
        if (h_pos[b] < 0 || h_pos[b] >= m->cfg.seq_len)
            return lmc_set_error(LMC_ERR_INVALID, "model_forward: position %d outside [0, %d)", h_pos[b], m->cfg.seq_len);
    }
    if (m->page_size) { /* row b is sequence b: pages up to its position */
        int *sp = (int *)malloc(sizeof(int) * 2 * (size_t)B);
        if (!sp) return lmc_set_error(LMC_ERR_OOM, "model_forward: host");
        for (int b = 0; b < B; b++) { sp[b] = b; sp[B + b] = h_pos[b] + 1; }
        const int rc = pages_reserve(m, B, sp, sp + B);
        free(sp);
        TRY(rc);
    }
    lmc_step_prog *p = fwd_prog(m, B);
    if (p) {
        /* the persistent step takes the tokens and positions in its launch
         * and writes its picks into mapped host memory: no copies */
        TRY(lmc_step_prog_launch_imm(p, m->stream, h_tokens, h_pos, B, m->d_tok, m->d_pos));
    } else {
        memcpy(m->h_stage, h_tokens, sizeof(int) * B);
        memcpy(m->h_stage + B, h_pos, sizeof(int) * B);
        CUTRY(cudaMemcpyAsync(m->d_tok, m->h_stage, sizeof(int) * B, cudaMemcpyHostToDevice, m->stream));
        CUTRY(cudaMemcpyAsync(m->d_pos, m->h_stage + B, sizeof(int) * B, cudaMemcpyHostToDevice, m->stream));
        TRY(step(m, B));
        TRY(lmc_keys_to_ids_launch(m->d_keys, m->d_next, B, m->stream));
    }
    if (h_logits) /* [B][vocab rows of this rank] (the whole vocabulary without sharding) */
        CUTRY(cudaMemcpyAsync(h_logits, m->logits, sizeof(float) * (size_t)B * m->vl, cudaMemcpyDeviceToHost,
                              m->stream));
    if (!p) CUTRY(cudaMemcpyAsync(m->h_stage + 2 * B, m->d_next, sizeof(int) * B, cudaMemcpyDeviceToHost, m->stream));
    TRY(model_sync(m));
    if (h_next) memcpy(h_next, p ? m->h_next_map : m->h_stage + 2 * B, sizeof(int) * B);
    return LMC_OK;
}

/* Prompt chunks of sequence `seq` (validated by the caller); `head`: run the
 * lm_head for the last position (its greedy key in d_keys[0]). */
static int prefill_chunks(lmc_model *m, int seq, const int *h_tokens, int n, int start_pos, int head) {
    cudaStream_t s = m->stream;
    const int R = m->max_rows;
    int rc = LMC_OK;
    for (int i0 = 0; i0 < n && !rc; i0 += R) {
        const int c = n - i0 < R ? n - i0 : R;
        for (int r = 0; r < c; r++) {
            m->h_stage[r] = h_tokens[i0 + r];
            m->h_stage[R + r] = start_pos + i0 + r;
            m->h_stage[2 * R + r] = seq;
        }
        CUTRY(cudaMemcpyAsync(m->d_tok, m->h_stage, sizeof(int) * c, cudaMemcpyHostToDevice, s));
        CUTRY(cudaMemcpyAsync(m->d_pos, m->h_stage + R, sizeof(int) * c, cudaMemcpyHostToDevice, s));
        CUTRY(cudaMemcpyAsync(m->d_seq, m->h_stage + 2 * R, sizeof(int) * c, cudaMemcpyHostToDevice, s));
        m->prefill = 1;
        m->prefill_head = head && i0 + c == n;
        if (m->prefill_head) CUTRY(cudaMemsetAsync(m->d_keys, 0, sizeof(unsigned long long), s));
        rc = step(m, c);
        m->prefill = m->prefill_head = 0;
        /* the staging buffer is rewritten for the next chunk */
        if (!rc) rc = model_sync(m);
    }
    return rc;
}

int lmc_model_prefill(lmc_model *m, int seq, const int *h_tokens, int n, int start_pos, float *h_logits, int *h_next) {
    if (!m || !h_tokens || n <= 0 || seq < 0 || seq >= m->max_batch || start_pos < 0 ||
        start_pos > m->cfg.seq_len || n > m->cfg.seq_len - start_pos) /* (no int overflow) */
        return lmc_set_error(LMC_ERR_INVALID, "model_prefill: sequence %d (of %d), positions %d + %d (context %d)", seq,
                             m ? m->max_batch : 0, start_pos, n, m ? m->cfg.seq_len : 0);
    for (int i = 0; i < n; i++)
        if (h_tokens[i] < 0 || h_tokens[i] >= m->cfg.vocab_size)
            return lmc_set_error(LMC_ERR_INVALID, "model_prefill: token %d outside [0, %d)", h_tokens[i], m->cfg.vocab_size);
    cudaStream_t s = m->stream;
    const int npos = start_pos + n;
    TRY(pages_reserve(m, 1, &seq, &npos));
    TRY(prefill_chunks(m, seq, h_tokens, n, start_pos, 1));
    TRY(lmc_keys_to_ids_launch(m->d_keys, m->d_next, 1, s));
    if (h_logits) CUTRY(cudaMemcpyAsync(h_logits, m->logits, sizeof(float) * m->vl, cudaMemcpyDeviceToHost, s));
    CUTRY(cudaMemcpyAsync(m->h_stage, m->d_next, sizeof(int), cudaMemcpyDeviceToHost, s));
    TRY(model_sync(m));
    if (h_next) *h_next = m->h_stage[0];
    return LMC_OK;
}

/* step + bookkeeping, the unit that is captured as one graph */
static int gen_step(lmc_model *m, int B, int n_prompt, int n_new) {
    if (m->pgen) return lmc_step_prog_launch(m->pgen, m->stream);
    TRY(step(m, B));
    if (m->smp)
        TRY(lmc_sample_launch(m->logits, m->cfg.vocab_size, m->vl, B, m->smp_t, m->smp_p, m->d_rng, m->d_next,
                              m->d_step, n_prompt, m->stream));
    return lmc_advance_launch(m->d_keys, m->d_next, m->d_tok, m->d_pos, m->d_step, m->d_prompt, n_prompt, m->d_ids, n_new, B,
                              m->smp, m->stream);
}

static int ensure_gen_buffers(lmc_model *m, int B, int n_prompt, int n_new) {
    if (m->prompt_cap < B * n_prompt) {
        if (m->d_prompt) cudaFree(m->d_prompt);
        m->d_prompt = NULL;
        TRY(dev_alloc((void **)&m->d_prompt, sizeof(int) * (size_t)B * n_prompt));
        m->prompt_cap = B * n_prompt;
        if (m->gexec) { cudaGraphExecDestroy(m->gexec); m->gexec = NULL; }
    }
    if (m->ids_cap < B * n_new) {
        if (m->d_ids) cudaFree(m->d_ids);
        m->d_ids = NULL;
        TRY(dev_alloc((void **)&m->d_ids, sizeof(int) * (size_t)B * n_new));
        m->ids_cap = B * n_new;
        if (m->gexec) { cudaGraphExecDestroy(m->gexec); m->gexec = NULL; }
    }
    return LMC_OK;
}

static int generate(lmc_model *m, const int *h_prompt, int n_prompt, int B, int n_new, int use_graph,
                    int *h_out_ids);

int lmc_model_generate(lmc_model *m, const int *h_prompt, int n_prompt, int B, int n_new, int use_graph,
                       int *h_out_ids) {
    if (m) m->smp = 0;
    return generate(m, h_prompt, n_prompt, B, n_new, use_graph, h_out_ids);
}

int lmc_model_generate_sample(lmc_model *m, const int *h_prompt, int n_prompt, int B, int n_new, float temperature,
                              float top_p, unsigned long long seed, int use_graph, int *h_out_ids) {
    if (!m || B <= 0 || B > m->max_batch) return lmc_set_error(LMC_ERR_INVALID, "model_generate_sample: args");
    if (temperature != temperature || top_p != top_p)
        return lmc_set_error(LMC_ERR_INVALID, "model_generate_sample: NaN temperature or top_p");
    if (m->tp_size > 1)
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "model_generate_sample: the vocabulary is sharded across ranks");
    /* sequence b draws from its own stream, seeded as LMc seeds its one
     * stream (src/lmc.c:30-31) with seed + b */
    unsigned long long *st = (unsigned long long *)malloc(sizeof(unsigned long long) * (size_t)B);
    if (!st) return lmc_set_error(LMC_ERR_OOM, "model_generate_sample: host");
    for (int b = 0; b < B; b++) st[b] = lmc_rng_seed(seed + (unsigned long long)b);
    cudaError_t e = cudaMemcpy(m->d_rng, st, sizeof(unsigned long long) * (size_t)B, cudaMemcpyHostToDevice);
    free(st);
    if (e != cudaSuccess) return lmc_set_error(LMC_ERR_CUDA, "model_generate_sample: %s", cudaGetErrorString(e));
    m->smp = 1;
    m->smp_t = temperature;
    m->smp_p = top_p;
    const int rc = generate(m, h_prompt, n_prompt, B, n_new, use_graph, h_out_ids);
    m->smp = 0;
    return rc;
}

static int generate(lmc_model *m, const int *h_prompt, int n_prompt, int B, int n_new, int use_graph,
                    int *h_out_ids) {
    if (!m || !h_prompt || n_prompt <= 0 || n_new <= 0 || B <= 0 || B > m->max_batch || !h_out_ids)
        return lmc_set_error(LMC_ERR_INVALID, "model_generate: args");
    if (n_prompt > m->cfg.seq_len || n_new - 1 > m->cfg.seq_len - n_prompt) /* (no int overflow) */
        return lmc_set_error(LMC_ERR_INVALID, "model_generate: %d + %d tokens exceed the context of %d", n_prompt,
                             n_new, m->cfg.seq_len);
    for (int i = 0; i < B * n_prompt; i++)
        if (h_prompt[i] < 0 || h_prompt[i] >= m->cfg.vocab_size)
            return lmc_set_error(LMC_ERR_INVALID, "model_generate: token %d out of range", h_prompt[i]);
    TRY(ensure_gen_buffers(m, B, n_prompt, n_new));
    /* the loop writes positions 0 .. n_prompt + n_new - 2 of sequences 0 .. B-1 */
    TRY(pages_reserve_all(m, B, n_prompt + n_new - 1));
    /* LMC_NO_GRAPH=1 launches the kernels directly (profilers that cannot
     * replay graph kernel nodes one by one); the kernels are the same. */
    const char *ng = getenv("LMC_NO_GRAPH");
    if (ng && ng[0] == '1') use_graph = 0;
    cudaStream_t s = m->stream;
    /* With more rows per step than sequences (lmc_model_load_ex) every prompt
     * but its last token goes through batched prefill; the step loop then
     * starts at the last prompt position (same ids: the cache holds the same
     * rows either way). */
    const int p0 = m->max_rows > m->max_batch && n_prompt > 1 ? n_prompt - 1 : 0;
    for (int b = 0; b < B && p0; b++) TRY(prefill_chunks(m, b, h_prompt + (size_t)b * n_prompt, p0, 0, 0));
    CUTRY(cudaMemcpyAsync(m->d_prompt, h_prompt, sizeof(int) * (size_t)B * n_prompt, cudaMemcpyHostToDevice, s));
    for (int b = 0; b < B; b++) { m->h_stage[b] = h_prompt[(size_t)b * n_prompt + p0]; m->h_stage[B + b] = p0; }
    CUTRY(cudaMemcpyAsync(m->d_tok, m->h_stage, sizeof(int) * B, cudaMemcpyHostToDevice, s));
    CUTRY(cudaMemcpyAsync(m->d_pos, m->h_stage + B, sizeof(int) * B, cudaMemcpyHostToDevice, s));
    m->h_stage[2 * B] = p0;
    CUTRY(cudaMemcpyAsync(m->d_step, m->h_stage + 2 * B, sizeof(int), cudaMemcpyHostToDevice, s));
    const int steps = n_prompt + n_new - 1 - p0;
    /* the persistent program of this loop (its advance op holds the prompt
     * and id buffers and the loop's shape) */
    if (m->pgen && (m->pg_batch != B || m->pg_nprompt != n_prompt || m->pg_nnew != n_new ||
                    m->pg_prompt != m->d_prompt || m->pg_ids != m->d_ids || m->pg_smp != m->smp ||
                    (m->smp && (m->pg_t != m->smp_t || m->pg_p != m->smp_p)))) {
        if (m->gexec) { cudaGraphExecDestroy(m->gexec); m->gexec = NULL; }
        lmc_step_prog_free(m->pgen);
        m->pgen = NULL;
    }
    if (!m->pgen && B <= 2 && !m->gen_persist_failed) {
        if (build_prog(m, B, 1, n_prompt, n_new, &m->pgen) == LMC_OK) {
            m->pg_batch = B; m->pg_nprompt = n_prompt; m->pg_nnew = n_new;
            m->pg_prompt = m->d_prompt; m->pg_ids = m->d_ids;
            m->pg_smp = m->smp; m->pg_t = m->smp_t; m->pg_p = m->smp_p;
            if (m->gexec) { cudaGraphExecDestroy(m->gexec); m->gexec = NULL; }
        } else {
            m->gen_persist_failed = 1;
        }
    }
    if (use_graph) {
        if (m->gexec && (m->g_batch != B || m->g_nprompt != n_prompt || m->g_nnew != n_new || m->g_smp != m->smp ||
                         (m->smp && (m->g_t != m->smp_t || m->g_p != m->smp_p)))) {
            cudaGraphExecDestroy(m->gexec);
            m->gexec = NULL;
        }
        if (!m->gexec) {
            cudaGraph_t g;
            CUTRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
            int rc = gen_step(m, B, n_prompt, n_new);
            cudaError_t e = cudaStreamEndCapture(s, &g);
            if (rc) { if (e == cudaSuccess) cudaGraphDestroy(g); return rc; }
            if (e != cudaSuccess) return lmc_set_error(LMC_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
            size_t nn = 0;
            m->g_kernels = 0;
            if (cudaGraphGetNodes(g, NULL, &nn) == cudaSuccess && nn) {
                cudaGraphNode_t *nodes = (cudaGraphNode_t *)malloc(sizeof(cudaGraphNode_t) * nn);
                if (nodes && cudaGraphGetNodes(g, nodes, &nn) == cudaSuccess)
                    for (size_t i = 0; i < nn; i++) {
                        enum cudaGraphNodeType ty;
                        if (cudaGraphNodeGetType(nodes[i], &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel)
                            m->g_kernels++;
                    }
                free(nodes);
            }
            e = cudaGraphInstantiate(&m->gexec, g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) return lmc_set_error(LMC_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
            m->g_batch = B; m->g_nprompt = n_prompt; m->g_nnew = n_new;
            m->g_smp = m->smp; m->g_t = m->smp_t; m->g_p = m->smp_p;
        }
        for (int i = 0; i < steps; i++) CUTRY(cudaGraphLaunch(m->gexec, s));
    } else {
        if (m->gexec) { cudaGraphExecDestroy(m->gexec); m->gexec = NULL; }
        m->g_batch = B; m->g_nprompt = n_prompt; m->g_nnew = n_new;
        m->g_smp = m->smp; m->g_t = m->smp_t; m->g_p = m->smp_p;
        for (int i = 0; i < steps; i++) TRY(gen_step(m, B, n_prompt, n_new));
    }
    /* the last greedy pick needs no forward of its own: take it from the
     * last step's argmax (the advance kernel recorded it as well) */
    CUTRY(cudaMemcpyAsync(h_out_ids, m->d_ids, sizeof(int) * (size_t)B * n_new, cudaMemcpyDeviceToHost, s));
    TRY(model_sync(m));
    m->g_pos = n_prompt + n_new - 1;
    return LMC_OK;
}

/* Runs `n` more steps of the last generation (its captured graph, or direct
 * launches when it ran without one) without resetting state: timed decode
 * steps continue from the current device-side position. */
int lmc_model_replay(lmc_model *m, int n, void *stream_out) {
    if (!m || !m->g_batch) return lmc_set_error(LMC_ERR_INVALID, "model_replay: no generation to continue");
    if (m->page_size) { /* pages for the positions these steps write */
        if (n < 0 || n > m->cfg.seq_len - m->g_pos)
            return lmc_set_error(LMC_ERR_INVALID, "model_replay: positions %d + %d exceed the context of %d", m->g_pos,
                                 n, m->cfg.seq_len);
        TRY(pages_reserve_all(m, m->g_batch, m->g_pos + n));
    }
    m->g_pos += n > 0 ? n : 0;
    m->smp = m->g_smp; /* the last generation's pick: greedy or its top-p draw */
    m->smp_t = m->g_t;
    m->smp_p = m->g_p;
    int rc = LMC_OK;
    for (int i = 0; i < n && !rc; i++) {
        if (m->gexec) {
            if (cudaGraphLaunch(m->gexec, m->stream) != cudaSuccess) rc = lmc_set_error(LMC_ERR_CUDA, "graph launch");
        } else {
            rc = gen_step(m, m->g_batch, m->g_nprompt, m->g_nnew);
        }
    }
    m->smp = 0;
    TRY(rc);
    if (stream_out) *(cudaStream_t *)stream_out = m->stream;
    return LMC_OK;
}

int lmc_model_graph_kernels(const lmc_model *m) { return m && m->gexec ? m->g_kernels : -1; }

const lmc_qtensor *lmc_model_matrix(const lmc_model *m, int layer, int which) {
    if (!m) return NULL;
    if (which == LMC_W_TOKEN_EMBD) return m->wte;
    if (which == LMC_W_OUTPUT) return m->lm_head;
    if (layer < 0 || layer >= m->cfg.n_layers) return NULL;
    const Layer *w = &m->layers[layer];
    const int gpt2 = m->cfg.arch == 1;
    switch (which) {
    case LMC_W_QKV: return gpt2 ? w->qkv : NULL;
    case LMC_W_ATTN_OUT: return gpt2 ? w->proj : w->o;
    case LMC_W_FFN_UP: return gpt2 ? w->fc : w->up;
    case LMC_W_FFN_DOWN: return gpt2 ? w->fc2 : w->down;
    case LMC_W_Q: return gpt2 ? NULL : w->q;
    case LMC_W_K: return gpt2 ? NULL : w->k;
    case LMC_W_V: return gpt2 ? NULL : w->v;
    case LMC_W_GATE: return gpt2 ? NULL : w->gate;
    default: return NULL;
    }
}

const float *lmc_model_vector(const lmc_model *m, int layer, int which, int *len) {
    if (!m) return NULL;
    const lmc_model_config *c = &m->cfg;
    const int D = c->embed_dim, gpt2 = c->arch == 1;
    const float *v = NULL;
    int n = D;
    switch (which) {
    case LMC_V_POS_EMBD: v = gpt2 ? m->wpe : NULL; n = c->seq_len * D; break;
    case LMC_V_OUTPUT_NORM: v = gpt2 ? m->lnf_w : m->rmsf; break;
    case LMC_V_OUTPUT_NORM_B: v = gpt2 ? m->lnf_b : NULL; break;
    case LMC_V_ROPE_COS: v = gpt2 ? NULL : m->rope_cos; n = c->seq_len * (c->head_dim / 2); break;
    case LMC_V_ROPE_SIN: v = gpt2 ? NULL : m->rope_sin; n = c->seq_len * (c->head_dim / 2); break;
    default: {
        if (layer < 0 || layer >= c->n_layers) return NULL;
        const Layer *w = &m->layers[layer];
        switch (which) {
        case LMC_V_ATTN_NORM: v = gpt2 ? w->ln1_w : w->rms_attn; break;
        case LMC_V_ATTN_NORM_B: v = gpt2 ? w->ln1_b : NULL; break;
        case LMC_V_FFN_NORM: v = gpt2 ? w->ln2_w : w->rms_ffn; break;
        case LMC_V_FFN_NORM_B: v = gpt2 ? w->ln2_b : NULL; break;
        case LMC_V_QKV_B: v = gpt2 ? w->qkv_b : NULL; n = 3 * D; break;
        case LMC_V_ATTN_OUT_B: v = gpt2 ? w->proj_b : NULL; break;
        case LMC_V_FFN_UP_B: v = gpt2 ? w->fc_b : NULL; n = c->ffn_dim; break;
        case LMC_V_FFN_DOWN_B: v = gpt2 ? w->fc2_b : NULL; break;
        default: return NULL;
        }
    }
    }
    if (v && len) *len = n;
    return v;
}
