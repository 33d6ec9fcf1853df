/* host_shard_fakes.c - host stand-ins for what the model loader
 * (lmc_b200/host/lmc_model.c) calls on the device side, so the loader runs
 * on a machine without a GPU (tests/test_host_shards.py).  Device memory is
 * host memory; every qtensor upload is written to $LMC_FAKE_DUMP/NNNN.bin
 * and logged on stdout as "Q <n> <type> <rows> <cols> <bytes>", every
 * host-to-device copy as "M <bytes>"; the NCCL communicator is a token.
 * Nothing here computes: the kernel launchers and collectives fail if
 * called (loading calls none of them). */
#include <stdarg.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* The few declarations needed, written here: the library's headers declare
 * the same functions with CUDA types, which these stand-ins replace. */
enum { LMC_OK = 0, LMC_ERR_INVALID = -1, LMC_ERR_UNSUPPORTED = -2, LMC_ERR_IO = -5, LMC_KV_F16 = 1 };
enum { LMC_TYPE_F32 = 0, LMC_TYPE_F16 = 1, LMC_TYPE_Q4_0 = 2, LMC_TYPE_Q4_1 = 3, LMC_TYPE_Q5_0 = 6,
       LMC_TYPE_Q5_1 = 7, LMC_TYPE_Q8_0 = 8, LMC_TYPE_Q2_K = 10, LMC_TYPE_Q3_K = 11, LMC_TYPE_Q4_K = 12,
       LMC_TYPE_Q5_K = 13, LMC_TYPE_Q6_K = 14, LMC_TYPE_IQ3_XXS = 18, LMC_TYPE_IQ3_S = 21, LMC_TYPE_IQ4_XS = 23 };
/* struct lmc_qtensor as lmc_internal.h lays it out; main() compares the
 * field offsets with qt_layout[], which the test compiles from that header */
typedef struct {
    uint32_t type;
    int rows, cols;
    size_t bytes;
    void *blocks, *tiled;
    size_t tiled_bytes;
    int tiled_rows;
    float gemm_wscale;
} lmc_qtensor;
extern const size_t qt_layout[5];
typedef struct lmc_model lmc_model;
int lmc_model_load(const char *path, int max_batch, int kv_dtype, lmc_model **out);
int lmc_model_load_tp(const char *path, int max_batch, int kv_dtype, int tp_rank, int tp_size, const void *id,
                      lmc_model **out);
int lmc_model_free(lmc_model *m);
int lmc_model_load_paged(const char *path, int max_batch, int max_rows, int kv_dtype, int page_size, int n_pages,
                         int tp_rank, int tp_size, const void *id, lmc_model **out);
int lmc_model_forward(lmc_model *m, const int *h_tokens, const int *h_pos, int batch, float *h_logits, int *h_next);
int lmc_model_release_seq(lmc_model *m, int seq);
int lmc_model_kv_pages(const lmc_model *m, int *page_size, int *n_pages, int *n_free);
int lmc_model_prefill(lmc_model *m, int seq, const int *h_tokens, int n, int start_pos, float *h_logits, int *h_next);
int lmc_model_generate(lmc_model *m, const int *h_prompt, int n_prompt, int batch, int n_new, int use_graph,
                       int *h_out_ids);
int lmc_model_replay(lmc_model *m, int n, void *stream_out);

static char g_err[512];
int lmc_set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}
const char *lmc_last_error(void) { return g_err; }

/* GGUF block geometry (elements, bytes per block) */
int lmc_tensor_bytes(uint32_t type, size_t n, size_t *bytes) {
    static const struct { uint32_t t; int be, bb; } g[] = {
        {LMC_TYPE_F32, 1, 4},      {LMC_TYPE_F16, 1, 2},      {LMC_TYPE_Q4_0, 32, 18},  {LMC_TYPE_Q4_1, 32, 20},
        {LMC_TYPE_Q5_0, 32, 22},   {LMC_TYPE_Q5_1, 32, 24},   {LMC_TYPE_Q8_0, 32, 34},  {LMC_TYPE_Q2_K, 256, 84},
        {LMC_TYPE_Q3_K, 256, 110}, {LMC_TYPE_Q4_K, 256, 144}, {LMC_TYPE_Q5_K, 256, 176}, {LMC_TYPE_Q6_K, 256, 210},
        {LMC_TYPE_IQ3_XXS, 256, 98}, {LMC_TYPE_IQ3_S, 256, 110}, {LMC_TYPE_IQ4_XS, 256, 136}};
    for (size_t i = 0; i < sizeof g / sizeof g[0]; i++)
        if (g[i].t == type) {
            if (n % (size_t)g[i].be) return lmc_set_error(LMC_ERR_INVALID, "not whole blocks");
            *bytes = n / (size_t)g[i].be * (size_t)g[i].bb;
            return LMC_OK;
        }
    return lmc_set_error(LMC_ERR_UNSUPPORTED, "type %u", type);
}

static int g_n;
int lmc_qtensor_upload(uint32_t type, int rows, int cols, const void *h, size_t bytes, lmc_qtensor **out) {
    size_t need;
    int rc = lmc_tensor_bytes(type, (size_t)rows * cols, &need);
    if (rc) return rc;
    if (bytes < need) return lmc_set_error(LMC_ERR_INVALID, "short upload");
    const char *dir = getenv("LMC_FAKE_DUMP");
    if (dir) {
        char p[1024];
        snprintf(p, sizeof p, "%s/%04d.bin", dir, g_n);
        FILE *f = fopen(p, "wb");
        if (!f || fwrite(h, 1, need, f) != need) return lmc_set_error(LMC_ERR_IO, "dump");
        fclose(f);
    }
    printf("Q %d %u %d %d %zu\n", g_n++, type, rows, cols, need);
    lmc_qtensor *t = (lmc_qtensor *)calloc(1, sizeof *t);
    t->type = type;
    t->rows = rows;
    t->cols = cols;
    t->bytes = need;
    t->blocks = malloc(1);
    *out = t;
    return LMC_OK;
}
int lmc_qtensor_free(lmc_qtensor *t) {
    if (t) {
        free(t->blocks);
        free(t);
    }
    return LMC_OK;
}
int lmc_qtensor_concat(const lmc_qtensor *const *parts, int n, lmc_qtensor **out) {
    lmc_qtensor *t = (lmc_qtensor *)calloc(1, sizeof *t);
    *t = *parts[0];
    for (int i = 1; i < n; i++) {
        t->rows += parts[i]->rows;
        t->bytes += parts[i]->bytes;
    }
    t->blocks = malloc(1);
    *out = t;
    return LMC_OK;
}
int lmc_qtensor_has_tiled(const lmc_qtensor *t) { (void)t; return 0; }
int lmc_dequant(uint32_t type, const void *b, size_t n, float *o, void *s) { (void)type; (void)b; (void)n; (void)o; (void)s; return LMC_OK; }
size_t lmc_attention_workspace_bytes(int b, int h, int d, int s) { (void)b; (void)h; (void)d; (void)s; return 1024; }
int lmc_gemm_reserve(int r, int k, void *s) { (void)r; (void)k; (void)s; return LMC_OK; }
size_t lmc_peer_region_bytes(void) { return 1024; }
int lmc_peer_max_floats(void) { return 256; }
unsigned long long lmc_rng_seed(unsigned long long s) { return s; }
void lmc_step_prog_free(void *p) { (void)p; }

/* launches and collectives: never reached while loading.  The empty
 * parameter lists are deliberate: these only have to satisfy the linker for
 * calls the loader makes on other paths, whatever their signatures. */
#define FAIL(name) int name() { return lmc_set_error(LMC_ERR_UNSUPPORTED, #name ": no device here"); }
FAIL(lmc_advance_launch) FAIL(lmc_argmax_keys_launch) FAIL(lmc_attention_rows_launch)
FAIL(lmc_attention_rows_paged_launch) FAIL(lmc_embed_launch) FAIL(lmc_keys_to_ids_launch) FAIL(lmc_layer_norm)
FAIL(lmc_matmul) FAIL(lmc_peer_allreduce) FAIL(lmc_rms_norm) FAIL(lmc_sample_launch) FAIL(lmc_step_prog_build)
FAIL(lmc_step_prog_launch) FAIL(lmc_step_prog_launch_imm) FAIL(lmc_swiglu) FAIL(lmc_tiled_gemv_ex)
FAIL(lmc_qtensor_interleave)

/* CUDA runtime: host memory, no streams */
int cudaMalloc(void **p, size_t n) { *p = calloc(1, n ? n : 1); return *p ? 0 : 2; }
int cudaFree(void *p) { free(p); return 0; }
int cudaMallocHost(void **p, size_t n) { return cudaMalloc(p, n); }
int cudaHostAlloc(void **p, size_t n, unsigned f) { (void)f; return cudaMalloc(p, n); }
int cudaFreeHost(void *p) { free(p); return 0; }
int cudaHostGetDevicePointer(void **d, void *h, unsigned f) { (void)f; *d = h; return 0; }
int cudaMemcpy(void *d, const void *s, size_t n, int kind) {
    memcpy(d, s, n);
    if (kind == 1) printf("M %zu\n", n);
    return 0;
}
int cudaMemcpyAsync(void *d, const void *s, size_t n, int kind, void *st) { (void)st; return cudaMemcpy(d, s, n, kind); }
int cudaMemset(void *p, int v, size_t n) { memset(p, v, n); return 0; }
int cudaMemsetAsync(void *p, int v, size_t n, void *st) { (void)st; return cudaMemset(p, v, n); }
int cudaStreamCreateWithFlags(void **s, unsigned f) { (void)f; *s = (void *)1; return 0; }
int cudaStreamDestroy(void *s) { (void)s; return 0; }
int cudaStreamSynchronize(void *s) { (void)s; return 0; }
int cudaStreamQuery(void *s) { (void)s; return 0; }
int cudaDeviceSynchronize(void) { return 0; }
int cudaGetLastError(void) { return 0; }
const char *cudaGetErrorString(int e) { (void)e; return "no device (host stand-in)"; }
FAIL(cudaGraphDestroy) FAIL(cudaGraphExecDestroy) FAIL(cudaGraphGetNodes) FAIL(cudaGraphInstantiate)
FAIL(cudaGraphLaunch) FAIL(cudaGraphNodeGetType) FAIL(cudaStreamBeginCapture) FAIL(cudaStreamEndCapture)
FAIL(cudaIpcCloseMemHandle) FAIL(cudaIpcGetMemHandle) FAIL(cudaIpcOpenMemHandle)

/* NCCL: a communicator token, nothing exchanged */
typedef struct { char internal[128]; } fake_nccl_id;
int ncclCommInitRank(void **comm, int n, fake_nccl_id id, int rank) {
    (void)n; (void)id; (void)rank;
    *comm = (void *)1;
    return 0;
}
int ncclCommDestroy(void *c) { (void)c; return 0; }
int ncclCommAbort(void *c) { (void)c; return 0; }
int ncclCommGetAsyncError(void *c, int *e) { (void)c; *e = 0; return 0; }
const char *ncclGetErrorString(int r) { (void)r; return "host stand-in"; }
int ncclGetUniqueId(fake_nccl_id *id) { memset(id, 0, sizeof *id); return 0; }
FAIL(ncclAllGather) FAIL(ncclAllReduce)

/* The paged cache's page accounting (argv[3] == "paged"): a model with 2
 * sequences and a pool of 6 pages of 16 positions; each forward takes its
 * pages and then stops at its first kernel launch (there is no device
 * here), so the pool's count shows what it took.  One line per step:
 * "P <rc> <free pages>". */
static void paged_step(lmc_model *m, int rc) {
    int ps = 0, np = 0, nf = -1;
    lmc_model_kv_pages(m, &ps, &np, &nf);
    printf("P %d %d\n", rc, nf);
}
static int paged_scenario(const char *path) {
    lmc_model *m = NULL;
    int rc = lmc_model_load_paged(path, 2, 2, LMC_KV_F16, 16, 6, 0, 1, NULL, &m);
    printf("rc %d %s\n", rc, rc ? lmc_last_error() : "");
    if (rc) return 0;
    const int tok[2] = {1, 2};
    int pos[2] = {0, 0};
    paged_step(m, lmc_model_forward(m, tok, pos, 2, NULL, NULL)); /* one page each: 4 free */
    pos[0] = 39;
    paged_step(m, lmc_model_forward(m, tok, pos, 1, NULL, NULL)); /* sequence 0 up to 3 pages: 2 free */
    paged_step(m, lmc_model_release_seq(m, 0));                   /* 5 free */
    pos[0] = 0;
    pos[1] = 47;
    paged_step(m, lmc_model_forward(m, tok, pos, 2, NULL, NULL)); /* 1 + 2 more: 2 free */
    pos[0] = 40;
    pos[1] = 63;
    paged_step(m, lmc_model_forward(m, tok, pos, 2, NULL, NULL)); /* 2 + 1 wanted, 2 free: refused */
    pos[0] = 31;
    paged_step(m, lmc_model_forward(m, tok, pos, 1, NULL, NULL)); /* 1 more: 1 free */
    paged_step(m, lmc_model_release_seq(m, 1));                   /* 4 free */
    paged_step(m, lmc_model_release_seq(m, 2));                   /* no such sequence */
    lmc_model_free(m);
    return 0;
}

/* Argument checks of the model entry points on a loaded model (argv[3] ==
 * "args"): calls that must be refused before any work, sizes chosen so
 * that a check written as a sum would overflow an int.  One "A <rc>" line
 * per call. */
static int args_scenario(const char *path) {
    lmc_model *m = NULL;
    int rc = lmc_model_load(path, 2, LMC_KV_F16, &m);
    printf("rc %d %s\n", rc, rc ? lmc_last_error() : "");
    if (rc) return 0;
    const int big = 2147483600, tok[2] = {1, 2}, bad_tok[1] = {1 << 30}, pos_ok[2] = {0, 0};
    int pos_bad[1] = {-1}, ids[4];
    printf("A %d\n", lmc_model_forward(m, tok, pos_bad, 1, NULL, NULL));          /* negative position */
    pos_bad[0] = 1 << 30;
    printf("A %d\n", lmc_model_forward(m, tok, pos_bad, 1, NULL, NULL));          /* beyond the context */
    printf("A %d\n", lmc_model_forward(m, bad_tok, pos_ok, 1, NULL, NULL));       /* token beyond V */
    printf("A %d\n", lmc_model_forward(m, tok, pos_ok, 3, NULL, NULL));           /* more rows than sequences */
    printf("A %d\n", lmc_model_prefill(m, 0, tok, 100, big, NULL, NULL));         /* start + n past INT_MAX */
    printf("A %d\n", lmc_model_prefill(m, 2, tok, 2, 0, NULL, NULL));             /* no such sequence */
    printf("A %d\n", lmc_model_generate(m, tok, 2, 1, 2147483647, 1, ids));       /* n_prompt + n_new past INT_MAX */
    printf("A %d\n", lmc_model_generate(m, tok, big, 1, 4, 1, ids));              /* prompt beyond the context */
    printf("A %d\n", lmc_model_replay(m, 1, NULL));                               /* no generation yet */
    lmc_model_free(m);
    return 0;
}

/* Loads argv[1] as shard r of argv[2] ranks for every r, one "R r rc" line
 * each before its uploads' lines. */
int main(int argc, char **argv) {
    if (argc < 3) return 2;
    const size_t mine[5] = {offsetof(lmc_qtensor, rows), offsetof(lmc_qtensor, bytes), offsetof(lmc_qtensor, tiled),
                            offsetof(lmc_qtensor, gemm_wscale), sizeof(lmc_qtensor)};
    if (memcmp(mine, qt_layout, sizeof mine)) {
        fprintf(stderr, "struct lmc_qtensor changed: update the copy in host_shard_fakes.c\n");
        return 3;
    }
    if (argc > 3 && !strcmp(argv[3], "paged")) return paged_scenario(argv[1]);
    if (argc > 3 && !strcmp(argv[3], "args")) return args_scenario(argv[1]);
    const int n = atoi(argv[2]);
    char id[128] = {0};
    for (int r = 0; r < n; r++) {
        printf("R %d\n", r);
        lmc_model *m = NULL;
        const int rc = n > 1 ? lmc_model_load_tp(argv[1], 1, LMC_KV_F16, r, n, id, &m)
                             : lmc_model_load(argv[1], 1, LMC_KV_F16, &m);
        printf("rc %d %s\n", rc, rc ? lmc_last_error() : "");
        if (!rc) lmc_model_free(m);
    }
    return 0;
}
