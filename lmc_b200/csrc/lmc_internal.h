/* lmc_internal.h - declarations shared between the CUDA kernels (.cu) and
 * the C99 host runtime (lmc_b200/host) inside liblmc_b200.so.  Not installed. */
#ifndef LMC_INTERNAL_H
#define LMC_INTERNAL_H

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/lmc_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Zero bytes kept readable after every device block stream: IQ4_XS reads
 * two bytes past its last block (LMc src/quant.c:506,515), and the kernels
 * address F32/F16 tensors in whole 8-element groups (up to 28 bytes past). */
#define LMC_BLOCK_PAD 32

struct lmc_qtensor {
    uint32_t type;
    int rows, cols;
    size_t bytes;      /* raw GGUF block stream size */
    void *blocks;      /* device: raw blocks + LMC_BLOCK_PAD */
    void *tiled;       /* device: row-tiled copy for the tensor-core GEMV, or NULL */
    size_t tiled_bytes;
    int tiled_rows;    /* rows padded to the tile height */
    float gemm_wscale; /* power-of-two prescale of the fp16 weights in the batched GEMM (0: no GEMM) */
};

int lmc_set_error(int code, const char *fmt, ...);
/* Host -> device copy through pinned staging buffers (chunks filled by
 * host threads while the previous chunk's DMA runs); synchronous. */
int lmc_h2d_staged(void *d_dst, const void *h_src, size_t bytes);
int lmc_qtensor_concat(const struct lmc_qtensor *const *parts, int n, struct lmc_qtensor **out);
/* Row tiles of a and b interleaved (a tile, b tile, a tile, ...); tiled copy built. */
int lmc_qtensor_interleave(const struct lmc_qtensor *a, const struct lmc_qtensor *b, int tile_rows,
                           struct lmc_qtensor **out);
/* Persistent step GEMV epilogue: the row tiles come in (gate, up) pairs
 * (lmc_qtensor_interleave with 16-row tiles) and y = silu(gate) * up, one
 * output row per row of a pair (src/ops_llama.c:150-151). */
#define LMC_EPI_GLU_PAIRS 16
int lmc_tensor_bytes(uint32_t type, size_t n_elements, size_t *bytes);
int lmc_sm_count(void);

int lmc_gemv_generic_launch(uint32_t type, const void *d_blocks, int M, int K, const float *d_x, int ldx,
                            const float *d_bias, float *d_y, int ldy, int batch, int epi, cudaStream_t s);
/* Builds t->tiled when the type/shape has a tensor-core GEMV (else leaves it NULL). */
int lmc_tiled_build(struct lmc_qtensor *t);
int lmc_tiled_gemv_launch(const struct lmc_qtensor *t, const float *d_x, int ldx, const float *d_bias, float *d_y,
                          int ldy, int batch, int epi, cudaStream_t s);
/* Fused work around a tensor-core GEMV (tiled tensors only): a prologue op
 * applied to x as it is loaded, and a greedy-argmax epilogue. */
#define LMC_PRO_NONE 0
#define LMC_PRO_LAYERNORM 1 /* (x - mean) * rstd * w + b, eps 1e-5 (src/ops.c:47-59) */
#define LMC_PRO_RMSNORM 2   /* w * rs * x (src/ops_llama.c:24-33) */
#define LMC_PRO_SWIGLU 3    /* silu(x) * x2 (src/ops_llama.c:150-151) */
typedef struct {
    int pro;
    const float *w, *b, *x2;
    float eps;
    unsigned long long *keys; /* non-NULL: atomicMax of lmc_argmax_key(y, row + key_base) per batch row */
    int key_base;             /* global index of row 0 (a vocabulary shard of the lm_head) */
} lmc_gemv_extra;
int lmc_tiled_gemv_ex(const struct lmc_qtensor *t, const float *d_x, int ldx, const float *d_bias, float *d_y, int ldy,
                      int batch, int epi, const lmc_gemv_extra *ex, cudaStream_t s);
/* The latency (fp32) GEMV for short matrices at batch <= 2 (ff_gemv.cu);
 * LMC_ERR_UNSUPPORTED when the shape does not suit it. */
int lmc_ff_gemv_launch(const struct lmc_qtensor *t, const float *d_x, int ldx, const float *d_bias, float *d_y,
                       int ldy, int batch, int epi, const lmc_gemv_extra *ex, cudaStream_t s);
int lmc_ff_gemv_suits(const struct lmc_qtensor *t, int batch, int epi);
/* Batched GEMM on the tcgen05 tensor cores (batch widths > 8; gemm_tc.cu).
 * lmc_gemm_prepare sets t->gemm_wscale (needs cols % 64 == 0);
 * lmc_gemm_reserve sizes the activation workspace (call before any capture);
 * lmc_gemm_launch applies the prologue of `ex` (may be NULL) and the epilogue. */
int lmc_gemm_prepare(struct lmc_qtensor *t);
int lmc_gemm_reserve(int N, int K, cudaStream_t s);
int lmc_gemm_launch(const struct lmc_qtensor *t, const float *d_x, int ldx, const float *d_bias, float *d_y, int ldy,
                    int N, int epi, const lmc_gemv_extra *ex, cudaStream_t s);
int lmc_gemm_status(void);
/* Argmax over keys: reads each batch row's key (written by the fused
 * epilogue or by lmc_argmax_keys_launch), stores the row index in d_next and
 * resets the key to 0 for the next step. */
int lmc_argmax_keys_launch(const float *d_x, int n, int rows, unsigned long long *d_keys, cudaStream_t s);
int lmc_keys_to_ids_launch(unsigned long long *d_keys, int *d_next, int batch, cudaStream_t s);
int lmc_embed_launch(uint32_t type, const void *wte, const float *wpe, const int *d_tok, const int *d_pos, int D,
                     int V, int S, int batch, float *out, cudaStream_t s);
/* RoPE on `batch` rows (row stride ld floats) of n_heads x Dh, each at its
 * own position d_pos[b], from [S][Dh/2] cos/sin tables. */
int lmc_rope_pos_launch(float *v, int ld, int n_heads, int Dh, const float *cos_tab, const float *sin_tab,
                        const int *d_pos, int S, int batch, cudaStream_t s);
/* Attention with explicit row strides for q/out (ldq) and k_new/v_new (ldkv).
 * d_cnt: [batch][Hkv] arrival counters, zero before the first call, or NULL.
 * With counters the last split CTA of each (sequence, kv head) merges the
 * splits in the same launch (no separate combine kernel). */
int lmc_attention_launch(float *out, int ldo, const float *q, int ldq, const float *k_new, const float *v_new,
                         int ldkv, void *k_cache, void *v_cache, int kv_dtype, const int *d_pos, int batch, int H,
                         int Hkv, int Dh, int S, void *d_ws, size_t ws_bytes, int *d_cnt, cudaStream_t s);
/* Same, applying RoPE (src/ops_llama.c:39-48,75-78) from [S][Dh/2] tables to
 * q and to the new K row on the fly (no separate rope launch). */
int lmc_attention_rope_launch(float *out, int ldo, const float *q, int ldq, const float *k_new, const float *v_new,
                              int ldkv, void *k_cache, void *v_cache, int kv_dtype, const int *d_pos, int batch, int H,
                              int Hkv, int Dh, int S, void *d_ws, size_t ws_bytes, const float *rope_cos,
                              const float *rope_sin, int *d_cnt, cudaStream_t s);
/* As lmc_attention_rope_launch, with d_seq[b] the cache sequence of row b
 * (NULL: row b uses sequence b).  Rows may share a sequence (a prompt chunk,
 * one position per row): their K/V rows are appended by a separate kernel
 * first, so row b attends to every row of the chunk at positions <= pos[b]. */
int lmc_attention_rows_launch(float *out, int ldo, const float *q, int ldq, const float *k_new, const float *v_new,
                              int ldkv, void *k_cache, void *v_cache, int kv_dtype, const int *d_pos, const int *d_seq,
                              int batch, int H, int Hkv, int Dh, int S, void *d_ws, size_t ws_bytes,
                              const float *rope_cos, const float *rope_sin, int *d_cnt, cudaStream_t s);
/* lmc_attention_rows_launch over a paged cache: k_pool / v_pool are pools of
 * n_pages pages [page][Hkv][2^page_shift positions][row], and position t of
 * cache sequence s lives in page d_pages[s * max_pages + (t >> page_shift)]
 * (the context is max_pages << page_shift positions). */
int lmc_attention_rows_paged_launch(float *out, int ldo, const float *q, int ldq, const float *k_new,
                                    const float *v_new, int ldkv, void *k_pool, void *v_pool, int kv_dtype,
                                    const int *d_pos, const int *d_seq, int batch, int H, int Hkv, int Dh,
                                    const int *d_pages, int max_pages, int page_shift, int n_pages, void *d_ws,
                                    size_t ws_bytes, const float *rope_cos, const float *rope_sin, int *d_cnt,
                                    cudaStream_t s);
/* Generation bookkeeping after one step (see lmc_model_generate): the greedy
 * id of each sequence is read from (and reset in) d_keys, or, with
 * from_next, the pick is the one already in d_next (a sampler wrote it; the
 * keys are still reset). */
int lmc_advance_launch(unsigned long long *d_keys, int *d_next, int *d_tok, int *d_pos, int *d_step,
                       const int *d_prompt, int n_prompt, int *d_ids, int n_new, int batch, int from_next,
                       cudaStream_t s);
/* lmc_sample_top_p on rows of ld floats (ld must equal n) on stream s; with
 * d_step, only in steps whose pick is a generated token (step + 1 >= n_prompt). */
int lmc_sample_launch(const float *d_logits, int n, int ld, int rows, float temperature, float top_p,
                      unsigned long long *d_rng, int *d_idx, const int *d_step, int n_prompt, cudaStream_t s);
/* Split plan of the decode attention (attention.cu): positions per split
 * and split count for context S and bh = batch x heads; fine = the splits
 * are merged inside the launch (arrival counters). */
void lmc_attn_plan(int S, int bh, int fine, int *CH, int *nsplit);
/* LMC_OK, or LMC_ERR_INVALID once after a paged attention met a page id
 * outside its pool. */
int lmc_attn_status(void);

/* Tensor-parallel sums over peer memory (peer_allreduce.cu): every rank
 * allocates one region of lmc_peer_region_bytes() (zeroed) and maps every
 * peer's (CUDA IPC); bases[p] = rank p's region as seen by this rank.  Sums
 * of at most lmc_peer_max_floats() floats (a multiple of 4), collective:
 * every rank calls it with the same n in the same order. */
#define LMC_PEER_MAX 8
size_t lmc_peer_region_bytes(void);
int lmc_peer_max_floats(void);
int lmc_peer_allreduce(float *d_x, int n, int rank, int size, void *const *bases, cudaStream_t s);
int lmc_peer_status(void);
int lmc_peer_set_wait_limit(long long ns);

/* ---- persistent decode step (step_kernel.cu) -------------------------------
 * A whole decode step as ONE cooperative launch: every CTA walks the same list
 * of ops (embedding, tensor-core GEMVs with their prologue/epilogue, attention,
 * greedy bookkeeping) and the CTAs meet at a grid-wide barrier (a counter in
 * device memory, bounded wait) after each op instead of at a kernel boundary.
 * While a CTA waits, the weights of its share of the next GEMV are already
 * being copied into its shared memory. */
#define LMC_OP_EMBED 1   /* x[b] = wte[tok[b]] (+ wpe[pos[b]])                     */
#define LMC_OP_GEMV 2    /* tiled qtensor, batch <= 2, prologue + epilogue of ex      */
#define LMC_OP_ATTN 3    /* decode attention, K/V append, optional RoPE, merge      */
#define LMC_OP_KEYS 4    /* next[b] = greedy key index, keys reset (model_forward)  */
#define LMC_OP_ADVANCE 5 /* the generate() bookkeeping of lmc_advance_launch         */
#define LMC_OP_SAMPLE 6  /* top-p draw per row into next (lmc_sample_launch)      */
typedef struct {
    int kind, batch;
    /* GEMV */
    const struct lmc_qtensor *w;
    const float *x, *bias;
    float *y;
    int ldx, ldy, epi;
    lmc_gemv_extra ex;
    /* ATTN */
    float *out;
    const float *q, *k_new, *v_new;
    int ldo, ldq, ldkv;
    void *k_cache, *v_cache;
    int kv_dtype, H, Hkv, Dh, S;
    const float *rope_cos, *rope_sin;
    void *ws;
    size_t ws_bytes;
    int *cnt;
    /* EMBED (tok, pos), ATTN (pos), KEYS / ADVANCE */
    uint32_t wte_type;
    const void *wte;
    const float *wpe;
    int D, V;
    int *tok, *pos;
    unsigned long long *keys;
    int *next, *step, *ids;
    int *next_host; /* KEYS: picks also written to this mapped host memory (NULL: none) */
    const int *prompt;
    int n_prompt, n_new;
    /* SAMPLE (logits in y, V, rng, next, step, n_prompt); ADVANCE: from_next */
    float temperature, top_p;
    unsigned long long *rng;
    int from_next;
    /* norm statistics passed from the op that writes x to the norm that reads
     * it: slot number + 1 (0 = none).  stats_out on EMBED and on GEMVs that
     * add into the residual; stats_in on GEMVs with a LayerNorm/RMSNorm
     * prologue (which then skip their own statistics passes). */
    int stats_in, stats_out;
} lmc_step_op;
typedef struct lmc_step_prog lmc_step_prog;
/* LMC_ERR_UNSUPPORTED when an op cannot run inside the persistent kernel
 * (the caller then launches the step kernel by kernel). */
int lmc_step_prog_build(const lmc_step_op *ops, int n, lmc_step_prog **out);
int lmc_step_prog_launch(const lmc_step_prog *p, cudaStream_t s);
/* The same, with this step's tokens and positions passed in the launch
 * (no host -> device copies): the kernel stores them to d_tok / d_pos. */
int lmc_step_prog_launch_imm(const lmc_step_prog *p, cudaStream_t s, const int *h_tok, const int *h_pos, int nb,
                             int *d_tok, int *d_pos);
void lmc_step_prog_free(lmc_step_prog *p);
/* LMC_OK, or LMC_ERR_TIMEOUT once after a persistent step gave up a bounded
 * wait (its barrier state is then reset for the next launch). */
int lmc_step_status(void);
/* Wait limit of the bounded device waits of the GEMV rings and of the
 * persistent step's barriers (nanoseconds; 0 restores the default). */
int lmc_tiled_set_wait_limit(long long ns);
int lmc_step_set_wait_limit(long long ns);
int lmc_gemm_set_wait_limit(long long ns);
/* Self-tests of the bounded waits: a wait on an mbarrier that nothing
 * completes (the GEMV's wait; *d_flag = 1 when it gave up), and a grid
 * barrier that can never complete (LMC_ERR_TIMEOUT when every CTA left). */
int lmc_tiled_wait_selftest(int *d_flag, cudaStream_t s);
int lmc_step_barrier_selftest(int *d_left, cudaStream_t s);

#ifdef __cplusplus
}
#endif
#endif /* LMC_INTERNAL_H */
