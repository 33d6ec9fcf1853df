/* lmc_cuda.h - C ABI of the B200-native LMc hot path (liblmc_b200.so).
 *
 * Plain C99 declarations: pointers, sizes and status codes; no CUDA, C++ or
 * PyTorch types.  Device pointers are marked d_*, host pointers h_*; a
 * `stream` argument is a cudaStream_t passed as void* (NULL = the legacy
 * default stream).  Every entry point returns LMC_OK (0) or a negative
 * LMC_ERR_* code and records a message for lmc_last_error(); none of them
 * falls back to the CPU - without a usable sm_100 device they fail.
 *
 * Each entry point names the LMc interface (nile-agi/LMc, file:line) whose
 * behaviour it replaces.  LMc reports hard errors through LMC_FATAL
 * (src/utils.h:68-69, exit(1)); this ABI returns the status instead and the
 * C99 drop-in layer (include/lmc_ops.h) maps a failure back to LMC_FATAL.
 */
#ifndef LMC_CUDA_H
#define LMC_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define LMC_OK               0
#define LMC_ERR_INVALID     -1   /* bad argument (null pointer, bad size/shape) */
#define LMC_ERR_UNSUPPORTED -2   /* tensor type or shape not handled            */
#define LMC_ERR_CUDA        -3   /* CUDA runtime error                          */
#define LMC_ERR_OOM         -4   /* device or host allocation failed            */
#define LMC_ERR_IO          -5   /* file missing, short read, bad GGUF          */
#define LMC_ERR_TIMEOUT     -6   /* a bounded wait ran out                      */
#define LMC_ERR_NCCL        -7   /* NCCL error                                  */

/* GGUF tensor type IDs (src/quant.h:27-45). */
#define LMC_TYPE_F32      0
#define LMC_TYPE_F16      1
#define LMC_TYPE_Q4_0     2
#define LMC_TYPE_Q4_1     3
#define LMC_TYPE_Q5_0     6
#define LMC_TYPE_Q5_1     7
#define LMC_TYPE_Q8_0     8
#define LMC_TYPE_Q2_K    10
#define LMC_TYPE_Q3_K    11
#define LMC_TYPE_Q4_K    12
#define LMC_TYPE_Q5_K    13
#define LMC_TYPE_Q6_K    14
#define LMC_TYPE_IQ3_XXS 18
#define LMC_TYPE_IQ3_S   21
#define LMC_TYPE_IQ4_XS  23

/* Message for the last failing call on this host thread ("" if none). */
const char *lmc_last_error(void);

/* LMC_OK, or LMC_ERR_TIMEOUT (once; the flag is then cleared) when a kernel
 * of this library gave up one of its bounded waits on the device - every
 * spin-wait in the kernels has an iteration limit instead of hanging. */
int lmc_device_status(void);

/* Limit of every bounded wait inside the kernels - the bulk-copy rings of
 * the GEMV and GEMM, the grid barriers of the persistent decode step - in
 * nanoseconds; 0 restores the default of one second.  A wait that runs out
 * records a timeout that lmc_device_status reports; the kernel drains its
 * own copies and returns, and the context stays usable.  No counterpart in
 * LMc (a CPU program has no device waits). */
int lmc_set_wait_limit(long long ns);
/* Self-test of that failure path: runs a device wait that nothing can
 * complete - which = 0: a GEMV ring's mbarrier wait, 1: a persistent-step
 * grid barrier (two CTAs) - under the current limit.  Returns LMC_ERR_TIMEOUT
 * when the wait ran out as designed (and clears the recorded timeout). */
int lmc_wait_selftest(int which);

/* Select and initialise CUDA device `device` for the calling thread.
 * Fails with LMC_ERR_CUDA when no sm_100 device is present. */
int lmc_init(int device);

/* Number of elements and bytes of one block of `type`
 * (replaces the *_BLOCK_SIZE / *_BYTES_PER_BLOCK constants, src/quant.h:54-99). */
int lmc_block_geometry(uint32_t type, int *block_elems, int *block_bytes);

/* ---- K1: block dequantization ------------------------------------------------
 * Replaces dequant_q4_0 ... dequant_iq4_xs (src/quant.c:178-521) and the
 * F32/F16 cases of the loader switch (src/gguf.c:316-345).  Decodes
 * n_elements weights from the flat block stream d_blocks into d_out (fp32),
 * bit-exact to LMc.  n_elements must be a multiple of the block size.
 * d_blocks must hold (n_elements / block) * block_bytes bytes, plus 2
 * readable bytes for IQ4_XS (LMc reads 2 bytes of the next block,
 * src/quant.c:506,515). */
int lmc_dequant(uint32_t type, const void *d_blocks, size_t n_elements,
                float *d_out, void *stream);

/* ---- quantized tensors on the device ---------------------------------------
 * LMc dequantizes every tensor to fp32 at load time and frees the raw bytes
 * (LOAD_QUANT, src/gguf.c:100-111).  A qtensor keeps the raw GGUF blocks on
 * the device instead and, for the formats with a tensor-core GEMV, a
 * row-tiled copy of the same bytes rearranged for it.  A tensor is `rows`
 * rows of `cols` weights stored as one flat block stream (blocks may
 * straddle rows when cols is not a multiple of the block size, as in LMc). */
typedef struct lmc_qtensor lmc_qtensor;

int lmc_qtensor_upload(uint32_t type, int rows, int cols, const void *h_blocks,
                       size_t bytes, lmc_qtensor **out);
int lmc_qtensor_free(lmc_qtensor *t);
/* Device pointer to the raw GGUF block stream (read-only view). */
const void *lmc_qtensor_blocks(const lmc_qtensor *t);
/* Type and shape of a qtensor (any output pointer may be NULL). */
int lmc_qtensor_shape(const lmc_qtensor *t, uint32_t *type, int *rows, int *cols);
/* 1 when the tensor-core GEMV layout was built for this tensor. */
int lmc_qtensor_has_tiled(const lmc_qtensor *t);

/* ---- K2: quantized matrix-vector products ------------------------------------
 * Replaces matmul_vec (src/ops.c:69-97): for each of `batch` input vectors,
 *   y[b][m] = bias[m] + sum_k W[m][k] * x[b][k]   (fp32 accumulation)
 * x is batch rows of ldx floats, y batch rows of ldy floats; bias may be
 * NULL.  `epilogue` is a bit set:
 *   LMC_EPI_GELU  apply gelu (src/ops.c:20-24) to the result,
 *   LMC_EPI_ACCUM add the result into y instead of overwriting it (the
 *                 residual adds of src/ops.c:198,205).
 * lmc_matmul uses the fastest layout the qtensor carries; lmc_matmul_blocks
 * runs the generic kernel straight on a raw block stream. */
#define LMC_EPI_NONE  0
#define LMC_EPI_GELU  1
#define LMC_EPI_ACCUM 2
int lmc_matmul(const lmc_qtensor *w, const float *d_x, int ldx, const float *d_bias,
               float *d_y, int ldy, int batch, int epilogue, void *stream);
/* Which kernel lmc_matmul runs for this tensor, batch width and epilogue
 * (a static string, for reports): the latency GEMV (short matrices, batch
 * <= 2), the tensor-core GEMV (tiled Q4_K / Q6_K / Q8_0), the tcgen05 GEMM
 * (batch > 8) or the generic GEMV. */
const char *lmc_matmul_kernel(const lmc_qtensor *w, int batch, int epilogue);
int lmc_matmul_blocks(uint32_t type, const void *d_blocks, int rows, int cols,
                      const float *d_x, int ldx, const float *d_bias, float *d_y,
                      int ldy, int batch, int epilogue, void *stream);

/* ---- device buffers ------------------------------------------------------------
 * Plain device memory for callers without CUDA headers (the ops.h drop-in
 * layer keeps its scratch and KV-cache mirrors in these).  No counterpart in
 * LMc, whose buffers are host arrays (src/models.c:122-164).  lmc_copy
 * direction: LMC_H2D, LMC_D2H or LMC_D2D; it is ordered on `stream` and
 * returns once the copy is enqueued (host memory must stay valid until
 * lmc_stream_sync). */
#define LMC_H2D 0
#define LMC_D2H 1
#define LMC_D2D 2
int lmc_buffer_alloc(size_t bytes, void **d_out);
int lmc_buffer_free(void *d);
int lmc_copy(void *dst, const void *src, size_t bytes, int direction, void *stream);
int lmc_stream_sync(void *stream);

/* ---- small ops kept on the device --------------------------------------------
 * Each processes `rows` independent rows. */
/* layer_norm (src/ops.c:47-59), eps fixed at 1e-5 as in LMc. */
int lmc_layer_norm(float *d_out, const float *d_x, const float *d_w, const float *d_b,
                   int dim, int rows, void *stream);
/* rms_norm (src/ops_llama.c:24-33). */
int lmc_rms_norm(float *d_out, const float *d_x, const float *d_w, int dim, int rows,
                 float eps, void *stream);
/* softmax in place (src/ops.c:32-44), uniform when the exp-sum < 1e-30. */
int lmc_softmax(float *d_x, int n, int rows, void *stream);
/* gelu / silu in place (src/ops.c:20-29). */
int lmc_gelu(float *d_x, size_t n, void *stream);
int lmc_silu(float *d_x, size_t n, void *stream);
/* d_gate[i] = silu(d_gate[i]) * d_up[i] (src/ops_llama.c:150-151). */
int lmc_swiglu(float *d_gate, const float *d_up, size_t n, void *stream);
/* rope_apply (src/ops_llama.c:39-48) on n_heads consecutive head vectors. */
int lmc_rope_apply(float *d_vec, const float *d_cos_row, const float *d_sin_row,
                   int head_dim, int n_heads, void *stream);
/* Greedy pick (src/lmc.c:45-47): first index of the maximum of each row. */
int lmc_argmax(const float *d_x, int n, int rows, int *d_idx, void *stream);
/* Top-p (nucleus) sampling with temperature, sample_top_p (src/lmc.c:42-59),
 * for `rows` rows of n logits (read only; LMc scales its logits in place):
 * below temperature 1e-6 the greedy pick, else softmax(logits / temperature),
 * the shortest run of the most probable tokens whose probability reaches
 * top_p, and a draw r from the row's xorshift64 state d_rng[row]
 * (src/lmc.c:31-33, advanced once per draw) picks the first token of that
 * run, in descending order, whose running probability passes r.  Tokens of
 * exactly equal probability are taken in index order (LMc leaves their order
 * to qsort).  d_idx[row] receives the token. */
int lmc_sample_top_p(const float *d_logits, int n, int rows, float temperature, float top_p,
                     unsigned long long *d_rng, int *d_idx, void *stream);
/* The xorshift64 state LMc's rng_seed makes from a seed (src/lmc.c:30-31). */
unsigned long long lmc_rng_seed(unsigned long long seed);

/* ---- K4: attention over the head-major KV cache -------------------------------
 * Replaces the cache write and per-head read of attention_forward
 * (src/ops.c:122-178) and llama_attention_forward (src/ops_llama.c:80-134).
 * Cache layout per layer: [Hkv][S][row] (src/models.h:149-162), a row being
 * Dh fp32 values (LMC_KV_F32, LMc's layout), Dh fp16 values (LMC_KV_F16), or
 * Dh int8 codes followed by a 16-byte tail whose first 4 bytes hold the
 * row's fp32 scale (LMC_KV_Q8: value = code * scale; a new row is quantized
 * with m = max|x|, code = clamp(rint(x * (127 / m)), +-127), scale = m / 127;
 * Dh + 16 bytes per row, head sizes that are multiples of 16 up to 512;
 * LMC_KV_ROW_BYTES gives the row size).  For `batch` sequences
 * the caches are batch consecutive [Hkv][S][Dh] slabs and q/k_new/v_new/out
 * are batch rows of H*Dh (q, out) and Hkv*Dh (k_new, v_new) floats.
 * d_pos[b] is the position written this step; positions 0..d_pos[b] are
 * attended.  Query head h reads kv head h / (H / Hkv) (src/ops_llama.c:95).
 * Like LMc's caller-supplied scores_buf, the scratch for the split-context
 * partial results is supplied by the caller: d_workspace must hold
 * lmc_attention_workspace_bytes(batch, H, Dh, S) bytes (0 = none needed). */
#define LMC_KV_F32 0
#define LMC_KV_F16 1
#define LMC_KV_Q8 2
#define LMC_KV_ROW_BYTES(kv_dtype, Dh) \
    ((kv_dtype) == LMC_KV_F32 ? 4 * (size_t)(Dh) : (kv_dtype) == LMC_KV_F16 ? 2 * (size_t)(Dh) : (size_t)(Dh) + 16)
size_t lmc_attention_workspace_bytes(int batch, int H, int Dh, int S);
int lmc_attention_decode(float *d_out, const float *d_q, const float *d_k_new,
                         const float *d_v_new, void *d_k_cache, void *d_v_cache,
                         int kv_dtype, const int *d_pos, int batch, int H, int Hkv,
                         int Dh, int S, void *d_workspace, size_t workspace_bytes,
                         void *stream);
/* lmc_attention_decode without a workspace, for callers that cannot
 * allocate device memory where they decode (inside CUDA-graph capture,
 * loops that must not let cudaMalloc/cudaFree synchronize the device, hosts
 * that own every device allocation).  No counterpart in LMc: it is an
 * addition of this library.  The split-context scratch is a fixed 4 MiB
 * array compiled into liblmc_b200.so (held by every GPU that loads the
 * library until exit); shapes whose lmc_attention_workspace_bytes exceed it
 * are rejected with LMC_ERR_INVALID.  The first call on each device looks up
 * the array's device address (cudaGetSymbolAddress), so make that first call
 * before any stream capture; the address is kept for the life of the
 * process, so cudaDeviceReset after that first call is not supported.  The
 * call allocates nothing.  All calls on a device share the one array, which
 * keeps the last call's contents: calls that may overlap on the GPU
 * (different streams without ordering) race. */
int lmc_attention_decode_noalloc(float *d_out, const float *d_q, const float *d_k_new,
                                 const float *d_v_new, void *d_k_cache, void *d_v_cache,
                                 int kv_dtype, const int *d_pos, int batch, int H, int Hkv,
                                 int Dh, int S, void *stream);
/* lmc_attention_decode over a paged cache, for servers that keep many
 * sequences of different lengths in one pool (LMc's cache is one contiguous
 * [Hkv][S][Dh] slab per layer, src/models.h:149-162; paging is an addition
 * of this library).  d_k_pool / d_v_pool hold n_pages pages; page p is
 * [Hkv][page_size][row] (rows as in lmc_attention_decode, kv_dtype any of
 * LMC_KV_*) and holds page_size consecutive positions of one sequence.
 * d_pages[b * max_pages + j] is the page of positions
 * [j * page_size, (j + 1) * page_size) of sequence b; page_size is a power of
 * two >= 16 and the context limit is max_pages * page_size.  The new K/V row
 * is written at d_pos[b] through the table, so the page of that position
 * must be assigned before the call.  A page id outside [0, n_pages) is not
 * read (page 0 is) and lmc_device_status() then reports LMC_ERR_INVALID.
 * d_workspace: lmc_attention_workspace_bytes(batch, H, Dh, max_pages *
 * page_size) bytes. */
int lmc_attention_decode_paged(float *d_out, const float *d_q, const float *d_k_new,
                               const float *d_v_new, void *d_k_pool, void *d_v_pool,
                               int kv_dtype, int n_pages, const int *d_pages, int max_pages,
                               int page_size, const int *d_pos, int batch, int H, int Hkv,
                               int Dh, void *d_workspace, size_t workspace_bytes,
                               void *stream);

/* ---- whole model: load_model + model_forward on the device -------------------
 * lmc_model_load parses a GGUF v1-3 file the way load_model does
 * (src/gguf.c:114-353, src/models.c:52-164) but uploads the raw blocks
 * instead of dequantizing them, allocates the KV cache and activations on
 * the device, and precomputes the RoPE table with LMc's formula
 * (src/models.c:101-117).  max_batch sequences can be decoded together. */
typedef struct lmc_model lmc_model;
typedef struct {
    int arch;        /* 1 = GPT-2, 2 = LLaMA (src/models.h:28-32) */
    int vocab_size, seq_len, n_layers, n_heads, n_kv_heads, embed_dim, ffn_dim, head_dim;
    float rope_theta, norm_eps;
} lmc_model_config;

int lmc_model_load(const char *gguf_path, int max_batch, int kv_dtype, lmc_model **out);
/* Tensor-parallel shard tp_rank of tp_size (LLaMA; one process per GPU, the
 * caller selects the device first).  No counterpart in LMc, which runs on
 * one CPU: q/k/v rows by heads (attention local to a rank), ffn gate/up rows
 * and the lm_head vocabulary split by rows, attn_output and ffn_down split by
 * columns; each layer sums the ranks' partial residual with one NCCL
 * all-reduce after attn_output and one after ffn_down (NVLink), and the
 * greedy pick is an all-reduce max of 64-bit (logit, index) keys.  nccl_id:
 * 128 bytes from lmc_nccl_unique_id on one rank, given to all.  Every rank
 * makes the same calls (forward / generate) in the same order.  h_logits of
 * lmc_model_forward then receives batch x vocab_rows (this rank's slice,
 * lmc_model_shard). */
int lmc_nccl_unique_id(void *nccl_id_128);
int lmc_model_load_tp(const char *gguf_path, int max_batch, int kv_dtype, int tp_rank, int tp_size,
                      const void *nccl_id_128, lmc_model **out);
/* lmc_model_load / lmc_model_load_tp with max_rows >= max_batch rows per
 * step: the prompt chunk length of lmc_model_prefill (the KV cache still
 * holds max_batch sequences; activations are sized for max_rows rows).
 * tp_size 1 (nccl_id NULL) loads the whole model. */
int lmc_model_load_ex(const char *gguf_path, int max_batch, int max_rows, int kv_dtype, int tp_rank, int tp_size,
                      const void *nccl_id_128, lmc_model **out);
/* lmc_model_load_ex with a paged KV cache, for servers whose sequences are
 * of very different lengths.  No counterpart in LMc, whose cache is one
 * [Hkv][S][Dh] array per layer (src/models.h:149-162).  Each layer's cache
 * is a pool of n_pages pages of page_size positions (a power of two in
 * [16, 65536] that divides the context; n_pages above max_batch x
 * context / page_size is lowered to that), so max_batch sequences share
 * n_pages x page_size positions instead of holding the whole context each.
 * A sequence takes pages from the pool as its positions grow: forward,
 * prefill, generate and replay take the pages their steps write before the
 * steps run, and fail with LMC_ERR_OOM (nothing taken) when the pool has
 * too few free.  lmc_model_release_seq gives sequence seq's pages back (its
 * cached rows are gone: start it again at position 0).  The results are the
 * same as with the contiguous cache (such models always run the step
 * kernel by kernel, not as the persistent single-launch step). */
int lmc_model_load_paged(const char *gguf_path, int max_batch, int max_rows, int kv_dtype, int page_size,
                         int n_pages, int tp_rank, int tp_size, const void *nccl_id_128, lmc_model **out);
int lmc_model_release_seq(lmc_model *m, int seq);
/* Page size (0: contiguous cache), pages in the pool and pages free. */
int lmc_model_kv_pages(const lmc_model *m, int *page_size, int *n_pages, int *n_free);
int lmc_model_shard(const lmc_model *m, int *tp_rank, int *tp_size, int *vocab_begin, int *vocab_rows);
int lmc_model_get_config(const lmc_model *m, lmc_model_config *cfg);
int lmc_model_free(lmc_model *m);
/* model_forward (src/ops.c:212-237, src/ops_llama.c:157-192) for `batch`
 * sequences at once: h_tokens[b] at position h_pos[b].  Writes the next
 * greedy id of each sequence to h_next (may be NULL) and, when h_logits is
 * not NULL, the batch x vocab logits. */
int lmc_model_forward(lmc_model *m, const int *h_tokens, const int *h_pos, int batch,
                      float *h_logits, int *h_next);
/* Batched prefill of one sequence's prompt: the n tokens h_tokens at
 * positions start_pos .. start_pos + n - 1 of sequence `seq` run as the rows
 * of one step, max_rows positions at a time (the projections become GEMMs
 * over the chunk; each row attends to positions <= its own, including the
 * chunk's earlier rows).  Replaces LMc's token-by-token prompt feed
 * (src/lmc.c:109-112), which is what lmc_model_generate does: the KV cache of
 * `seq` and the logits of the last position come out the same (within
 * floating-point rounding).  Writes the next greedy id to h_next and, when
 * h_logits is not NULL, the last position's logits (vocab rows of this
 * rank).  Continue with lmc_model_forward at position start_pos + n. */
int lmc_model_prefill(lmc_model *m, int seq, const int *h_tokens, int n, int start_pos, float *h_logits,
                      int *h_next);
/* The generate() loop of src/lmc.c:108-132 without tokenizer or EOS, run
 * entirely on the device: the n_prompt prompt tokens of each sequence are
 * fed one position at a time, then n_new greedy steps; h_out_ids receives
 * batch x n_new ids.  With use_graph = 1 every step is one CUDA-graph
 * launch and the host does not wait between steps.  A model loaded with
 * more rows than sequences (lmc_model_load_ex) prefills all but the last
 * prompt token of each sequence in chunks first (lmc_model_prefill) and
 * starts the step loop at the last prompt position: the same ids. */
int lmc_model_generate(lmc_model *m, const int *h_prompt, int n_prompt, int batch,
                       int n_new, int use_graph, int *h_out_ids);
/* lmc_model_generate with LMc's top-p sampling (src/lmc.c:42-59,123)
 * instead of the greedy pick: each generated token is drawn on the device by
 * lmc_sample_top_p from the step's logits (temperature below 1e-6: greedy).
 * Sequence b draws from its own xorshift64 stream, seeded as LMc seeds its
 * one stream (src/lmc.c:30-31) with seed + b, so sequence 0 with `seed`
 * follows LMc's stream; the prompt steps draw nothing.  Needs the whole
 * vocabulary on this GPU (not a tensor-parallel shard). */
int lmc_model_generate_sample(lmc_model *m, const int *h_prompt, int n_prompt, int batch, int n_new,
                              float temperature, float top_p, unsigned long long seed, int use_graph,
                              int *h_out_ids);
/* Runs `n` more steps of the last lmc_model_generate (replaying its CUDA
 * graph, or launching the kernels directly when it ran without one),
 * continuing from the current device-side positions (a timing helper:
 * positions must stay below seq_len).  Enqueues only; the stream the steps
 * run on is written to *stream_out when it is not NULL. */
int lmc_model_replay(lmc_model *m, int n, void *stream_out);
/* Kernel launches in one captured step (graph kernel nodes), -1 if none. */
int lmc_model_graph_kernels(const lmc_model *m);
/* Device-side buffers of the model, for callers that drive steps themselves:
 * which = 0 logits [max_batch][V] fp32. */
void *lmc_model_device_buffer(lmc_model *m, int which);
/* The model's weights on the device, by LMc's names (LayerWeights and
 * ModelWeights, src/models.h:79-150), for callers that run single ops on them
 * (the ops.h drop-in layer, include/lmc_ops.h, resolves LMc's weight
 * pointers through these).  No counterpart in LMc, whose weights are fp32
 * host arrays.  Matrices are qtensors; vectors are device fp32 arrays of
 * *len floats.  `layer` is ignored for the whole-model tensors.  NULL when
 * the model has no such tensor (the other architecture's, or out of range). */
#define LMC_W_TOKEN_EMBD 0  /* wte            [V][D]    */
#define LMC_W_OUTPUT     1  /* lm_head        [V][D]    */
#define LMC_W_QKV        2  /* GPT-2 qkv      [3D][D]   */
#define LMC_W_ATTN_OUT   3  /* attn_proj / o  [D][H Dh] */
#define LMC_W_FFN_UP     4  /* GPT-2 fc / LLaMA up [F][D] */
#define LMC_W_FFN_DOWN   5  /* fc2 / down     [D][F]    */
#define LMC_W_Q          6  /* LLaMA q        [H Dh][D] */
#define LMC_W_K          7  /* LLaMA k        [Hkv Dh][D] */
#define LMC_W_V          8  /* LLaMA v        [Hkv Dh][D] */
#define LMC_W_GATE       9  /* LLaMA gate     [F][D]    */
const lmc_qtensor *lmc_model_matrix(const lmc_model *m, int layer, int which);
#define LMC_V_POS_EMBD      0  /* GPT-2 wpe [S][D] */
#define LMC_V_OUTPUT_NORM   1  /* ln_f weight / rms_f weight */
#define LMC_V_OUTPUT_NORM_B 2  /* ln_f bias */
#define LMC_V_ATTN_NORM     3  /* ln1 weight / rms_attn weight */
#define LMC_V_ATTN_NORM_B   4  /* ln1 bias */
#define LMC_V_FFN_NORM      5  /* ln2 weight / rms_ffn weight */
#define LMC_V_FFN_NORM_B    6  /* ln2 bias */
#define LMC_V_QKV_B         7
#define LMC_V_ATTN_OUT_B    8
#define LMC_V_FFN_UP_B      9
#define LMC_V_FFN_DOWN_B   10
#define LMC_V_ROPE_COS     11  /* LLaMA [S][Dh/2] (src/models.c:101-117) */
#define LMC_V_ROPE_SIN     12
const float *lmc_model_vector(const lmc_model *m, int layer, int which, int *len);

#ifdef __cplusplus
}
#endif
#endif /* LMC_CUDA_H */
