/* lmc_oracle.h - CPU restatement of LMc's quantized-weight hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the oracle the CUDA path is compared
 * against; it is never linked into, called by or shipped with the product
 * library (lmc_b200/liblmc_b200.so).  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg use it.
 *
 * Every function restates one LMc function (nile-agi/LMc, file:line cited
 * per function).  Parity of this restatement is pinned against LMc's own
 * sources, compiled from source into oracle/_ref/ by oracle/Makefile, on
 * seeded random blocks for all 13 block formats plus F16/F32, on single ops,
 * and on whole-model logits (tests/test_oracle.py), and against the
 * committed golden fixtures in tests/golden/ (made by
 * tests/golden/make_golden.py from the same compiled LMc sources).
 */
#ifndef LMC_ORACLE_H
#define LMC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor type IDs, LMc src/quant.h:27-45. */
enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q4_1 = 3, ORC_Q5_0 = 6,
    ORC_Q5_1 = 7, ORC_Q8_0 = 8, ORC_Q2_K = 10, ORC_Q3_K = 11, ORC_Q4_K = 12,
    ORC_Q5_K = 13, ORC_Q6_K = 14, ORC_IQ3_XXS = 18, ORC_IQ3_S = 21,
    ORC_IQ4_XS = 23
};

/* Block geometry (elements per block, bytes per block), LMc src/quant.h:54-99.
 * Returns 0 on success, -1 for an unsupported type. */
int   orc_block_geometry(uint32_t type, int *block_elems, int *block_bytes);

float orc_f16_to_f32(uint16_t h);                             /* quant.c:19-38 */

/* Decode n_elements weights of `type` from the flat block stream `src`
 * into dst.  n_elements must be a multiple of the block size.  For IQ4_XS
 * the caller must provide 2 readable bytes past the last block (LMc reads
 * them, quant.c:506,515).  Returns 0, or -1 for a bad type / size. */
int   orc_dequant(uint32_t type, const uint8_t *src, float *dst, size_t n_elements);

/* out[M] = W[M x K] . in[K] (+ bias), fp32 weights, double accumulation
 * (the reference value; LMc's own summation order differs only by
 * rounding).  ops.c:69-97 */
void  orc_matmul_vec(float *out, const float *w, const float *bias,
                     const float *in, int M, int K);

float orc_gelu(float x);                                       /* ops.c:20-24 */
float orc_silu(float x);                                       /* ops.c:26-29 */
void  orc_softmax(float *x, int n);                            /* ops.c:32-44 */
void  orc_layer_norm(float *out, const float *x, const float *w,
                     const float *b, int dim);                 /* ops.c:47-59 */
void  orc_rms_norm(float *out, const float *x, const float *w,
                   int dim, float eps);                  /* ops_llama.c:24-33 */
void  orc_rope_apply(float *vec, const float *cos_row,
                     const float *sin_row, int head_dim); /* ops_llama.c:39-48 */
void  orc_rope_cache(float *cos_tab, float *sin_tab, int S, int Dh,
                     float theta);                        /* models.c:101-117 */

/* One decode-step attention read for all query heads over a head-major
 * cache [Hkv][S][Dh] holding positions 0..pos (the new K/V already written).
 * Query head h reads kv head h / (H / Hkv).  ops.c:128-178,
 * ops_llama.c:88-134. */
void  orc_attention(float *out, const float *q, const float *k_cache,
                    const float *v_cache, int H, int Hkv, int Dh, int S,
                    int pos);

/* KV rows as the device cache may store them instead of LMc's fp32 rows
 * (models.h:149-162 keeps fp32; the compact forms are this project's
 * extension, restated here so the device path can be checked exactly):
 *   mode 0 fp32 (LMc), 1 fp16 (round to nearest even), 2 int8 codes with one
 *   fp32 scale per row: m = max|x|, q = clamp(rint(x * (127 / m)), +-127),
 *   scale = m / 127, value = q * scale (m = 0: all zero).
 * orc_kv_q8_row quantizes one row; orc_kv_round_row replaces a row by the
 * values the cache returns for it. */
void  orc_kv_q8_row(const float *x, int n, int8_t *q, float *scale);
void  orc_kv_round_row(float *row, int n, int mode);
float orc_f32_to_f16_to_f32(float x);

/* First index of the maximum (strict '>' scan), lmc.c:45-47. */
int   orc_argmax(const float *x, int n);

/* Top-p sampling with temperature as lmc.c:42-59 (logits scaled in place,
 * softmax, qsort descending, nucleus, one draw of the xorshift64 state
 * *rng as lmc.c:31-33).  Returns the token.  margin (may be NULL) receives
 * the distance, in probability, from the draw to the nearest cdf boundary of
 * the walk (a draw that close may land elsewhere under other rounding). */
int   orc_sample_top_p(float *logits, int V, float temperature, float top_p,
                       uint64_t *rng, double *margin);

/* ---- whole-model restatement (gguf.c load + ops.c/ops_llama.c forward) ---- */
typedef struct OrcModel OrcModel;
/* Parse a GGUF v1-3 file the way LMc's load_model_gguf does
 * (gguf.c:114-353) and dequantize every tensor to fp32. NULL on error. */
OrcModel *orc_model_load(const char *path);
void      orc_model_free(OrcModel *m);
/* cfg[0..10] = arch(1 gpt2, 2 llama), V, S, L, H, Hkv, D, F, Dh, theta*1000, eps*1e9 */
void      orc_model_config(const OrcModel *m, int *cfg);
/* model_forward(token, pos) (ops.c:212-237 / ops_llama.c:157-192): writes
 * V logits to `logits`.  Positions must be fed in order 0,1,2,... */
int       orc_model_forward(OrcModel *m, int token, int pos, float *logits);
/* Store K/V rows in the given kv mode (see orc_kv_round_row); default 0. */
void      orc_model_set_kv(OrcModel *m, int mode);

#ifdef __cplusplus
}
#endif
#endif /* LMC_ORACLE_H */
