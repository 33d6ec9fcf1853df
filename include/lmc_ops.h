/* lmc_ops.h - the C99 drop-in layer: LMc's own ops.h / gguf.h entry points,
 * run on the B200 through liblmc_b200.so (include/lmc_cuda.h).
 *
 * The layer is one C file, lmc_b200/dropin/lmc_ops.c, compiled against LMc's
 * headers in place of LMc's gguf.c, ops.c and ops_llama.c.  It defines, with
 * LMc's exact signatures (nile-agi/LMc src/ops.h:22-136, src/gguf.h:127):
 *
 *   load_model          src/gguf.c:114-353   GGUF -> device model; fills g_cfg
 *                                            and g_weights (see below)
 *   model_forward       src/ops.c:212-237,   whole step on the device; returns
 *                       src/ops_llama.c:157-192  g_act.logits (host, [V])
 *   matmul_vec          src/ops.c:69-97
 *   layer_norm          src/ops.c:47-59
 *   rms_norm            src/ops_llama.c:24-33
 *   softmax             src/ops.c:32-44
 *   gelu, silu          src/ops.c:20-29
 *   rope_apply          src/ops_llama.c:39-48
 *   attention_forward   src/ops.c:105-179
 *   llama_attention_forward   src/ops_llama.c:54-135
 *   swiglu_ffn_forward  src/ops_llama.c:140-153
 *   transformer_block_forward src/ops.c:182-206 (both architectures)
 *
 * Every one of them computes on the GPU; the host pointers LMc passes are
 * copied to and from device scratch around each call.  There is no CPU path:
 * a failing device call ends the process through LMC_FATAL, as LMc's own
 * errors do (src/utils.h:68-69).
 *
 * Weights.  LMc dequantizes every tensor into a host fp32 arena where
 * LOAD_QUANT runs (src/gguf.c:100-111).  load_model keeps the GGUF blocks on
 * the device instead and points each g_weights matrix field (qkv_weight,
 * q_weight, ..., wte, lm_head) at a small placeholder in LMc's arena that it
 * registers, with the device tensor, in a table; the matrix kernels resolve
 * LMc's weight pointers through that table.  The placeholders hold no weights
 * and must not be read as fp32 matrices.  Vector fields (norm weights and
 * biases, wpe, the RoPE tables) are real host copies and are registered with
 * their device copies.  An fp32 matrix that a caller passes to matmul_vec
 * without registering it is uploaded on first use and cached by its address.
 *
 * KV caches.  attention_forward / llama_attention_forward keep a device copy
 * of each host cache they are given (keyed by its address, filled from the
 * host cache on first use) and write every new K/V row to both, so LMc's host
 * cache stays what LMc's own attention would have left in it.
 *
 * The functions below are the layer's own additions (no counterpart in LMc).
 */
#ifndef LMC_OPS_DROPIN_H
#define LMC_OPS_DROPIN_H

#include "lmc_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The device model behind load_model (NULL before it). */
lmc_model *lmcdrop_model(void);

/* Register a host address that LMc code will pass as a weight matrix, with
 * the device tensor that stands for it (what load_model does for every
 * matrix of the model). */
void lmcdrop_register_matrix(const float *host, const lmc_qtensor *t);

/* Register a host fp32 vector of n floats with a device copy of it. */
void lmcdrop_register_vector(const float *host, const float *d_vec, int n);

/* Device tensor registered for a host weight pointer, or NULL. */
const lmc_qtensor *lmcdrop_lookup_matrix(const float *host);

#ifdef __cplusplus
}
#endif
#endif /* LMC_OPS_DROPIN_H */
