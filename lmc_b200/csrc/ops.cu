// ops.cu - the small ops that keep activations on the device: LayerNorm,
// RMSNorm, softmax, GELU/SiLU/SwiGLU, RoPE, greedy argmax, embedding rows.
// All are HBM/L2-bound and tiny at decode sizes; each row is one CTA so a
// batch of rows is one launch.
#include "lmc_blocks.cuh"
#include "lmc_common.cuh"
#include "lmc_internal.h"

#include <algorithm>

// src/ops.c:47-59: mean, variance, (x - mean) * inv_std * w + b, eps 1e-5.
__global__ void k_layer_norm(float *__restrict__ out, const float *__restrict__ x, const float *__restrict__ w,
                             const float *__restrict__ b, int dim) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ float red[32];
    const float *xr = x + (size_t)blockIdx.x * dim;
    float *orow = out + (size_t)blockIdx.x * dim;
    float s = 0.0f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) s += xr[i];
    const float mean = block_sum(s, red) / (float)dim;
    float v = 0.0f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) { float d = xr[i] - mean; v += d * d; }
    const float var = block_sum(v, red);
    const float inv_std = 1.0f / sqrtf(var / (float)dim + 1e-5f);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) orow[i] = (xr[i] - mean) * inv_std * w[i] + b[i];
}

// src/ops_llama.c:24-33
__global__ void k_rms_norm(float *__restrict__ out, const float *__restrict__ x, const float *__restrict__ w,
                           int dim, float eps) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ float red[32];
    const float *xr = x + (size_t)blockIdx.x * dim;
    float *orow = out + (size_t)blockIdx.x * dim;
    float s = 0.0f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) s += xr[i] * xr[i];
    const float ss = 1.0f / sqrtf(block_sum(s, red) / (float)dim + eps);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) orow[i] = w[i] * ss * xr[i];
}

// src/ops.c:32-44
__global__ void k_softmax(float *__restrict__ x, int n) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ float red[32];
    float *r = x + (size_t)blockIdx.x * n;
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, r[i]);
    mx = block_max(mx, red);
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) { float e = expf(r[i] - mx); r[i] = e; s += e; }
    s = block_sum(s, red);
    if (s < 1e-30f) {
        for (int i = threadIdx.x; i < n; i += blockDim.x) r[i] = 1.0f / (float)n;
        return;
    }
    const float inv = 1.0f / s;
    for (int i = threadIdx.x; i < n; i += blockDim.x) r[i] *= inv;
}

__global__ void k_act(float *__restrict__ x, size_t n, int kind) {
    pdl_wait();
    pdl_launch_dependents();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        x[i] = kind == 0 ? lmc_gelu_f(x[i]) : lmc_silu_f(x[i]);
}

// src/ops_llama.c:150-151
__global__ void k_swiglu(float *__restrict__ g, const float *__restrict__ u, size_t n) {
    pdl_wait();
    pdl_launch_dependents();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        g[i] = lmc_silu_f(g[i]) * u[i];
}

// src/ops_llama.c:39-48, for n_heads consecutive vectors sharing one row.
__global__ void k_rope(float *__restrict__ v, const float *__restrict__ c, const float *__restrict__ s, int Dh,
                       int n_pairs) {
    pdl_wait();
    pdl_launch_dependents();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_pairs) return;
    const int d = i % (Dh / 2);
    const float v0 = v[2 * i], v1 = v[2 * i + 1];
    v[2 * i] = v0 * c[d] - v1 * s[d];
    v[2 * i + 1] = v0 * s[d] + v1 * c[d];
}

// src/lmc.c:45-47: strict '>' scan, so the first index of the maximum wins.
// Each thread keeps its first maximum; the merge prefers the larger value,
// then the smaller index.
__device__ __forceinline__ void am_merge(float &v, int &i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}
__global__ void k_argmax(const float *__restrict__ x, int n, int *__restrict__ idx) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ float sv[32];
    __shared__ int si[32];
    const float *r = x + (size_t)blockIdx.x * n;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = r[i];
        if (v > bv || bi == 0x7fffffff) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        am_merge(bv, bi, v2, i2);
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) { sv[wid] = bv; si[wid] = bi; }
    __syncthreads();
    if (wid == 0) {
        const int nw = blockDim.x >> 5;
        bv = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            am_merge(bv, bi, v2, i2);
        }
        if (lane == 0) idx[blockIdx.x] = (bi == 0x7fffffff) ? 0 : bi;
    }
}

// Embedding rows (src/ops.c:216-219, src/ops_llama.c:163): for sequence b,
// out[b] = dequant(row tok[b] of wte) (+ wpe[pos[b]] when wpe != NULL).
// The token row is the flat element range [tok*D, tok*D + D) of the block
// stream, decoded with the bit-exact decoders.
template <int T>
__global__ void k_embed(const uint8_t *__restrict__ wte, const float *__restrict__ wpe, const int *__restrict__ tok,
                        const int *__restrict__ pos, int D, int V, int S, float *__restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    using F = lmcq::Fmt<T>;
    const int b = blockIdx.x;
    // the host validates tokens and positions; never index outside wte / wpe
    if (tok[b] < 0 || tok[b] >= V || (wpe && (pos[b] < 0 || pos[b] >= S))) return;
    const size_t r0 = (size_t)tok[b] * D, r1 = r0 + D;
    for (size_t g = (r0 >> 3) + threadIdx.x; g < ((r1 + 7) >> 3); g += blockDim.x) {
        const size_t e = g << 3;
        float w[8];
        lmcq::decode8<T>(wte + (e / F::BE) * F::BB, (int)(e % F::BE), w);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const long long k = (long long)(e + i) - (long long)r0;
            if (k >= 0 && k < D) {
                float v = w[i];
                if (wpe) v = v + wpe[(size_t)pos[b] * D + k];
                out[(size_t)b * D + k] = v;
            }
        }
    }
}

extern "C" int lmc_embed_launch(uint32_t type, const void *wte, const float *wpe, const int *d_tok,
                                const int *d_pos, int D, int V, int S, int batch, float *out, cudaStream_t s) {
    switch (type) {
#define CASE(T) \
    case T: LMC_LAUNCH("embed", k_embed<T>, batch, 256, 0, s, (const uint8_t *)wte, wpe, d_tok, d_pos, D, V, S, out); break;
        LMC_FOR_EACH_TYPE(CASE)
#undef CASE
    default:
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "embed: type %u", type);
    }
    return LMC_OK;
}

static int rows_threads(int dim) { return dim >= 1024 ? 1024 : (dim >= 256 ? 256 : 128); }

extern "C" int lmc_layer_norm(float *out, const float *x, const float *w, const float *b, int dim, int rows,
                              void *stream) {
    if (!out || !x || !w || !b || dim <= 0 || rows < 0) return lmc_set_error(LMC_ERR_INVALID, "layer_norm: args");
    if (!rows) return LMC_OK;
    LMC_LAUNCH("layer_norm", k_layer_norm, rows, rows_threads(dim), 0, lmc_stream(stream), out, x, w, b, dim);
    return LMC_OK;
}

extern "C" int lmc_rms_norm(float *out, const float *x, const float *w, int dim, int rows, float eps, void *stream) {
    if (!out || !x || !w || dim <= 0 || rows < 0) return lmc_set_error(LMC_ERR_INVALID, "rms_norm: args");
    if (!rows) return LMC_OK;
    LMC_LAUNCH("rms_norm", k_rms_norm, rows, rows_threads(dim), 0, lmc_stream(stream), out, x, w, dim, eps);
    return LMC_OK;
}

extern "C" int lmc_softmax(float *x, int n, int rows, void *stream) {
    if (!x || n <= 0 || rows < 0) return lmc_set_error(LMC_ERR_INVALID, "softmax: args");
    if (!rows) return LMC_OK;
    k_softmax<<<rows, rows_threads(n), 0, lmc_stream(stream)>>>(x, n);
    LMC_LAUNCH_CHECK("softmax");
    return LMC_OK;
}

static int act(float *x, size_t n, int kind, void *stream) {
    if (!x) return lmc_set_error(LMC_ERR_INVALID, "activation: null");
    if (!n) return LMC_OK;
    k_act<<<std::min<size_t>(lmc_cdiv(n, 256), 148 * 16), 256, 0, lmc_stream(stream)>>>(x, n, kind);
    LMC_LAUNCH_CHECK("activation");
    return LMC_OK;
}
extern "C" int lmc_gelu(float *x, size_t n, void *stream) { return act(x, n, 0, stream); }
extern "C" int lmc_silu(float *x, size_t n, void *stream) { return act(x, n, 1, stream); }

extern "C" int lmc_swiglu(float *g, const float *u, size_t n, void *stream) {
    if (!g || !u) return lmc_set_error(LMC_ERR_INVALID, "swiglu: null");
    if (!n) return LMC_OK;
    LMC_LAUNCH("swiglu", k_swiglu, std::min<size_t>(lmc_cdiv(n, 256), 148 * 16), 256, 0, lmc_stream(stream), g, u, n);
    return LMC_OK;
}

extern "C" int lmc_rope_apply(float *v, const float *c, const float *s, int Dh, int n_heads, void *stream) {
    if (!v || !c || !s || Dh <= 0 || (Dh & 1) || n_heads < 0) return lmc_set_error(LMC_ERR_INVALID, "rope: args");
    const int pairs = n_heads * (Dh / 2);
    if (!pairs) return LMC_OK;
    k_rope<<<lmc_cdiv(pairs, 256), 256, 0, lmc_stream(stream)>>>(v, c, s, Dh, pairs);
    LMC_LAUNCH_CHECK("rope");
    return LMC_OK;
}

extern "C" int lmc_argmax(const float *x, int n, int rows, int *idx, void *stream) {
    if (!x || !idx || n <= 0 || rows < 0) return lmc_set_error(LMC_ERR_INVALID, "argmax: args");
    if (!rows) return LMC_OK;
    LMC_LAUNCH("argmax", k_argmax, rows, 1024, 0, lmc_stream(stream), x, n, idx);
    return LMC_OK;
}

// RoPE for a batch of rows, each at its own device-side position.
__global__ void k_rope_pos(float *__restrict__ v, int ld, int n_heads, int Dh, const float *__restrict__ ct,
                           const float *__restrict__ st, const int *__restrict__ pos, int S) {
    pdl_wait();
    pdl_launch_dependents();
    const int b = blockIdx.y, half = Dh / 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_heads * half || pos[b] < 0 || pos[b] >= S) return;
    const int d = i % half;
    const float c = ct[(size_t)pos[b] * half + d], s = st[(size_t)pos[b] * half + d];
    float *p = v + (size_t)b * ld + 2 * i;
    const float v0 = p[0], v1 = p[1];
    p[0] = v0 * c - v1 * s;
    p[1] = v0 * s + v1 * c;
}

extern "C" int lmc_rope_pos_launch(float *v, int ld, int n_heads, int Dh, const float *ct, const float *st,
                                   const int *d_pos, int S, int batch, cudaStream_t s) {
    const int pairs = n_heads * (Dh / 2);
    LMC_LAUNCH("rope_pos", k_rope_pos, dim3(lmc_cdiv(pairs, 128), batch), 128, 0, s, v, ld, n_heads, Dh, ct, st, d_pos, S);
    return LMC_OK;
}

// Greedy argmax producing the pick key of each row (see lmc_argmax_key):
// used when the lm_head GEMV cannot fuse the argmax itself.
__global__ void k_argmax_keys(const float *__restrict__ x, int n, unsigned long long *__restrict__ keys) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ unsigned long long sk[32];
    const float *r = x + (size_t)blockIdx.x * n;
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long k = lmc_argmax_key(r[i], i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    if ((threadIdx.x & 31) == 0) sk[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) best = sk[w] > best ? sk[w] : best;
        best = sk[0] > best ? sk[0] : best;
        keys[blockIdx.x] = best;
    }
}

extern "C" int lmc_argmax_keys_launch(const float *d_x, int n, int rows, unsigned long long *d_keys, cudaStream_t s) {
    LMC_LAUNCH("argmax_keys", k_argmax_keys, rows, 1024, 0, s, d_x, n, d_keys);
    return LMC_OK;
}

// key -> id, and reset the key for the next step
__global__ void k_keys_to_ids(unsigned long long *__restrict__ keys, int *__restrict__ next, int batch) {
    pdl_wait();
    pdl_launch_dependents();
    for (int b = threadIdx.x; b < batch; b += blockDim.x) {
        next[b] = lmc_key_index(keys[b]);
        keys[b] = 0ull;
    }
}

extern "C" int lmc_keys_to_ids_launch(unsigned long long *d_keys, int *d_next, int batch, cudaStream_t s) {
    LMC_LAUNCH("keys_to_ids", k_keys_to_ids, 1, 256, 0, s, d_keys, d_next, batch);
    return LMC_OK;
}

// Generation bookkeeping run after every step of lmc_model_generate: the
// step just computed position `step`; the next step feeds the next prompt
// token while the prompt lasts (token-by-token prefill, src/lmc.c:109-112),
// then the greedy pick (src/lmc.c:123,129), which is also recorded.  The
// pick is read from the step's argmax key, which is reset for the next step.
__global__ void k_advance(unsigned long long *__restrict__ keys, int *__restrict__ next, int *__restrict__ tok,
                          int *__restrict__ pos, int *__restrict__ step_p, const int *__restrict__ prompt, int n_prompt,
                          int *__restrict__ ids, int n_new, int batch, int from_next) {
    pdl_wait();
    pdl_launch_dependents();
    const int step = *step_p;
    for (int b = threadIdx.x; b < batch; b += blockDim.x) {
        const int nx = from_next ? next[b] : lmc_key_index(keys[b]);
        keys[b] = 0ull;
        next[b] = nx;
        if (step + 1 < n_prompt) {
            tok[b] = prompt[(size_t)b * n_prompt + step + 1];
        } else {
            const int k = step + 1 - n_prompt;
            tok[b] = nx;
            if (k < n_new) ids[(size_t)b * n_new + k] = nx;
        }
        pos[b] = step + 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) *step_p = step + 1;
}

extern "C" int lmc_advance_launch(unsigned long long *d_keys, int *d_next, int *d_tok, int *d_pos, int *d_step,
                                  const int *d_prompt, int n_prompt, int *d_ids, int n_new, int batch, int from_next,
                                  cudaStream_t s) {
    LMC_LAUNCH("advance", k_advance, 1, 256, 0, s, d_keys, d_next, d_tok, d_pos, d_step, d_prompt, n_prompt, d_ids,
               n_new, batch, from_next);
    return LMC_OK;
}
