// capi.cu - C ABI plumbing: error reporting, device init, block geometry,
// quantized tensors on the device and the matmul dispatcher.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include "lmc_common.cuh"
#include "lmc_internal.h"

#include <algorithm>
#include <mutex>
#include <thread>
#include <vector>

static thread_local char g_err[1024];

extern "C" int lmc_set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

extern "C" const char *lmc_last_error(void) { return g_err; }

// Programmatic dependent launch is on unless LMC_PDL=0 (A/B timing switch).
extern "C" int lmc_pdl_enabled(void) {
    static int flag = -1;
    if (flag < 0) {
        const char *e = getenv("LMC_PDL");
        flag = (e && e[0] == '0') ? 0 : 1;
    }
    return flag;
}

extern "C" int lmc_set_wait_limit(long long ns) {
    if (ns < 0) return lmc_set_error(LMC_ERR_INVALID, "set_wait_limit: %lld", ns);
    int rc = lmc_tiled_set_wait_limit(ns);
    if (!rc) rc = lmc_step_set_wait_limit(ns);
    if (!rc) rc = lmc_gemm_set_wait_limit(ns);
    if (!rc) rc = lmc_peer_set_wait_limit(ns);
    return rc;
}

extern "C" int lmc_wait_selftest(int which) {
    if (which != 0 && which != 1) return lmc_set_error(LMC_ERR_INVALID, "wait_selftest: %d", which);
    int *d = NULL;
    LMC_CUDA_TRY(cudaMalloc((void **)&d, sizeof(int)));
    LMC_CUDA_TRY(cudaMemset(d, 0, sizeof(int)));
    int rc;
    if (which == 0) {
        rc = lmc_tiled_wait_selftest(d, 0);
        if (!rc && cudaDeviceSynchronize() != cudaSuccess) rc = lmc_set_error(LMC_ERR_CUDA, "wait self-test sync");
        int gave_up = 0;
        if (!rc && cudaMemcpy(&gave_up, d, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = lmc_set_error(LMC_ERR_CUDA, "wait self-test read");
        if (!rc) rc = lmc_device_status(); /* reports (and clears) the recorded timeout */
        if (rc == LMC_OK && gave_up) rc = lmc_set_error(LMC_ERR_CUDA, "wait self-test: timeout not recorded");
    } else {
        rc = lmc_step_barrier_selftest(d, 0);
    }
    cudaFree(d);
    return rc;
}

extern "C" int lmc_init(int device) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0)
        return lmc_set_error(LMC_ERR_CUDA, "no CUDA device (%s)", cudaGetErrorString(e));
    if (device < 0 || device >= n) return lmc_set_error(LMC_ERR_INVALID, "device %d of %d", device, n);
    LMC_CUDA_TRY(cudaSetDevice(device));
    int major = 0, minor = 0;
    LMC_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    LMC_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
    if (major != 10 || minor != 0)
        return lmc_set_error(LMC_ERR_CUDA, "device %d is sm_%d%d; this library is built for sm_100a only", device,
                             major, minor);
    LMC_CUDA_TRY(cudaFree(0));  // create the context now
    return LMC_OK;
}

// src/quant.h:54-99 (F32/F16: one element of 4/2 bytes).
extern "C" int lmc_block_geometry(uint32_t type, int *be, int *bb) {
    int e, b;
    switch (type) {
    case LMC_TYPE_F32: e = 1; b = 4; break;
    case LMC_TYPE_F16: e = 1; b = 2; break;
    case LMC_TYPE_Q4_0: e = 32; b = 18; break;
    case LMC_TYPE_Q4_1: e = 32; b = 20; break;
    case LMC_TYPE_Q5_0: e = 32; b = 22; break;
    case LMC_TYPE_Q5_1: e = 32; b = 24; break;
    case LMC_TYPE_Q8_0: e = 32; b = 34; break;
    case LMC_TYPE_Q2_K: e = 256; b = 84; break;
    case LMC_TYPE_Q3_K: e = 256; b = 110; break;
    case LMC_TYPE_Q4_K: e = 256; b = 144; break;
    case LMC_TYPE_Q5_K: e = 256; b = 176; break;
    case LMC_TYPE_Q6_K: e = 256; b = 210; break;
    case LMC_TYPE_IQ3_XXS: e = 256; b = 98; break;
    case LMC_TYPE_IQ3_S: e = 256; b = 110; break;
    case LMC_TYPE_IQ4_XS: e = 256; b = 136; break;
    default: return lmc_set_error(LMC_ERR_UNSUPPORTED, "unsupported tensor type %u", type);
    }
    if (be) *be = e;
    if (bb) *bb = b;
    return LMC_OK;
}

extern "C" int lmc_tensor_bytes(uint32_t type, size_t n_elements, size_t *bytes) {
    int be, bb;
    int rc = lmc_block_geometry(type, &be, &bb);
    if (rc) return rc;
    if (n_elements % (size_t)be)
        return lmc_set_error(LMC_ERR_INVALID, "n_elements=%zu not a multiple of %d", n_elements, be);
    *bytes = n_elements / (size_t)be * (size_t)bb;
    return LMC_OK;
}

// ---------------------------------------------------------------------------
// qtensor: raw GGUF blocks on the device (+ a tiled copy for tensor-core GEMV)
// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// Host -> device copies of model weights through pinned staging buffers.
// A copy from pageable memory (or a mapped file, whose pages are read on
// first touch) is split into chunks: host threads copy chunk i into one of
// two pinned buffers while the DMA engine moves chunk i - 1 to the device,
// so reading the file and the PCIe transfer overlap.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t STAGE_BYTES = 32u << 20;  // per buffer
constexpr int STAGE_THREADS = 8;           // host threads filling a buffer
struct Stage {
    std::mutex mu;
    void *buf[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    cudaStream_t st = nullptr;
    int dev = -1;
};
Stage g_stage;

void par_copy(void *dst, const void *src, size_t n) {
    const size_t piece = (n + STAGE_THREADS - 1) / STAGE_THREADS;
    if (n < (4u << 20)) {
        memcpy(dst, src, n);
        return;
    }
    std::vector<std::thread> th;
    for (int i = 1; i < STAGE_THREADS; i++) {
        const size_t o = piece * i;
        if (o >= n) break;
        th.emplace_back([=] { memcpy((char *)dst + o, (const char *)src + o, std::min(piece, n - o)); });
    }
    memcpy(dst, src, std::min(piece, n));
    for (auto &t : th) t.join();
}
}  // namespace

extern "C" int lmc_h2d_staged(void *d_dst, const void *h_src, size_t bytes) {
    if (!bytes) return LMC_OK;
    if (bytes < (1u << 20)) {  // small: one plain copy
        const cudaError_t e = cudaMemcpy(d_dst, h_src, bytes, cudaMemcpyHostToDevice);
        return e == cudaSuccess ? LMC_OK : lmc_set_error(LMC_ERR_CUDA, "h2d: %s", cudaGetErrorString(e));
    }
    std::lock_guard<std::mutex> lock(g_stage.mu);
    int dev = 0;
    LMC_CUDA_TRY(cudaGetDevice(&dev));
    if (g_stage.dev != dev) {  // (re)create the staging set on this device
        for (int i = 0; i < 2; i++) {
            if (g_stage.buf[i]) cudaFreeHost(g_stage.buf[i]);
            if (g_stage.done[i]) cudaEventDestroy(g_stage.done[i]);
            g_stage.buf[i] = nullptr;
            g_stage.done[i] = nullptr;
        }
        if (g_stage.st) cudaStreamDestroy(g_stage.st);
        g_stage.st = nullptr;
        g_stage.dev = -1;
        for (int i = 0; i < 2; i++) {
            LMC_CUDA_TRY(cudaHostAlloc(&g_stage.buf[i], STAGE_BYTES, cudaHostAllocDefault));
            LMC_CUDA_TRY(cudaEventCreateWithFlags(&g_stage.done[i], cudaEventDisableTiming));
        }
        LMC_CUDA_TRY(cudaStreamCreateWithFlags(&g_stage.st, cudaStreamNonBlocking));
        g_stage.dev = dev;
    }
    int k = 0;
    for (size_t o = 0; o < bytes; o += STAGE_BYTES, k ^= 1) {
        const size_t n = std::min(STAGE_BYTES, bytes - o);
        LMC_CUDA_TRY(cudaEventSynchronize(g_stage.done[k]));  // the DMA that last read buffer k is over
        par_copy(g_stage.buf[k], (const char *)h_src + o, n);
        LMC_CUDA_TRY(cudaMemcpyAsync((char *)d_dst + o, g_stage.buf[k], n, cudaMemcpyHostToDevice, g_stage.st));
        LMC_CUDA_TRY(cudaEventRecord(g_stage.done[k], g_stage.st));
    }
    LMC_CUDA_TRY(cudaStreamSynchronize(g_stage.st));
    return LMC_OK;
}

extern "C" int lmc_qtensor_upload(uint32_t type, int rows, int cols, const void *h_blocks, size_t bytes,
                                  lmc_qtensor **out) {
    if (!out || !h_blocks || rows <= 0 || cols <= 0) return lmc_set_error(LMC_ERR_INVALID, "qtensor_upload: args");
    *out = NULL;
    size_t need;
    int rc = lmc_tensor_bytes(type, (size_t)rows * cols, &need);
    if (rc) return rc;
    if (bytes < need) return lmc_set_error(LMC_ERR_INVALID, "qtensor_upload: %zu bytes < %zu needed", bytes, need);
    lmc_qtensor *t = (lmc_qtensor *)calloc(1, sizeof(lmc_qtensor));
    if (!t) return lmc_set_error(LMC_ERR_OOM, "qtensor_upload: host alloc");
    t->type = type;
    t->rows = rows;
    t->cols = cols;
    t->bytes = need;
    // LMC_BLOCK_PAD zero bytes after the stream: IQ4_XS decoding reads two
    // bytes past the last block (src/quant.c:506,515).
    cudaError_t e = cudaMalloc(&t->blocks, need + LMC_BLOCK_PAD);
    if (e != cudaSuccess) { free(t); return lmc_set_error(LMC_ERR_OOM, "qtensor_upload: %s", cudaGetErrorString(e)); }
    rc = lmc_h2d_staged(t->blocks, h_blocks, need);
    if (rc) {
        cudaFree(t->blocks);
        free(t);
        return rc;
    }
    e = cudaMemset((char *)t->blocks + need, 0, LMC_BLOCK_PAD);
    if (e != cudaSuccess) {
        cudaFree(t->blocks);
        free(t);
        return lmc_set_error(LMC_ERR_CUDA, "qtensor_upload: %s", cudaGetErrorString(e));
    }
    rc = lmc_tiled_build(t);
    if (!rc) rc = lmc_gemm_prepare(t);
    if (rc) {
        lmc_qtensor_free(t);
        return rc;
    }
    *out = t;
    return LMC_OK;
}

// Rows of several tensors of the same type and width stacked into one tensor
// (block streams concatenated; each part's n_elements is a multiple of the
// block size, so the result is a valid block stream).  *out = NULL when the
// parts do not match.
extern "C" int lmc_qtensor_concat(const lmc_qtensor *const *parts, int n, lmc_qtensor **out) {
    *out = NULL;
    if (n <= 0 || !parts[0]) return LMC_OK;
    int rows = 0;
    size_t bytes = 0;
    for (int i = 0; i < n; i++) {
        if (!parts[i] || parts[i]->type != parts[0]->type || parts[i]->cols != parts[0]->cols) return LMC_OK;
        rows += parts[i]->rows;
        bytes += parts[i]->bytes;
    }
    lmc_qtensor *t = (lmc_qtensor *)calloc(1, sizeof(lmc_qtensor));
    if (!t) return lmc_set_error(LMC_ERR_OOM, "qtensor_concat: host alloc");
    t->type = parts[0]->type;
    t->rows = rows;
    t->cols = parts[0]->cols;
    t->bytes = bytes;
    cudaError_t e = cudaMalloc(&t->blocks, bytes + LMC_BLOCK_PAD);
    if (e != cudaSuccess) { free(t); return lmc_set_error(LMC_ERR_OOM, "qtensor_concat: %s", cudaGetErrorString(e)); }
    size_t off = 0;
    for (int i = 0; i < n && e == cudaSuccess; i++) {
        e = cudaMemcpy((char *)t->blocks + off, parts[i]->blocks, parts[i]->bytes, cudaMemcpyDeviceToDevice);
        off += parts[i]->bytes;
    }
    if (e == cudaSuccess) e = cudaMemset((char *)t->blocks + bytes, 0, LMC_BLOCK_PAD);
    if (e != cudaSuccess) {
        lmc_qtensor_free(t);
        return lmc_set_error(LMC_ERR_CUDA, "qtensor_concat: %s", cudaGetErrorString(e));
    }
    int rc = lmc_tiled_build(t);
    if (!rc) rc = lmc_gemm_prepare(t);
    if (rc) { lmc_qtensor_free(t); return rc; }
    *out = t;
    return LMC_OK;
}

// Two tensors of the same shape with their row tiles interleaved:
// [a rows 0..T-1][b rows 0..T-1][a rows T..2T-1][b rows T..2T-1]... (T =
// tile_rows; each row a whole block stream).  Used for the gate and up
// projections of a SwiGLU FFN, so that one CTA owns both halves of the rows
// it finishes.
extern "C" int lmc_qtensor_interleave(const lmc_qtensor *a, const lmc_qtensor *b, int tile_rows, lmc_qtensor **out) {
    *out = NULL;
    size_t rb;
    if (!a || !b || a->type != b->type || a->rows != b->rows || a->cols != b->cols || tile_rows <= 0 ||
        a->rows % tile_rows || lmc_tensor_bytes(a->type, (size_t)a->cols, &rb))
        return lmc_set_error(LMC_ERR_INVALID, "qtensor_interleave: shapes");
    lmc_qtensor *t = (lmc_qtensor *)calloc(1, sizeof(lmc_qtensor));
    if (!t) return lmc_set_error(LMC_ERR_OOM, "qtensor_interleave: host alloc");
    t->type = a->type;
    t->rows = 2 * a->rows;
    t->cols = a->cols;
    t->bytes = a->bytes + b->bytes;
    cudaError_t e = cudaMalloc(&t->blocks, t->bytes + LMC_BLOCK_PAD);
    if (e != cudaSuccess) { free(t); return lmc_set_error(LMC_ERR_OOM, "qtensor_interleave: %s", cudaGetErrorString(e)); }
    const size_t tb = rb * tile_rows, nt = (size_t)a->rows / tile_rows;
    e = cudaMemcpy2D(t->blocks, 2 * tb, a->blocks, tb, tb, nt, cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess) e = cudaMemcpy2D((char *)t->blocks + tb, 2 * tb, b->blocks, tb, tb, nt, cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess) e = cudaMemset((char *)t->blocks + t->bytes, 0, LMC_BLOCK_PAD);
    if (e != cudaSuccess) {
        lmc_qtensor_free(t);
        return lmc_set_error(LMC_ERR_CUDA, "qtensor_interleave: %s", cudaGetErrorString(e));
    }
    const int rc = lmc_tiled_build(t);
    if (rc) { lmc_qtensor_free(t); return rc; }
    *out = t;
    return LMC_OK;
}

extern "C" int lmc_qtensor_free(lmc_qtensor *t) {
    if (!t) return LMC_OK;
    if (t->blocks) cudaFree(t->blocks);
    if (t->tiled) cudaFree(t->tiled);
    free(t);
    return LMC_OK;
}

extern "C" const void *lmc_qtensor_blocks(const lmc_qtensor *t) { return t ? t->blocks : NULL; }
extern "C" int lmc_qtensor_shape(const lmc_qtensor *t, uint32_t *type, int *rows, int *cols) {
    if (!t) return lmc_set_error(LMC_ERR_INVALID, "qtensor_shape: null");
    if (type) *type = t->type;
    if (rows) *rows = t->rows;
    if (cols) *cols = t->cols;
    return LMC_OK;
}

// ---------------------------------------------------------------------------
// device buffers for callers without CUDA headers
// ---------------------------------------------------------------------------
extern "C" int lmc_buffer_alloc(size_t bytes, void **d_out) {
    if (!d_out) return lmc_set_error(LMC_ERR_INVALID, "buffer_alloc: null");
    *d_out = NULL;
    cudaError_t e = cudaMalloc(d_out, bytes ? bytes : 16);
    if (e != cudaSuccess) return lmc_set_error(LMC_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    return LMC_OK;
}
extern "C" int lmc_buffer_free(void *d) {
    if (d) LMC_CUDA_TRY(cudaFree(d));
    return LMC_OK;
}
extern "C" int lmc_copy(void *dst, const void *src, size_t bytes, int dir, void *stream) {
    if ((!dst || !src) && bytes) return lmc_set_error(LMC_ERR_INVALID, "copy: null pointer");
    if (dir < LMC_H2D || dir > LMC_D2D) return lmc_set_error(LMC_ERR_INVALID, "copy: direction %d", dir);
    if (!bytes) return LMC_OK;
    const cudaMemcpyKind k = dir == LMC_H2D ? cudaMemcpyHostToDevice
                             : dir == LMC_D2H ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
    LMC_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, k, lmc_stream(stream)));
    return LMC_OK;
}
extern "C" int lmc_stream_sync(void *stream) {
    LMC_CUDA_TRY(cudaStreamSynchronize(lmc_stream(stream)));
    return LMC_OK;
}
extern "C" int lmc_qtensor_has_tiled(const lmc_qtensor *t) { return t && t->tiled ? 1 : 0; }

// ---------------------------------------------------------------------------
// matmul dispatch
// ---------------------------------------------------------------------------
static int check_mm(const float *x, int ldx, float *y, int ldy, int rows, int cols, int batch) {
    if (!x || !y || rows <= 0 || cols <= 0 || batch <= 0)
        return lmc_set_error(LMC_ERR_INVALID, "matmul: null pointer or empty shape");
    if (ldx < cols || ldy < rows) return lmc_set_error(LMC_ERR_INVALID, "matmul: ldx %d < %d or ldy %d < %d", ldx, cols,
                                                       ldy, rows);
    return LMC_OK;
}

extern "C" int lmc_matmul_blocks(uint32_t type, const void *d_blocks, int rows, int cols, const float *d_x, int ldx,
                                 const float *d_bias, float *d_y, int ldy, int batch, int epi, void *stream) {
    int rc = check_mm(d_x, ldx, d_y, ldy, rows, cols, batch);
    if (rc) return rc;
    size_t need;
    if ((rc = lmc_tensor_bytes(type, (size_t)rows * cols, &need))) return rc;
    if (!d_blocks) return lmc_set_error(LMC_ERR_INVALID, "matmul: null weights");
    if ((type == LMC_TYPE_F32 && ((uintptr_t)d_blocks & 15)) || ((uintptr_t)d_blocks & 1))
        return lmc_set_error(LMC_ERR_INVALID, "matmul: misaligned weights");
    if ((type == LMC_TYPE_F32 || type == LMC_TYPE_F16) && ((size_t)rows * cols) % 8)
        return lmc_set_error(LMC_ERR_UNSUPPORTED, "matmul: raw F32/F16 weights need rows*cols %% 8 == 0 "
                             "(upload a qtensor instead)");
    return lmc_gemv_generic_launch(type, d_blocks, rows, cols, d_x, ldx, d_bias, d_y, ldy, batch, epi,
                                   lmc_stream(stream));
}

extern "C" const char *lmc_matmul_kernel(const lmc_qtensor *w, int batch, int epi) {
    if (!w || batch <= 0) return "none";
    if (batch > 8 && w->gemm_wscale > 0.0f)
        return w->tiled ? "tcgen05 GEMM (tiled units)" : "tcgen05 GEMM (generic decoders)";
    if (w->tiled)
        return lmc_ff_gemv_suits(w, batch, epi) ? "latency GEMV (tiled units, fp32 FMA)"
                                                : "tensor-core GEMV (tiled units, int8 mma.sync)";
    return "generic GEMV (bit-exact decoders, CUDA cores)";
}

extern "C" int lmc_matmul(const lmc_qtensor *w, const float *d_x, int ldx, const float *d_bias, float *d_y, int ldy,
                          int batch, int epi, void *stream) {
    if (!w) return lmc_set_error(LMC_ERR_INVALID, "matmul: null qtensor");
    int rc = check_mm(d_x, ldx, d_y, ldy, w->rows, w->cols, batch);
    if (rc) return rc;
    // batch widths above the GEMV's 8 rows: the tensor-core GEMM
    if (batch > 8 && w->gemm_wscale > 0.0f && !((uintptr_t)d_x & 15) && !(ldx & 3))
        return lmc_gemm_launch(w, d_x, ldx, d_bias, d_y, ldy, batch, epi, NULL, lmc_stream(stream));
    if (w->tiled) return lmc_tiled_gemv_launch(w, d_x, ldx, d_bias, d_y, ldy, batch, epi, lmc_stream(stream));
    return lmc_gemv_generic_launch(w->type, w->blocks, w->rows, w->cols, d_x, ldx, d_bias, d_y, ldy, batch, epi,
                                   lmc_stream(stream));
}
