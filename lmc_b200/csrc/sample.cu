// sample.cu - top-p (nucleus) sampling with temperature on the device: the
// C ABI entry (lmc_sample_top_p) and the xorshift64 seeding LMc uses.
// Replaces sample_top_p and the RNG of LMc's generate loop (src/lmc.c:29-59);
// the algorithm is in sample.cuh.
#include "lmc_internal.h"
#include "sample.cuh"

namespace {

constexpr int SMP_THREADS = 1024;

// d_step (may be NULL): the generate loop's step counter; the draw is made
// only when this step's pick is a generated token (step + 1 >= n_prompt), so
// the prompt steps leave the RNG untouched, as LMc's loop does.
__global__ void __launch_bounds__(SMP_THREADS) k_sample(const float *__restrict__ lg, int V, float temperature,
                                                        float top_p, unsigned long long *rng, int *out,
                                                        const int *d_step, int n_prompt) {
    __shared__ SampleSmem S;
    pdl_wait();
    pdl_launch_dependents();
    if (d_step && __ldcg(d_step) + 1 < n_prompt) return;
    sample_row<SMP_THREADS>(lg + (size_t)blockIdx.x * V, V, temperature, top_p, rng + blockIdx.x, out + blockIdx.x,
                            S);
}

}  // namespace

// src/lmc.c:30-31: state = seed ^ 0xdeadbeefcafe, never 0.
extern "C" unsigned long long lmc_rng_seed(unsigned long long seed) {
    const unsigned long long s = seed ^ 0xdeadbeefcafeULL;
    return s ? s : 1ULL;
}

extern "C" int lmc_sample_top_p(const float *d_logits, int n, int rows, float temperature, float top_p,
                                unsigned long long *d_rng, int *d_idx, void *stream) {
    if (!d_logits || !d_rng || !d_idx || n <= 0 || rows < 0)
        return lmc_set_error(LMC_ERR_INVALID, "sample_top_p: args");
    if (temperature != temperature || top_p != top_p)
        return lmc_set_error(LMC_ERR_INVALID, "sample_top_p: NaN temperature or top_p");
    if (!rows) return LMC_OK;
    LMC_LAUNCH("sample_top_p", k_sample, rows, SMP_THREADS, 0, lmc_stream(stream), d_logits, n, temperature, top_p,
               d_rng, d_idx, (const int *)NULL, 0);
    return LMC_OK;
}

extern "C" int lmc_sample_launch(const float *d_logits, int n, int ld, int rows, float temperature, float top_p,
                                 unsigned long long *d_rng, int *d_idx, const int *d_step, int n_prompt,
                                 cudaStream_t s) {
    if (ld != n) return lmc_set_error(LMC_ERR_INVALID, "sample: logits rows must be contiguous");
    LMC_LAUNCH("sample", k_sample, rows, SMP_THREADS, 0, s, d_logits, n, temperature, top_p, d_rng, d_idx, d_step,
               n_prompt);
    return LMC_OK;
}
