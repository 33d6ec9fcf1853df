// host_decoders.cpp - compiles the CUDA block decoders (lmc_blocks.cuh) as
// host C++ so their logic can be checked bit for bit against the oracle on
// a machine without a GPU.  Built by tests/test_host_decoders.py with
// -ffp-contract=off; the CUDA intrinsics are mapped to plain IEEE float
// operations with the same rounding.
#include <stdint.h>
#include <string.h>
#include <stddef.h>

#define __device__
#define __forceinline__ inline
struct float4 { float x, y, z, w; };
static inline unsigned char __ldg(const unsigned char *p) { return *p; }
static inline unsigned short __ldg(const unsigned short *p) { return *p; }
static inline unsigned int __ldg(const unsigned int *p) { return *p; }
static inline float4 __ldg(const float4 *p) { return *p; }
static inline float __fmul_rn(float a, float b) { return a * b; }
static inline float __fadd_rn(float a, float b) { return a + b; }
static inline float __fsub_rn(float a, float b) { return a - b; }
static inline int __clz(unsigned x) { return x ? __builtin_clz(x) : 32; }
static inline float __uint_as_float(unsigned u) { float f; memcpy(&f, &u, 4); return f; }

#include "../lmc_b200/csrc/lmc_blocks.cuh"

template <int T> static void run(const uint8_t *src, float *dst, size_t n) {
    using F = lmcq::Fmt<T>;
    for (size_t g = 0; g < n / 8; g++) {
        size_t e = g * 8;
        lmcq::decode8<T>(src + (e / F::BE) * F::BB, (int)(e % F::BE), dst + e);
    }
}

extern "C" int host_decode8(uint32_t type, const uint8_t *src, float *dst, size_t n) {
    switch (type) {
#define CASE(T) case T: run<T>(src, dst, n); return 0;
        LMC_FOR_EACH_TYPE(CASE)
#undef CASE
    default: return -1;
    }
}
