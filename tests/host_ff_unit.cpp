// host_ff_unit.cpp - compiles the latency GEMV's unit bodies
// (lmc_b200/csrc/ff_unit.cuh: one 16-row x 256-column unit of the tiled
// layout dotted with fp32 activations, per lane) as host C++, so their
// arithmetic can be checked against the oracle on a machine without a GPU.
// Built by tests/test_host_ff_unit.py with -ffp-contract=off.  The CUDA
// intrinsics the bodies use are given exact host meanings: __byte_perm
// selects bytes of {y:x} by the low three bits of each selector nibble,
// fmaf is the C library's correctly rounded fused multiply-add, halves are
// converted exactly.  The per-lane results are added here the way the
// kernel's flush adds them (the four lanes of a row, then the units of a
// row tile), in a fixed order.
#include <math.h>
#include <stdint.h>
#include <string.h>

#define __device__
#define __forceinline__ inline

struct uint4 { uint32_t x, y, z, w; };
struct float4 { float x, y, z, w; };
struct float2 { float x, y; };
struct __half { uint16_t bits; };
struct __half2 { __half lo, hi; };

static inline float __uint_as_float(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline uint32_t __byte_perm(uint32_t x, uint32_t y, uint32_t s) {
    const uint64_t v = ((uint64_t)y << 32) | x;
    uint32_t r = 0;
    for (int n = 0; n < 4; n++) r |= (uint32_t)((v >> (8 * ((s >> (4 * n)) & 7))) & 0xFF) << (8 * n);
    return r;
}
// IEEE binary16 -> binary32, exact (normal, subnormal, inf, nan)
static inline float h2f(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    if (e == 31) return __uint_as_float(s | 0x7F800000u | (m << 13));
    if (e) return __uint_as_float(s | ((e + 112) << 23) | (m << 13));
    const float v = (float)m * (1.0f / 16777216.0f);  // m * 2^-24, exact
    return s ? -v : v;
}
static inline float __half2float(__half h) { return h2f(h.bits); }
static inline float2 __half22float2(__half2 h) { return float2{h2f(h.lo.bits), h2f(h.hi.bits)}; }
// fflush (the in-kernel lane reduction) is compiled but not called here
static inline float __shfl_xor_sync(unsigned, float v, int) { return v; }
static inline float atomicAdd(float *p, float v) {
    const float o = *p;
    *p = o + v;
    return o;
}

constexpr uint32_t LO4 = 0x0F0F0F0Fu;
#include "../lmc_b200/csrc/ff_unit.cuh"

// y[b][16 rt + r] = sum over the row tile's KB units of the unit bodies'
// lane results, for b < nb (1 or 2); units: RT x KB units of the tiled layout
// (row-tile major) of format qt (4: Q4_K, 6: Q6_K, 8: Q8_0); x: nb rows of
// K = 256 KB floats.
extern "C" int host_ff_gemv(int qt, const uint8_t *units, int RT, int KB, const float *x, int nb, float *y) {
    const int K = 256 * KB, U = qt == 4 ? 2304 : qt == 6 ? 3360 : qt == 8 ? 4352 : 0;
    if (!U || nb < 1 || nb > 2) return -1;
    for (int rt = 0; rt < RT; rt++) {
        float tile[2][16] = {};
        for (int kb = 0; kb < KB; kb++) {
            const uint8_t *u = units + (size_t)(rt * KB + kb) * U;
            float unit[2][16] = {};
            for (int lane = 0; lane < 32; lane++) {
                FAcc o;
                o.zero();
                if (qt == 4) nb == 1 ? funit_q4k<1>(o, u, x, K, 256 * kb, lane) : funit_q4k<2>(o, u, x, K, 256 * kb, lane);
                if (qt == 6) nb == 1 ? funit_q6k<1>(o, u, x, K, 256 * kb, lane) : funit_q6k<2>(o, u, x, K, 256 * kb, lane);
                if (qt == 8) nb == 1 ? funit_q80<1>(o, u, x, K, 256 * kb, lane) : funit_q80<2>(o, u, x, K, 256 * kb, lane);
                const int g = lane >> 2;
                for (int b = 0; b < nb; b++) {
                    unit[b][g] += o.v[b][0];
                    unit[b][g + 8] += o.v[b][1];
                }
            }
            for (int b = 0; b < nb; b++)
                for (int r = 0; r < 16; r++) tile[b][r] += unit[b][r];
        }
        for (int b = 0; b < nb; b++)
            for (int r = 0; r < 16; r++) y[(size_t)b * RT * 16 + rt * 16 + r] = tile[b][r];
    }
    return 0;
}
