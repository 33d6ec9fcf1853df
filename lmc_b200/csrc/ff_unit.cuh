// ff_unit.cuh - the latency ("fp32") form of the GEMV unit bodies, shared by
// the persistent decode step (step_kernel.cu) and the standalone latency GEMV
// (ff_gemv.cu): one 16-row x 256-column unit of the tiled layout (the layout
// the tensor-core GEMV reads, tiled_gemv.cuh) dotted with fp32 activations in
// shared memory.  Include it after tiled_gemv.cuh, inside the includer's
// anonymous namespace (each translation unit gets its own copy).
#pragma once
// ---------------------------------------------------------------------------
// The latency GEMV.  The tensor-core GEMV quantizes x into three int8 limbs
// per CTA (several dependent passes and CTA-wide reductions), which pays off
// when each warp streams many units.  In a decode step most GEMVs give a warp
// one to a few units, and that set-up is most of the op's time.  For those
// ops x is staged once as fp32 in shared memory (after its prologue) and each
// lane dots the 128 weights it holds in a unit - rows
// g and g + 8 of the tile at the same 64 columns, in the tiled layout the
// tensor-core GEMV reads - against it with fp32 FMAs, applies the sub-block
// scales, and the four lanes of a row are summed by shuffles.  Results agree
// with the tensor-core path to fp32 rounding.
// ---------------------------------------------------------------------------
// Byte i of w as the float 2^23 + byte (one PRMT: the byte under 0x4B0000);
// subtracting 2^23 (or 2^23 + an offset) gives the byte exactly.
template <int I> __device__ __forceinline__ float byte_2p23(uint32_t w) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u + I));
}
// Byte i of w (which has its top bit set) as the float 0x3F 0x(80|v) 0 0 =
// 1 + v * 2^-7: one PRMT, no subtraction.  The Q4_K / Q6_K bodies place a
// 4-bit code at bits 3..6 (1 + q / 16) or a 6-bit code at bits 1..6
// (1 + q / 64) of each byte, so a dot product of n such weights with x is
// sum x + sum q x / 2^k: the sum of x (needed anyway for the mins and the
// offset) is subtracted once per 32 (16) columns, and 2^k goes into the
// block scale.  The subtraction cancels at most the 1 + ... part, so the
// relative rounding of the result stays near 2^-24 times the number of
// terms of the chunk, far inside the 1e-3 bound.
template <int I> __device__ __forceinline__ float byte_1p(uint32_t w) {
    return __uint_as_float(__byte_perm(w, 0x3F000000u, 0x7044u + (I << 8)));
}

struct FAcc {
    float v[2][2];  // [batch row][row half: g, g + 8]
    __device__ __forceinline__ void zero() { v[0][0] = v[0][1] = v[1][0] = v[1][1] = 0.0f; }
};

// Q4_K unit: d * sum_j sc_j (sum q x) - dmin * sum_j m_j (sum x)  (src/quant.c:275-303)
template <int NBR>
__device__ __forceinline__ void funit_q4k(FAcc &o, const uint8_t *u, const float *xs, int K, int k0, int lane) {
    const int g = lane >> 2, c = lane & 3;
    const uint4 H0 = *reinterpret_cast<const uint4 *>(u + 16 * g);
    const uint4 H1 = *reinterpret_cast<const uint4 *>(u + 16 * g + 128);
    const uint4 *cw = reinterpret_cast<const uint4 *>(u + 256) + lane;
    const uint4 q0 = cw[0], q1 = cw[32], q2 = cw[64], q3 = cw[96];
    const uint32_t qs[16] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w,
                             q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
    // 6-bit scales / mins, four per word (src/quant.c:44-53)
    const uint32_t sc0[2] = {H0.y & 0x3F3F3F3Fu, (H0.w & LO4) | ((H0.y >> 2) & 0x30303030u)};
    const uint32_t sc1[2] = {H1.y & 0x3F3F3F3Fu, (H1.w & LO4) | ((H1.y >> 2) & 0x30303030u)};
    const uint32_t mn0[2] = {H0.z & 0x3F3F3F3Fu, ((H0.w >> 4) & LO4) | ((H0.z >> 2) & 0x30303030u)};
    const uint32_t mn1[2] = {H1.z & 0x3F3F3F3Fu, ((H1.w >> 4) & LO4) | ((H1.z >> 2) & 0x30303030u)};
    float sg[NBR], s8[NBR], mg[NBR], m8[NBR];
#pragma unroll
    for (int b = 0; b < NBR; b++) sg[b] = s8[b] = mg[b] = m8[b] = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        // byte i of P: code(32j + 4c + i) | code(32j + 16 + 4c + i) << 4 (row g); Q: row g + 8
        const uint32_t P = qs[2 * j], Q = qs[2 * j + 1];
        // codes at bits 3..6 under the top bit: 1 + q / 16
        const uint32_t Pl = ((P << 3) & 0x78787878u) | 0x80808080u, Ph = ((P >> 1) & 0x78787878u) | 0x80808080u;
        const uint32_t Ql = ((Q << 3) & 0x78787878u) | 0x80808080u, Qh = ((Q >> 1) & 0x78787878u) | 0x80808080u;
        const float ag[8] = {byte_1p<0>(Pl), byte_1p<1>(Pl), byte_1p<2>(Pl), byte_1p<3>(Pl),
                             byte_1p<0>(Ph), byte_1p<1>(Ph), byte_1p<2>(Ph), byte_1p<3>(Ph)};
        const float a8[8] = {byte_1p<0>(Ql), byte_1p<1>(Ql), byte_1p<2>(Ql), byte_1p<3>(Ql),
                             byte_1p<0>(Qh), byte_1p<1>(Qh), byte_1p<2>(Qh), byte_1p<3>(Qh)};
        const int sh = 8 * (j & 3);
        const float scg = (float)((sc0[j >> 2] >> sh) & 63u), sc8 = (float)((sc1[j >> 2] >> sh) & 63u);
        const float mng = (float)((mn0[j >> 2] >> sh) & 63u), mn8 = (float)((mn1[j >> 2] >> sh) & 63u);
#pragma unroll
        for (int b = 0; b < NBR; b++) {
            const float4 xa = *reinterpret_cast<const float4 *>(xs + b * K + k0 + 32 * j + 4 * c);
            const float4 xb = *reinterpret_cast<const float4 *>(xs + b * K + k0 + 32 * j + 16 + 4 * c);
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            // ag[i] = 1 + q / 16: sum ag x - sum x = sum q x / 16 (the chain starts at -sum x)
            const float X = ((xv[0] + xv[1]) + (xv[2] + xv[3])) + ((xv[4] + xv[5]) + (xv[6] + xv[7]));
            float pg = -X, p8 = -X;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                pg = fmaf(ag[i], xv[i], pg);
                p8 = fmaf(a8[i], xv[i], p8);
            }
            sg[b] = fmaf(scg, pg, sg[b]);
            s8[b] = fmaf(sc8, p8, s8[b]);
            mg[b] = fmaf(mng, X, mg[b]);
            m8[b] = fmaf(mn8, X, m8[b]);
        }
    }
    const float2 dd0 = __half22float2(*reinterpret_cast<const __half2 *>(&H0.x));  // (d, dmin)
    const float2 dd1 = __half22float2(*reinterpret_cast<const __half2 *>(&H1.x));
#pragma unroll
    for (int b = 0; b < NBR; b++) {
        o.v[b][0] += (16.0f * dd0.x) * sg[b] - dd0.y * mg[b];
        o.v[b][1] += (16.0f * dd1.x) * s8[b] - dd1.y * m8[b];
    }
}

// Q6_K unit: d * sum_chunks sc * sum (q - 32) x  (src/quant.c:386-414)
template <int NBR>
__device__ __forceinline__ void funit_q6k(FAcc &o, const uint8_t *u, const float *xs, int K, int k0, int lane) {
    const int g = lane >> 2, c = lane & 3;
    const uint4 s0v = *reinterpret_cast<const uint4 *>(u + 16 * g);
    const uint4 s1v = *reinterpret_cast<const uint4 *>(u + 16 * g + 128);
    const float d0 = __half2float(*reinterpret_cast<const __half *>(u + 256 + 2 * g));
    const float d1 = __half2float(*reinterpret_cast<const __half *>(u + 256 + 2 * g + 16));
    const uint4 *lw = reinterpret_cast<const uint4 *>(u + 288) + lane;
    const uint4 *hw = reinterpret_cast<const uint4 *>(u + 288 + 2048) + lane;
    const uint4 l0 = lw[0], l1 = lw[32], l2 = lw[64], l3 = lw[96], h0 = hw[0], h1 = hw[32];
    const uint32_t lo[16] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w,
                             l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
    const uint32_t hs[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    const uint32_t sw0[4] = {s0v.x, s0v.y, s0v.z, s0v.w}, sw1[4] = {s1v.x, s1v.y, s1v.z, s1v.w};
    float sg[NBR], s8[NBR];
#pragma unroll
    for (int b = 0; b < NBR; b++) sg[b] = s8[b] = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        // byte i of P: lo(g, k) | lo(g + 8, k) << 4, k = 16 j + 4 c + i; H (chunk
        // pair j / 2): hi(g, k) | hi(g+8, k) << 2 | hi(g, k+16) << 4 | hi(g+8, k+16) << 6
        const uint32_t P = lo[j], H = (j & 1) ? hs[j >> 1] >> 4 : hs[j >> 1];
        // the 6-bit code at bits 1..6 under the top bit: 1 + q / 64
        const uint32_t wg = ((P << 1) & 0x1E1E1E1Eu) | ((H << 5) & 0x60606060u) | 0x80808080u;  // row g
        const uint32_t w8 = ((P >> 3) & 0x1E1E1E1Eu) | ((H << 3) & 0x60606060u) | 0x80808080u;  // row g + 8
        const float vg[4] = {byte_1p<0>(wg), byte_1p<1>(wg), byte_1p<2>(wg), byte_1p<3>(wg)};
        const float v8[4] = {byte_1p<0>(w8), byte_1p<1>(w8), byte_1p<2>(w8), byte_1p<3>(w8)};
        const float scg = (float)(int)(int8_t)(sw0[j >> 2] >> (8 * (j & 3)));
        const float sc8 = (float)(int)(int8_t)(sw1[j >> 2] >> (8 * (j & 3)));
#pragma unroll
        for (int b = 0; b < NBR; b++) {
            const float4 x = *reinterpret_cast<const float4 *>(xs + b * K + k0 + 16 * j + 4 * c);
            // v = 1 + q / 64: sum v x - 1.5 sum x = sum (q - 32) x / 64 (the chain starts at -1.5 sum x)
            const float X15 = -1.5f * ((x.x + x.y) + (x.z + x.w));
            const float pg = fmaf(vg[3], x.w, fmaf(vg[2], x.z, fmaf(vg[1], x.y, fmaf(vg[0], x.x, X15))));
            const float p8 = fmaf(v8[3], x.w, fmaf(v8[2], x.z, fmaf(v8[1], x.y, fmaf(v8[0], x.x, X15))));
            sg[b] = fmaf(scg, pg, sg[b]);
            s8[b] = fmaf(sc8, p8, s8[b]);
        }
    }
#pragma unroll
    for (int b = 0; b < NBR; b++) {
        o.v[b][0] += (64.0f * d0) * sg[b];
        o.v[b][1] += (64.0f * d1) * s8[b];
    }
}

// Q8_0 unit: sum_blocks d * sum q x  (src/quant.c:419-429)
template <int NBR>
__device__ __forceinline__ void funit_q80(FAcc &o, const uint8_t *u, const float *xs, int K, int k0, int lane) {
    const int g = lane >> 2, c = lane & 3;
    const uint4 H0 = *reinterpret_cast<const uint4 *>(u + 16 * g);
    const uint4 H1 = *reinterpret_cast<const uint4 *>(u + 16 * g + 128);
    const uint32_t hw0[4] = {H0.x, H0.y, H0.z, H0.w}, hw1[4] = {H1.x, H1.y, H1.z, H1.w};
    const uint4 *cw = reinterpret_cast<const uint4 *>(u + 256) + lane;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        // int8 codes with the sign bit flipped are the unsigned byte q + 128
        const uint4 A = cw[32 * j];
        const uint32_t ax = A.x ^ 0x80808080u, ay = A.y ^ 0x80808080u, az = A.z ^ 0x80808080u,
                       aw = A.w ^ 0x80808080u;
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&hw0[j >> 1]));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&hw1[j >> 1]));
        const float dg = (j & 1) ? f0.y : f0.x, d8 = (j & 1) ? f1.y : f1.x;
        constexpr float B = 8388736.0f;  // 2^23 + 128
        const float ag[8] = {byte_2p23<0>(ax) - B, byte_2p23<1>(ax) - B, byte_2p23<2>(ax) - B, byte_2p23<3>(ax) - B,
                             byte_2p23<0>(az) - B, byte_2p23<1>(az) - B, byte_2p23<2>(az) - B, byte_2p23<3>(az) - B};
        const float a8[8] = {byte_2p23<0>(ay) - B, byte_2p23<1>(ay) - B, byte_2p23<2>(ay) - B, byte_2p23<3>(ay) - B,
                             byte_2p23<0>(aw) - B, byte_2p23<1>(aw) - B, byte_2p23<2>(aw) - B, byte_2p23<3>(aw) - B};
#pragma unroll
        for (int b = 0; b < NBR; b++) {
            const float4 xa = *reinterpret_cast<const float4 *>(xs + b * K + k0 + 32 * j + 4 * c);
            const float4 xb = *reinterpret_cast<const float4 *>(xs + b * K + k0 + 32 * j + 16 + 4 * c);
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            float pg = 0.0f, p8 = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                pg = fmaf(ag[i], xv[i], pg);
                p8 = fmaf(a8[i], xv[i], p8);
            }
            o.v[b][0] = fmaf(dg, pg, o.v[b][0]);
            o.v[b][1] = fmaf(d8, p8, o.v[b][1]);
        }
    }
}

// A row tile's partial sums into the CTA accumulator acc[b][16]: the four
// lanes of each row are added by shuffles, one shared atomic per value.
__device__ __forceinline__ void fflush(const FAcc &o, float *acc_rt, int nb, int lane) {
    const int g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int b = 0; b < 2; b++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float v = o.v[b][h];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            if (c == 0 && b < nb) atomicAdd(acc_rt + b * 16 + g + 8 * h, v);
        }
}

