// g4_quant.cuh — warp-level Q8_K block quantizer shared by the kernels
// (quantize_row_q8_K, gemma4-4b/cpu-blas/main.c:282-340).
#pragma once
#include "g4_internal.cuh"

namespace g4 {

// Quantize the 256 floats xb[0..255] (any memory space); lane l owns
// elements 8l..8l+7.  Returns the lane's 8 int8 values packed in q[2], the
// block scale d, and the lane's sum of its 8 values.
__device__ __forceinline__ void warp_quant_block(const float *xb, int lane, uint32_t q[2], float &d, int &lsum) {
    float v[8];
    const float4 a = *reinterpret_cast<const float4 *>(xb + 8 * lane);
    const float4 b = *reinterpret_cast<const float4 *>(xb + 8 * lane + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    // first index of the largest |x| (strict '>' scan, main.c:288-296)
    float amax = 0.0f, maxv = 0.0f;
    int idx = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float ax = fabsf(v[i]);
        if (ax > amax) { amax = ax; maxv = v[i]; idx = 8 * lane + i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const float ov = __shfl_xor_sync(0xffffffffu, maxv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (oa > amax || (oa == amax && oi < idx)) { amax = oa; maxv = ov; idx = oi; }
    }
    if (amax == 0.0f) {  // all-zero block (main.c:297-302)
        q[0] = q[1] = 0u; d = 0.0f; lsum = 0;
        return;
    }
    const float iscale = __fdiv_rn(-127.0f, maxv);
    int s = 0;
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int qi = __float2int_rn(__fmul_rn(iscale, v[i]));  // round half to even, like _mm256_round_ps
        qi = qi > 127 ? 127 : (qi < -128 ? -128 : qi);
        s += qi;
        if (i < 4) w0 |= ((uint32_t)qi & 0xffu) << (8 * i);
        else w1 |= ((uint32_t)qi & 0xffu) << (8 * (i - 4));
    }
    q[0] = w0; q[1] = w1;
    d = __fdiv_rn(1.0f, iscale);
    lsum = s;
}

// Store one quantized block in the BlockQ8_K byte layout (292 B, 4-aligned).
__device__ __forceinline__ void store_q8_block(uint8_t *yb, int lane, const uint32_t q[2], float d, int lsum) {
    const int pair = lsum + __shfl_xor_sync(0xffffffffu, lsum, 1);
    if (lane == 0) *reinterpret_cast<float *>(yb) = d;
    uint32_t *qs = reinterpret_cast<uint32_t *>(yb + 4 + 8 * lane);
    qs[0] = q[0];
    qs[1] = q[1];
    if ((lane & 1) == 0) reinterpret_cast<int16_t *>(yb + 260)[lane >> 1] = (int16_t)pair;
}

}  // namespace g4

namespace g4 {

// ---------------------------------------------------------------- Q6_K activation pieces
//
// The Q6_K weights are multiplied against the fp32 activation (mm_quant_rows,
// gemma4-4b/cpu-blas/main.c:1539-1556).  To make that dot product exact and
// independent of summation order (so the streaming GEMV and the tensor-core
// GEMM agree bit for bit), each 256-element block of the activation is put on
// a fixed-point grid: with E the exponent that bounds the block (max|x| < 2^E),
//   X_i = rint(x_i * 2^(22-E))          |X_i| <= 2^22
//   X_i = a0_i * 2^16 + a1_i * 2^8 + a2_i   (signed bytes, |a0| <= 64)
// and the block's scale is 2^(E-22).  The integer dot sum_i v_i X_i of the
// weight integers v = sc*(q-32) with the X is then exact (it fits in 44 bits),
// and is turned into a float once per block.  Elements far below the block
// maximum keep 22 bits relative to that maximum.

// 2^e as a float, exact for e in [-149, 127] (subnormal below -126), 0 below.
__device__ __forceinline__ float pow2f(int e) {
    if (e >= -126) return __uint_as_float((uint32_t)(e + 127) << 23);
    if (e >= -149) return __uint_as_float(1u << (e + 149));
    return 0.0f;
}

// One block: lane l holds elements 8l..8l+7 in v.  Returns the lane's three
// byte planes (p[2*j], p[2*j+1] = elements 8l..8l+3, 8l+4..8l+7 of piece j) and
// the block scale 2^(E-22) (0 for an all-zero block).
__device__ __forceinline__ void q6x_block(const float (&v)[8], uint32_t (&p)[6], float &ys) {
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) m = fmaxf(m, fabsf(v[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
#pragma unroll
    for (int j = 0; j < 6; j++) p[j] = 0u;
    if (!(m > 0.0f)) { ys = 0.0f; return; }
    const int be = (int)((__float_as_uint(m) >> 23) & 0xffu);
    const int E = be ? be - 126 : -126;  // m < 2^E
    const int k = 22 - E;                // scale up by 2^k (k may exceed 127 for tiny blocks: two steps, exact)
    const float s1 = pow2f(k > 127 ? 127 : k), s2 = pow2f(k > 127 ? k - 127 : 0);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int X = __float2int_rn(__fmul_rn(__fmul_rn(v[j], s1), s2));
        const int a2 = (int)(int8_t)(X & 0xff);
        const int X1 = (X - a2) >> 8;
        const int a1 = (int)(int8_t)(X1 & 0xff);
        const int a0 = (X1 - a1) >> 8;
        const int w = j >> 2, sh = 8 * (j & 3);
        p[w] |= ((uint32_t)a0 & 0xffu) << sh;
        p[2 + w] |= ((uint32_t)a1 & 0xffu) << sh;
        p[4 + w] |= ((uint32_t)a2 & 0xffu) << sh;
    }
    ys = pow2f(E - 22);
}

// The exact block dot from its three piece dots D_j = sum_i v_i * a_j,i:
// the float of D0*2^16 + D1*2^8 + D2 (|D_j| < 2^27), rounded once.  The sum
// is formed exactly in double (every partial is an integer below 2^44).
__device__ __forceinline__ float q6x_dot(int D0, int D1, int D2) {
    const double D = __fma_rn((double)D0, 65536.0, __fma_rn((double)D1, 256.0, (double)D2));
    return __double2float_rn(D);
}

}  // namespace g4
