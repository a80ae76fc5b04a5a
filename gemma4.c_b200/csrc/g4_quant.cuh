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
