// g4_tc.cuh — pieces shared by the tensor-core (tcgen05) GEMM kernels:
// launch arguments, packed fp16x2 / fp32x2 arithmetic.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "g4_async.cuh"
#include "g4_internal.cuh"

namespace g4 {

struct TcArgs {
    const uint8_t *w;   // weight rows (device layout), row_bytes apart
    size_t row_bytes;
    const uint8_t *bq;  // [nb][320*NP]: q8 quants (core-matrix layout) then the bsum operand
    const float *yd;    // [nb][NP] Q8_K block scales (0 for padding sequences)
    float *out;         // [B][ldo]
    float *part;        // [ksplit][NP][rows] slice partials (ksplit > 1)
    int *tickets;       // [row_tiles][8], zero between launches
    int *err;
    int nb, rows, B, ldo;
    int ksplit, kslice, units;
    int epi;                    // EPI_STORE, or EPI_SOFTCAP_ARGMAX (logits: out may be null)
    float cap;                  // softcap of EPI_SOFTCAP_ARGMAX
    unsigned long long *keys;   // [B] argmax keys of EPI_SOFTCAP_ARGMAX (atomicMax)
    // gemm_q4tc_kernel only: stream-K work split over the (row tile, super-block) units of up to
    // two matrices that share the activation (gate and up, or Q and K).
    const uint8_t *w2;          // second matrix: row tiles tiles0.. of the launch (null: none)
    float *out2;                // [B][ldo2]
    int rows2, ldo2, tiles0;
    int share;                  // consecutive units per CTA (tile-major, super-block minor)
    int total;                  // all tiles * nb
    int prow;                   // rows of a partial slice: all tiles * 128
    int all_part;               // 1: every tile goes through the partial slots (merge epilogue)
};

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hadd2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// fp16 bit pattern of the integer v (exact for |v| <= 2048 and for multiples of 1024 below 65536)
__device__ __forceinline__ uint32_t h_of_int(int v) { return (uint32_t)__half_as_ushort(__int2half_rn(v)); }

// packed fp32 pairs (two lanes of work per instruction)
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ unsigned long long f2_pack_u(uint32_t lo, uint32_t hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}

}  // namespace g4
