// g4_tc.cuh — pieces shared by the tensor-core (tcgen05) GEMM kernels:
// launch arguments, packed fp16x2 / fp32x2 arithmetic.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "g4_async.cuh"
#include "g4_internal.cuh"
#include "g4_quant.cuh"

namespace g4 {

// Split row tiles one CTA of a tensor-core GEMM may have to merge after its units.
constexpr int kTcMergeCap = 16;
// Sequences per MMA pass of gemm_q6tc for a group of NP sequences (the B operand rows of one pass
// are 3 pieces x tc6_npp(NP)).
__host__ __device__ constexpr int tc6_npp(int NP) { return NP < 32 ? NP : 32; }

struct TcArgs {
    const uint8_t *w;   // weight rows (device layout), row_bytes apart
    size_t row_bytes;
    const uint8_t *bq;  // [nb][320*NP]: q8 quants (core-matrix layout) then the bsum operand
    const float *yd;    // [nb][NP] Q8_K block scales (0 for padding sequences)
    float *out;         // [B][ldo]
    float *part;        // split partials: [ksplit][NP][rows] (K slices), or [slot][NP][prow]
                        // (gemm_q4tc stream-K: one slot per CTA sharing a row tile)
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
    int *tickets;               // per row tile, zero between launches: the last CTA to finish a split
                                // tile merges its partial slots (null: a separate merge launch)
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

// B operand of gemm_q4tc for super-block k: q8 as fp16, K-major core
// matrices (byte (k'/8)*(NP*16) + s*16 + (k'%8)*2, k' = weight index with
// positions 1 and 2 of every 4 swapped), then bsums[16] as fp16 (byte
// 512*NP + (t/8)*(NP*16) + s*16 + (t%8)*2).
__device__ __forceinline__ void tc4_store_q8(uint8_t *blk, float *ydk, int NP, int s, int lane, const uint32_t q[2],
                                             float d, int ls) {
    int v[8];
#pragma unroll
    for (int b = 0; b < 4; b++) {
        v[b] = (int)(int8_t)(q[0] >> (8 * b));
        v[4 + b] = (int)(int8_t)(q[1] >> (8 * b));
    }
    const uint4 o = make_uint4(h_of_int(v[0]) | (h_of_int(v[2]) << 16), h_of_int(v[1]) | (h_of_int(v[3]) << 16),
                               h_of_int(v[4]) | (h_of_int(v[6]) << 16), h_of_int(v[5]) | (h_of_int(v[7]) << 16));
    *reinterpret_cast<uint4 *>(blk + (size_t)lane * (NP * 16) + s * 16) = o;
    const int b16 = ls + __shfl_xor_sync(0xffffffffu, ls, 1);  // lanes 2t, 2t+1: elements 16t..16t+15
    if ((lane & 1) == 0) {
        const int t = lane >> 1;
        *reinterpret_cast<uint16_t *>(blk + 512 * NP + (t >> 3) * (NP * 16) + s * 16 + (t & 7) * 2) =
            (uint16_t)h_of_int(b16);
    }
    if (lane == 0) ydk[s] = d;
}

// B operand of gemm_q6tc for super-block k (768*NP bytes): the three fixed-point pieces of every
// sequence's block (q6x_block) as int8 K-major core matrices,
//   byte (kk/16)*(3*NP*16) + row*16 + kk%16,   row = (s/NPP)*3*NPP + j*NPP + s%NPP
// (MMA pass s/NPP, then piece j, then sequence; NPP = tc6_npp(NP)), from this lane's elements
// 8*lane .. 8*lane+7 (one warp per block and sequence).  ys[k][s] = 2^(E-22) (0 when !valid).
__device__ __forceinline__ void tc6_store_block(uint8_t *bq, float *ys, int k, int NP, int s, int lane, const float (&v)[8],
                                                bool valid) {
    float w[8];
#pragma unroll
    for (int j = 0; j < 8; j++) w[j] = valid ? v[j] : 0.0f;
    uint32_t p[6];
    float y;
    q6x_block(w, p, y);
    const int npp = tc6_npp(NP), pass = s / npp, sl = s % npp;
    uint8_t *blk = bq + (size_t)k * 768 * NP + (size_t)(lane >> 1) * (3 * NP * 16) + 8 * (lane & 1);
#pragma unroll
    for (int j = 0; j < 3; j++)
        *reinterpret_cast<uint2 *>(blk + (size_t)((pass * 3 + j) * npp + sl) * 16) = make_uint2(p[2 * j], p[2 * j + 1]);
    if (lane == 0) ys[(size_t)k * NP + s] = valid ? y : 0.0f;
}

// B operand of gemm_bf16tc for the 64-element group g of sequence s, from this lane's elements
// 2*lane, 2*lane+1 (one warp per group and sequence): x = x1 + x2 + x3 in bf16 (remainders exact in
// fp32), rows q*NP + s of K-major core matrices.
constexpr int kBfK = 64;  // weights per group (one pipeline stage of gemm_bf16tc)
__device__ __forceinline__ void bf3_store_group(uint8_t *bq, int g, int NP, int s, int lane, float v0, float v1) {
    uint8_t *blk = bq + (size_t)g * 3 * NP * kBfK * 2;
    const int k = 2 * lane;
    uint16_t p0[3], p1[3];
    float r0 = v0, r1 = v1;
#pragma unroll
    for (int q = 0; q < 3; q++) {  // remainders are exact in fp32
        const __nv_bfloat16 a0 = __float2bfloat16_rn(r0), a1 = __float2bfloat16_rn(r1);
        p0[q] = __bfloat16_as_ushort(a0);
        p1[q] = __bfloat16_as_ushort(a1);
        r0 -= __bfloat162float(a0);
        r1 -= __bfloat162float(a1);
    }
#pragma unroll
    for (int q = 0; q < 3; q++)
        *reinterpret_cast<uint32_t *>(blk + (k >> 3) * (3 * NP * 16) + (q * NP + s) * 16 + (k & 7) * 2) =
            (uint32_t)p0[q] | ((uint32_t)p1[q] << 16);
}

// Merge of split partials for G consecutive sequences of one output element:
// v[s] = ((0 + P_0) + P_1) + ... + P_{ns-1}, slot k of sequence s at
// p0[k * slot_stride + s * seq_stride].  The loads of a batch of slots are all
// issued before the adds (the partials sit in L2), so a merge costs about one
// L2 round trip per batch instead of one per slot and sequence; the additions
// keep the slot order.
template <int G>
__device__ __forceinline__ void slot_sums(const float *p0, size_t slot_stride, size_t seq_stride, int ns, float (&v)[G]) {
    constexpr int KU = G >= 16 ? 1 : 16 / G;  // slots per batch: 16 loads in flight
#pragma unroll
    for (int s = 0; s < G; s++) v[s] = 0.0f;
    for (int k0 = 0; k0 < ns; k0 += KU) {
        float t[KU][G];
#pragma unroll
        for (int u = 0; u < KU; u++)
            if (k0 + u < ns)
#pragma unroll
                for (int s = 0; s < G; s++) t[u][s] = __ldcg(p0 + (size_t)(k0 + u) * slot_stride + (size_t)s * seq_stride);
#pragma unroll
        for (int u = 0; u < KU; u++)
            if (k0 + u < ns)
#pragma unroll
                for (int s = 0; s < G; s++) v[s] = __fadd_rn(v[s], t[u][s]);
    }
}

}  // namespace g4
