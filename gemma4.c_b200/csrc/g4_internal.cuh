// g4_internal.cuh — shared device/host internals of libg4b200 (sm_100a).
//
// Weight tensors keep the GGUF super-block layouts of
// gemma4-4b/cpu-blas/main.c:95-115 in HBM (Q4_K 144 B and Q5_K 176 B blocks
// are multiples of 16 B, so rows are 16-byte aligned), except Q6_K: its
// 210-byte blocks are not, so each row of a Q6_K tensor is stored as four
// planes (ql, qh, scales, d) padded to a multiple of 16 B (see q6_row_bytes).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/g4b200.h"

#define G4_QK 256
#define G4_Q8_BYTES 292
#define G4_N_LAYER_KV 24  // layers 0..23 store KV, main.c:77

namespace g4 {

// ---------------------------------------------------------------- errors
void set_error(int code, const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what, const char *file, int line);
#define G4_CUDA(call)                                                       \
    do {                                                                    \
        cudaError_t e_ = (call);                                            \
        if (e_ != cudaSuccess) return ::g4::cuda_fail(e_, #call, __FILE__, __LINE__); \
    } while (0)
#define G4_LAUNCHED() ::g4::note_launch()
void note_launch();

inline size_t block_bytes(int type) {
    return type == G4_Q4_K ? 144 : type == G4_Q5_K ? 176 : type == G4_Q6_K ? 210 : 0;
}
inline size_t row_bytes(int type, int n) {
    if (type == G4_F32) return (size_t)n * 4;
    if (type == G4_F16 || type == G4_BF16) return (size_t)n * 2;
    return (size_t)(n / G4_QK) * block_bytes(type);
}
inline bool type_known(int t) {
    return t == G4_F32 || t == G4_F16 || t == G4_BF16 || t == G4_Q4_K || t == G4_Q5_K || t == G4_Q6_K;
}
inline bool is_q8_type(int t) { return t == G4_Q4_K || t == G4_Q5_K; }  // is_q8_mm_type, main.c:615-617

// Device copy of a Q6_K tensor: each row of nb super-blocks is stored as four
// planes, ql[nb][128] | qh[nb][64] | scales[nb][16] | d[nb] (padded to 16 B),
// the same bytes as the GGUF blocks but with every row contiguous and 16-byte
// aligned, so a tile of rows moves with one bulk copy and 128-bit loads.
__host__ __device__ inline size_t q6_row_bytes(int nb) {
    return (size_t)nb * 208 + (((size_t)nb * 2 + 15) & ~(size_t)15);
}
struct Q6Row {
    const uint4 *ql;
    const uint4 *qh;
    const uint4 *sc;
    const uint16_t *d;
};
__host__ __device__ inline Q6Row q6_row_at(const void *row_base, int nb) {
    const uint8_t *r = (const uint8_t *)row_base;
    Q6Row q;
    q.ql = (const uint4 *)r;
    q.qh = (const uint4 *)(r + (size_t)nb * 128);
    q.sc = (const uint4 *)(r + (size_t)nb * 192);
    q.d = (const uint16_t *)(r + (size_t)nb * 208);
    return q;
}
// Device byte size of a weight tensor of `rows` rows of `n` elements.
inline size_t device_tensor_bytes(int type, int n, int rows) {
    if (type == G4_Q6_K) return q6_row_bytes(n / G4_QK) * (size_t)rows;
    return row_bytes(type, n) * (size_t)rows;
}
// Device bytes of one row (the stride between rows on the device).
__host__ __device__ inline size_t device_row_bytes(int type, int n) {
    if (type == G4_Q6_K) return q6_row_bytes(n / G4_QK);
    if (type == G4_F32) return (size_t)n * 4;
    if (type == G4_F16 || type == G4_BF16) return (size_t)n * 2;
    return (size_t)(n / G4_QK) * (type == G4_Q4_K ? 144 : 176);
}

// Host -> device upload of one weight tensor (Q6_K rows split into planes).
int upload_tensor(void *dst_dev, const void *src_host, int type, int n, int rows, cudaStream_t st);

// ---------------------------------------------------------------- programmatic dependent launch
// Every kernel of the decode step is launched with programmatic stream
// serialization: it lets the next kernel be scheduled as soon as all of its
// own CTAs are running (pdl_trigger at entry), and waits for the previous
// kernel's results (pdl_wait) only before its first dependent global access.
// Work that reads nothing produced upstream (weight prefetch, barrier setup)
// runs before the wait and overlaps the previous kernel's tail.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ float f16_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ float bf16_to_f32(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

template <int W = 32>
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o, W);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// 6-bit scale and min of sub-block j of a Q4_K/Q5_K block (the bit packing
// of get_scale_min_k4, main.c:162-170).  s0/s1/s2 are scale bytes 0-3/4-7/8-11.
__device__ __forceinline__ void k4_scale_min(int j, uint32_t s0, uint32_t s1, uint32_t s2, int &sc, int &mn) {
    if (j < 4) {
        sc = (s0 >> (8 * j)) & 63;
        mn = (s1 >> (8 * j)) & 63;
    } else {
        const int i = j - 4;
        const uint32_t b8 = (s2 >> (8 * i)) & 0xff;       // byte j+4
        sc = (int)((b8 & 15) | (((s0 >> (8 * i + 6)) & 3) << 4));
        mn = (int)((b8 >> 4) | (((s1 >> (8 * i + 6)) & 3) << 4));
    }
}

// tanh-approximation GELU with the reference's constants and expression order
// (gelu_f32, main.c:1490-1492).
__device__ __forceinline__ float gelu_f32(float x) {
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * x * (1.0f + 0.044715f * x * x)));
}

// Packed (value, index) key whose unsigned max is the largest value with the
// LOWEST index among equals: the first-max rule of sample_token
// (main.c:2045-2050).  NaN is not expected (softcapped logits are finite).
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t b = __float_as_uint(v);
    if ((b & 0x7fffffffu) == 0u) b = 0u;               // -0 and +0 compare equal, as floats do
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // order-preserving map
    return ((unsigned long long)b << 32) | (uint32_t)(0xffffffffu - (uint32_t)idx);
}
__host__ __device__ inline int argmax_key_index(unsigned long long k) {
    return (int)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
}
// The key of a row-split LM head slice that starts at row row0, as a key over the whole vocabulary
// (0 = no row stays 0): the value part is unchanged, the index becomes row0 + local index, so the
// largest key over all slices is the first index of the largest logit.
__host__ __device__ inline unsigned long long lm_key_global(unsigned long long k, int row0) {
    if (!k) return 0ull;
    const uint32_t idx = 0xffffffffu - (uint32_t)(k & 0xffffffffu);
    return (k & 0xffffffff00000000ull) | (unsigned long long)(0xffffffffu - (idx + (uint32_t)row0));
}
// Merge of a row-split LM head for the B sequences of rank `rank`: keys_all[rr][world*B] are the
// slice keys of rank rr (slice rr starts at row rr*chunk) for every rank's sequences.
__host__ __device__ inline unsigned long long lm_split_merge_one(const unsigned long long *keys_all, int world,
                                                                int rank, int B, int chunk, int b) {
    unsigned long long best = 0ull;
    for (int rr = 0; rr < world; rr++) {
        const unsigned long long k = lm_key_global(keys_all[(size_t)rr * world * B + (size_t)rank * B + b], rr * chunk);
        best = k > best ? k : best;
    }
    return best;
}

}  // namespace g4
