// k_attn.cu — ISWA decode attention with Neox RoPE and shared KV.
//
// Reference: the attention block of forward (gemma4-4b/cpu-blas/main.c:
// 1878-1950): q/k per-head RMSNorm (1458-1466), v RMSNorm without weight
// (1468-1476), Neox RoPE (1725-1745), KV store (1901-1904), the window
// t_start = max(0, pos+1-window) for sliding-window layers (1909-1915), and per
// q head h: scores over the kv head h/(n_heads/n_kv) rows of the source
// layer's cache (scale 1), max-subtracted softmax (1478-1488) and the
// probability-weighted sum of V rows.  Layers >= 24 read layer 22 (sliding)
// or 23 (global) and store nothing (main.c:739-746).
//
// Device layout of a KV layer: K and V each [B][n_kv][slots][hd] fp32, where
// slots = the window (ring buffer, slot = pos % window) for sliding-window
// layers and max_seq (slot = pos) for global ones.  A ring reads the same
// logical rows in the same logical order as the reference's linear cache.
//
// Kernels:
//   attn_prep     per (head, sequence): q-norm + RoPE into qn; for layers
//                 that store KV, k-norm + RoPE and v-norm into the cache slot.
//   attn_decode   split-K flash-decoding: a CTA owns (chunk of 64 positions,
//                 kv head, sequence) and all G query heads of that kv head,
//                 so each K/V row is read from HBM once per step.
//   attn_combine  merges the chunk partials (max, sum, unnormalised output).
// The position is read from device memory so one CUDA graph serves all
// positions; the grid covers the largest window and idle chunks exit.
#include <math.h>

#include "g4_internal.cuh"
#include "g4_kernels.cuh"

namespace g4 {

constexpr int kChunk = 64;
int attn_chunk_size() { return kChunk; }

// Reference-exact RoPE angles (apply_rope_neox, main.c:1725-1745): theta
// starts at pos and is multiplied by theta_scale = powf(base, -2/n_rot) once
// per pair; angle = freq_scale * theta / ff[j].  cosf/sinf/powf are the host
// libm's, as in the reference, so the table matches it bit for bit.
void rope_table_host(float2 *out, int npos, int n_rot, float base, float freq_scale, const float *ff) {
    const float theta_scale = powf(base, -2.0f / (float)n_rot);
    const int half = n_rot / 2;
    for (int p = 0; p < npos; p++) {
        float theta = (float)p;
        for (int j = 0; j < half; j++) {
            const float f = ff ? ff[j] : 1.0f;
            const float angle = freq_scale * theta / f;
            out[(size_t)p * half + j] = make_float2(cosf(angle), sinf(angle));
            theta *= theta_scale;
        }
    }
}

// Sum over the whole CTA (any blockDim.x that is a multiple of 32, <= 1024).
__device__ __forceinline__ float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int nw = blockDim.x >> 5;
    if (nw == 1) return v;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; i++) t += red[i];
    return t;
}

// One CTA per (head, sequence); thread j owns the RoPE pair (j, j + hd/2).
__global__ void attn_prep_kernel(AttnLayer L, const float *__restrict__ q, const float *__restrict__ k,
                                 const float *__restrict__ v, float *__restrict__ qn, const int *__restrict__ pos_dev) {
    __shared__ float red[32];
    const int hd = L.hd, half = hd / 2, j = threadIdx.x;
    const int head = blockIdx.x, b = blockIdx.y;
    const int pos = *pos_dev;
    const bool is_q = head < L.n_heads;
    const int kvh = head - L.n_heads;
    const int qd = L.n_heads * hd, kvd = L.n_kv * hd;
    const float *src = is_q ? q + (size_t)b * qd + (size_t)head * hd : k + (size_t)b * kvd + (size_t)kvh * hd;
    float v0 = src[j], v1 = src[j + half];
    // per-head RMSNorm, seg[i] *= ss * w[i] (main.c:1458-1466)
    const float ss = block_sum(v0 * v0 + v1 * v1, red);
    const float inv = 1.0f / sqrtf(ss / (float)hd + L.eps);
    const float *w = is_q ? L.q_norm : L.k_norm;
    v0 = v0 * (inv * w[j]);
    v1 = v1 * (inv * w[j + half]);
    if (j < L.n_rot / 2) {  // Neox rotation, products rounded separately like the reference
        const float2 cs = L.rope[(size_t)pos * (L.n_rot / 2) + j];
        const float r0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
        const float r1 = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
        v0 = r0;
        v1 = r1;
    }
    if (is_q) {
        float *dst = qn + (size_t)b * qd + (size_t)head * hd;
        dst[j] = v0;
        dst[j + half] = v1;
        return;
    }
    // K row, then the V row normalised without weight (main.c:1468-1476)
    const int slot = pos % L.ring;
    const size_t row = (((size_t)b * L.n_kv + kvh) * L.ring + slot) * hd;
    L.kc[row + j] = v0;
    L.kc[row + j + half] = v1;
    const float *vs = v + (size_t)b * kvd + (size_t)kvh * hd;
    float u0 = vs[j], u1 = vs[j + half];
    const float vss = block_sum(u0 * u0 + u1 * u1, red);
    const float vinv = 1.0f / sqrtf(vss / (float)hd + L.eps);
    L.vc[row + j] = u0 * vinv;
    L.vc[row + j + half] = u1 * vinv;
}

int launch_attn_prep(const AttnLayer &L, const float *q, const float *k, const float *v, float *qn, int B,
                     const int *pos_dev, int max_seq, cudaStream_t st) {
    (void)max_seq;
    if (L.hd % 64 || L.hd > 512) { set_error(G4_ERR_ARG, "attention: head_dim %d unsupported", L.hd); return G4_ERR_ARG; }
    const int heads = L.n_heads + (L.append ? L.n_kv : 0);
    attn_prep_kernel<<<dim3(heads, B), L.hd / 2, 0, st>>>(L, q, k, v, qn, pos_dev);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

// Partial record of one (sequence, q head, chunk): m, l, o[hd].
__host__ __device__ inline size_t part_stride(int hd) { return (size_t)hd + 2; }

template <int EPL>
__device__ __forceinline__ void load_row(float (&dst)[EPL], const float *src) {
    if constexpr (EPL % 4 == 0) {
#pragma unroll
        for (int e = 0; e < EPL; e += 4) {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(src + e));
            dst[e] = a.x; dst[e + 1] = a.y; dst[e + 2] = a.z; dst[e + 3] = a.w;
        }
    } else {
#pragma unroll
        for (int e = 0; e < EPL; e += 2) {
            const float2 a = __ldg(reinterpret_cast<const float2 *>(src + e));
            dst[e] = a.x; dst[e + 1] = a.y;
        }
    }
}

template <int EPL, int G>
constexpr size_t decode_smem_bytes() {
    return sizeof(float) * ((size_t)8 * G * EPL * 32 + (size_t)G * kChunk + 2 * G);
}

template <int EPL, int G>
__global__ void __launch_bounds__(256) attn_decode_kernel(AttnLayer L, const float *__restrict__ qn,
                                                          float *__restrict__ part, int max_chunks,
                                                          const int *__restrict__ pos_dev) {
    constexpr int HD = EPL * 32;
    extern __shared__ __align__(16) float dsm[];
    float(*red)[G][HD] = reinterpret_cast<float(*)[G][HD]>(dsm);           // [8][G][HD]
    float(*sc)[kChunk] = reinterpret_cast<float(*)[kChunk]>(dsm + 8 * G * HD);  // [G][kChunk]
    float(*ml)[2] = reinterpret_cast<float(*)[2]>(dsm + 8 * G * HD + G * kChunk);
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = *pos_dev;
    int t0 = 0;
    if (L.window > 0) { t0 = pos + 1 - L.window; if (t0 < 0) t0 = 0; }
    const int nwin = pos + 1 - t0;
    const int cbeg = c * kChunk;
    if (cbeg >= nwin) return;
    const int cnt = min(kChunk, nwin - cbeg);

    float qv[G][EPL];
#pragma unroll
    for (int g = 0; g < G; g++)
        load_row<EPL>(qv[g], qn + ((size_t)b * L.n_heads + (size_t)h * G + g) * HD + lane * EPL);
    const size_t head_base = ((size_t)b * L.n_kv + h) * L.src_ring;
    // scores: one warp per cached row
    for (int tl = warp; tl < cnt; tl += 8) {
        const int t = t0 + cbeg + tl;
        const float *kr = L.src_kc + (head_base + (size_t)(t % L.src_ring)) * HD + lane * EPL;
        float kv[EPL];
        load_row<EPL>(kv, kr);
#pragma unroll
        for (int g = 0; g < G; g++) {
            float s = 0.0f;
#pragma unroll
            for (int e = 0; e < EPL; e++) s = fmaf(kv[e], qv[g][e], s);
            s = warp_sum(s);
            if (lane == 0) sc[g][tl] = s;
        }
    }
    __syncthreads();
    // chunk softmax statistics, one warp per query head
    if (warp < G) {
        float m = -INFINITY;
        for (int tl = lane; tl < cnt; tl += 32) m = fmaxf(m, sc[warp][tl]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int tl = lane; tl < cnt; tl += 32) {
            const float p = expf(sc[warp][tl] - m);
            sc[warp][tl] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) { ml[warp][0] = m; ml[warp][1] = l; }
    }
    __syncthreads();
    // unnormalised P.V over the chunk
    float acc[G][EPL];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[g][e] = 0.0f;
    for (int tl = warp; tl < cnt; tl += 8) {
        const int t = t0 + cbeg + tl;
        const float *vr = L.src_vc + (head_base + (size_t)(t % L.src_ring)) * HD + lane * EPL;
        float vv[EPL];
        load_row<EPL>(vv, vr);
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float p = sc[g][tl];
#pragma unroll
            for (int e = 0; e < EPL; e++) acc[g][e] = fmaf(p, vv[e], acc[g][e]);
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < EPL; e++) red[warp][g][lane * EPL + e] = acc[g][e];
    __syncthreads();
    for (int i = threadIdx.x; i < G * HD; i += 256) {
        const int g = i / HD, d = i % HD;
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) o += red[w][g][d];
        float *pr = part + (((size_t)b * L.n_heads + (size_t)h * G + g) * max_chunks + c) * part_stride(HD);
        pr[2 + d] = o;
        if (d == 0) { pr[0] = ml[g][0]; pr[1] = ml[g][1]; }
    }
}

// One CTA per (q head, sequence): merge the chunk partials.
__global__ void attn_combine_kernel(AttnLayer L, const float *__restrict__ part, float *__restrict__ qo,
                                    int max_chunks, const int *__restrict__ pos_dev) {
    extern __shared__ float wts[];  // [max_chunks]
    __shared__ float invL;
    const int h = blockIdx.x, b = blockIdx.y, hd = L.hd;
    const int pos = *pos_dev;
    int t0 = 0;
    if (L.window > 0) { t0 = pos + 1 - L.window; if (t0 < 0) t0 = 0; }
    const int nwin = pos + 1 - t0;
    const int nch = (nwin + kChunk - 1) / kChunk;
    const float *base = part + ((size_t)b * L.n_heads + h) * max_chunks * part_stride(hd);
    if (threadIdx.x == 0) {
        float M = -INFINITY;
        for (int c = 0; c < nch; c++) M = fmaxf(M, base[c * part_stride(hd)]);
        float S = 0.0f;
        for (int c = 0; c < nch; c++) {
            const float w = expf(base[c * part_stride(hd)] - M);
            wts[c] = w;
            S = fmaf(w, base[c * part_stride(hd) + 1], S);
        }
        invL = 1.0f / S;
    }
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.0f;
        for (int c = 0; c < nch; c++) o = fmaf(wts[c], base[c * part_stride(hd) + 2 + d], o);
        qo[(size_t)b * L.n_heads * hd + (size_t)h * hd + d] = o * invL;
    }
}

template <int EPL, int G>
static int launch_decode_eg(dim3 grid, const AttnLayer &L, const float *qn, float *part, int max_chunks,
                            const int *pos_dev, cudaStream_t st) {
    const size_t smem = decode_smem_bytes<EPL, G>();
    attn_decode_kernel<EPL, G><<<grid, 256, smem, st>>>(L, qn, part, max_chunks, pos_dev);
    return G4_OK;
}

template <int EPL>
static int launch_decode_g(const AttnLayer &L, int G, dim3 grid, const float *qn, float *part, int max_chunks,
                           const int *pos_dev, cudaStream_t st) {
    switch (G) {
    case 1: return launch_decode_eg<EPL, 1>(grid, L, qn, part, max_chunks, pos_dev, st);
    case 2: return launch_decode_eg<EPL, 2>(grid, L, qn, part, max_chunks, pos_dev, st);
    case 4: return launch_decode_eg<EPL, 4>(grid, L, qn, part, max_chunks, pos_dev, st);
    default: set_error(G4_ERR_ARG, "attention: GQA group %d unsupported", G); return G4_ERR_ARG;
    }
}

int launch_attn_decode(const AttnLayer &L, const float *qn, float *part, float *qo, int B, const int *pos_dev,
                       int max_chunks, int max_seq, cudaStream_t st) {
    const int G = L.n_heads / L.n_kv;
    if (L.n_heads % L.n_kv) { set_error(G4_ERR_ARG, "attention: n_heads %% n_kv != 0"); return G4_ERR_ARG; }
    const int span = L.window > 0 ? (L.window < max_seq ? L.window : max_seq) : max_seq;
    const int nch = (span + kChunk - 1) / kChunk;
    if (nch > max_chunks) { set_error(G4_ERR_ARG, "attention: %d chunks > scratch %d", nch, max_chunks); return G4_ERR_ARG; }
    dim3 grid(nch, L.n_kv, B);
    int rc;
    switch (L.hd) {
    case 64: rc = launch_decode_g<2>(L, G, grid, qn, part, max_chunks, pos_dev, st); break;
    case 128: rc = launch_decode_g<4>(L, G, grid, qn, part, max_chunks, pos_dev, st); break;
    case 256: rc = launch_decode_g<8>(L, G, grid, qn, part, max_chunks, pos_dev, st); break;
    case 512: rc = launch_decode_g<16>(L, G, grid, qn, part, max_chunks, pos_dev, st); break;
    default: set_error(G4_ERR_ARG, "attention: head_dim %d unsupported", L.hd); return G4_ERR_ARG;
    }
    if (rc) return rc;
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    attn_combine_kernel<<<dim3(L.n_heads, B), 128, (size_t)max_chunks * 4, st>>>(L, part, qo, max_chunks, pos_dev);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

}  // namespace g4

namespace g4 {
template <int EPL, int G>
static int prime_one() {
    G4_CUDA(cudaFuncSetAttribute(attn_decode_kernel<EPL, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)decode_smem_bytes<EPL, G>()));
    return G4_OK;
}
int prime_attn_attrs() {
    int rc = 0;
    rc |= prime_one<2, 1>(); rc |= prime_one<2, 2>(); rc |= prime_one<2, 4>();
    rc |= prime_one<4, 1>(); rc |= prime_one<4, 2>(); rc |= prime_one<4, 4>();
    rc |= prime_one<8, 1>(); rc |= prime_one<8, 2>(); rc |= prime_one<8, 4>();
    rc |= prime_one<16, 1>(); rc |= prime_one<16, 2>(); rc |= prime_one<16, 4>();
    return rc ? G4_ERR_CUDA : G4_OK;
}
}  // namespace g4
