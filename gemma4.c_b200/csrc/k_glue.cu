// k_glue.cu — the per-step glue of forward around the GEMVs and attention.
//
//   resnorm   x = (x + rmsnorm(delta)*w_post) * out_scale, then the next
//             pre-norm xn = rmsnorm(x)*w_pre and its Q8_K quantization
//             (residual chain of main.c:1959-2003, norms 1451-1456,
//             quantize_row_q8_K 282-340).  One CTA per sequence.
//   embed     token row of token_embd times sqrt(dim) and the per-layer
//             token row times sqrt(ple_dim) (main.c:1849-1854, 1753-1758,
//             emb_lookup 1696-1723).  The token comes from a token array or
//             straight from the previous step's argmax keys.
//   ple_mix   ple = (tok + rmsnorm(ctx / sqrt(dim)) * w) / sqrt(2) per layer
//             (build_ple, main.c:1760-1777).
#include <math.h>

#include "g4_internal.cuh"
#include "g4_kernels.cuh"
#include "g4_prologue.cuh"
#include "g4_quant.cuh"
#include "g4_tc.cuh"

namespace g4 {

__device__ __forceinline__ float cta_sum(float v, float *red) {
    v = warp_sum(v);
    const int nw = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; i++) t += red[i];
    return t;
}

// The tensor-core B operands (and Q8_K blocks) of the finished vector src[dim] of sequence b.
__device__ __forceinline__ void resnorm_operands(const ResNorm &r, const float *src, int b, bool q8) {
    const int nb = r.dim / G4_QK, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (q8) {
        uint8_t *q8o = (uint8_t *)r.q8_out + (size_t)b * nb * G4_Q8_BYTES;
        for (int k = warp; k < nb; k += nw) {
            uint32_t q[2];
            float d;
            int ls;
            warp_quant_block(src + k * G4_QK, lane, q, d, ls);
            store_q8_block(q8o + (size_t)k * G4_Q8_BYTES, lane, q, d, ls);
        }
    }
    if (r.tc4_bq)
        for (int k = warp; k < nb; k += nw) {
            uint32_t q[2];
            float d;
            int ls;
            warp_quant_block(src + k * G4_QK, lane, q, d, ls);
            tc4_store_q8(r.tc4_bq + (size_t)k * 544 * r.tc_np, r.tc4_yd + (size_t)k * r.tc_np, r.tc_np, b, lane, q, d, ls);
        }
    if (r.tc6_bq)
        for (int k = warp; k < nb; k += nw) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = src[k * G4_QK + 8 * lane + j];
            tc6_store_block(r.tc6_bq, r.tc6_ys, k, r.tc_np, b, lane, v, true);
        }
    if (r.bf3_bq)
        for (int g = warp; g < r.dim / kBfK; g += nw)
            bf3_store_group(r.bf3_bq, g, r.tc_np, b, lane, src[g * kBfK + 2 * lane], src[g * kBfK + 2 * lane + 1]);
}

// rmsnorm (main.c:1451-1456): o = (x * (1/sqrt(mean(x^2) + eps))) * w.
// 256 threads, one CTA per sequence; thread t owns elements t + 256k in
// registers, which is the element order of canon_sumsq, so the sums are those
// of the fused GEMV prologue.  The norm weights are loaded before the wait on
// the previous kernel and the residual inputs right after it, so the kernel
// makes one dependent trip to memory before its stores.
template <int NBM>
__global__ void __launch_bounds__(256) resnorm_reg_kernel(ResNorm r) {
    extern __shared__ __align__(16) float xs[];  // [dim] the finished vector (xn, or x without pre_w)
    __shared__ float red[8];
    pdl_trigger();
    const int b = blockIdx.x, dim = r.dim, t = threadIdx.x, nb = dim / G4_QK;
    float pw[NBM], qw[NBM], x[NBM], d[NBM];
#pragma unroll
    for (int k = 0; k < NBM; k++)
        if (k < nb) {
            pw[k] = r.delta ? __ldg(r.post_w + t + G4_QK * k) : 0.0f;
            qw[k] = r.pre_w ? __ldg(r.pre_w + t + G4_QK * k) : 0.0f;
        }
    pdl_wait();
    const float *xi = r.x_in + (size_t)b * dim;
    const float *dl = r.delta ? r.delta + (size_t)b * dim : nullptr;
#pragma unroll
    for (int k = 0; k < NBM; k++)
        if (k < nb) {
            x[k] = xi[t + G4_QK * k];
            d[k] = dl ? dl[t + G4_QK * k] : 0.0f;
        }
    auto tree = [&](float p) {  // canon_sumsq's reduction of the 256 per-thread chains
        p = warp_sum(p);
        __syncthreads();
        if ((t & 31) == 0) red[t >> 5] = p;
        __syncthreads();
        return ((red[0] + red[1]) + (red[2] + red[3])) + ((red[4] + red[5]) + (red[6] + red[7]));
    };
    if (dl) {
        float p = 0.0f;
#pragma unroll
        for (int k = 0; k < NBM; k++)
            if (k < nb) p = fmaf(d[k], d[k], p);
        const float ss = tree(p);
        const float inv = 1.0f / sqrtf(ss / (float)dim + r.eps);
#pragma unroll
        for (int k = 0; k < NBM; k++)
            if (k < nb) x[k] = __fadd_rn(x[k], __fmul_rn(__fmul_rn(d[k], inv), pw[k]));
    }
    if (r.scale) {
        const float sc = *r.scale;
#pragma unroll
        for (int k = 0; k < NBM; k++)
            if (k < nb) x[k] = __fmul_rn(x[k], sc);
    }
    if (r.x_out) {
        float *xo = r.x_out + (size_t)b * dim;
#pragma unroll
        for (int k = 0; k < NBM; k++)
            if (k < nb) xo[t + G4_QK * k] = x[k];
    }
    if (r.pre_w) {
        float p = 0.0f;
#pragma unroll
        for (int k = 0; k < NBM; k++)
            if (k < nb) p = fmaf(x[k], x[k], p);
        const float ss = tree(p);
        const float inv = 1.0f / sqrtf(ss / (float)dim + r.eps);
#pragma unroll
        for (int k = 0; k < NBM; k++)
            if (k < nb) {
                x[k] = __fmul_rn(__fmul_rn(x[k], inv), qw[k]);
                if (r.xn_out) r.xn_out[(size_t)b * dim + t + G4_QK * k] = x[k];
            }
    }
    const bool q8 = r.pre_w && r.q8_out;
    if (!q8 && !r.tc4_bq && !r.tc6_bq && !r.bf3_bq) return;
#pragma unroll
    for (int k = 0; k < NBM; k++)
        if (k < nb) xs[t + G4_QK * k] = x[k];
    __syncthreads();
    resnorm_operands(r, xs, b, q8);
}

// The same for any dim (the vector staged in shared memory), 512 threads.
__global__ void __launch_bounds__(512) resnorm_kernel(ResNorm r) {
    extern __shared__ __align__(16) float xs[];  // [dim] x, then [dim] xn
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x, dim = r.dim, tid = threadIdx.x;
    float *xn = xs + dim;
    const float *xi = r.x_in + (size_t)b * dim;
    for (int i = tid; i < dim; i += blockDim.x) xs[i] = xi[i];
    if (r.delta) {
        const float *dl = r.delta + (size_t)b * dim;
        const float ss = canon_sumsq(dl, dim, red);
        const float inv = 1.0f / sqrtf(ss / (float)dim + r.eps);
        for (int i = tid; i < dim; i += blockDim.x)
            xs[i] = __fadd_rn(xs[i], __fmul_rn(__fmul_rn(dl[i], inv), r.post_w[i]));
    }
    if (r.scale) {
        const float sc = *r.scale;
        for (int i = tid; i < dim; i += blockDim.x) xs[i] = __fmul_rn(xs[i], sc);
    }
    __syncthreads();
    if (r.x_out) {
        float *xo = r.x_out + (size_t)b * dim;
        for (int i = tid; i < dim; i += blockDim.x) xo[i] = xs[i];
    }
    if (r.pre_w) {
        const float ss = canon_sumsq(xs, dim, red);
        const float inv = 1.0f / sqrtf(ss / (float)dim + r.eps);
        for (int i = tid; i < dim; i += blockDim.x) {
            const float v = __fmul_rn(__fmul_rn(xs[i], inv), r.pre_w[i]);
            xn[i] = v;
            if (r.xn_out) r.xn_out[(size_t)b * dim + i] = v;
        }
    }
    const bool q8 = r.pre_w && r.q8_out;
    if (!q8 && !r.tc4_bq && !r.tc6_bq && !r.bf3_bq) return;
    __syncthreads();
    resnorm_operands(r, r.pre_w ? xn : xs, b, q8);
}

int launch_resnorm(const ResNorm &r, int B, cudaStream_t st) {
    if ((r.q8_out || r.tc4_bq || r.tc6_bq) && r.dim % G4_QK) { set_error(G4_ERR_ARG, "resnorm: dim %d not a multiple of 256", r.dim); return G4_ERR_ARG; }
    if (r.bf3_bq && r.dim % kBfK) { set_error(G4_ERR_ARG, "resnorm: dim %d not a multiple of %d", r.dim, kBfK); return G4_ERR_ARG; }
    if ((r.tc4_bq || r.tc6_bq || r.bf3_bq) && (B > r.tc_np || (r.tc_np != 16 && r.tc_np != 32 && r.tc_np != 64))) {
        set_error(G4_ERR_ARG, "resnorm: %d sequences in a tensor-core group of %d", B, r.tc_np);
        return G4_ERR_ARG;
    }
    if (r.dim % G4_QK == 0 && r.dim <= 16 * G4_QK) {
        G4_CUDA(launch_pdl(resnorm_reg_kernel<16>, dim3(B), dim3(256), (size_t)r.dim * 4, st, r));
        G4_LAUNCHED();
        return G4_OK;
    }
    const size_t smem = (size_t)r.dim * 8;
    if (smem > 100 * 1024) { set_error(G4_ERR_ARG, "resnorm: dim %d too large", r.dim); return G4_ERR_ARG; }
    G4_CUDA(launch_pdl(resnorm_kernel, dim3(B), dim3(512), smem, st, r));
    G4_LAUNCHED();
    return G4_OK;
}

// Element e of row `row` of a weight tensor with `ncols` columns, dequantized
// with the reference's float expressions (dequant_q4_k/q5_k/q6_k,
// main.c:172-237; f16/bf16 decode 128-156).  Q6_K uses the device planes.
__device__ __forceinline__ float weight_elem(const void *w, int type, int ncols, size_t nrows_total, long row, int e) {
    if (type == G4_F32) return ((const float *)w)[(size_t)row * ncols + e];
    if (type == G4_F16) return f16_to_f32(((const uint16_t *)w)[(size_t)row * ncols + e]);
    if (type == G4_BF16) return bf16_to_f32(((const uint16_t *)w)[(size_t)row * ncols + e]);
    const int nb = ncols / G4_QK, k = e / G4_QK, i = e % G4_QK;
    if (type == G4_Q6_K) {
        const Q6Row P = q6_row_at((const uint8_t *)w + (size_t)row * q6_row_bytes(nb), nb);
        const uint8_t *ql = (const uint8_t *)(P.ql + (size_t)k * 8);
        const uint8_t *qh = (const uint8_t *)(P.qh + (size_t)k * 4);
        const int8_t *sc = (const int8_t *)(P.sc + k);
        const int n6 = i / 128, r = i % 128, qd = r / 32, l = r % 32;
        const int qlb = ql[64 * n6 + (qd & 1) * 32 + l];
        const int lo = (qd >= 2) ? (qlb >> 4) : (qlb & 15);
        const int q = (lo | (((qh[32 * n6 + l] >> (2 * qd)) & 3) << 4)) - 32;
        const float d = f16_to_f32(P.d[k]);
        return __fmul_rn(__fmul_rn(d, (float)sc[8 * n6 + l / 16 + 2 * qd]), (float)q);
    }
    const size_t bb = type == G4_Q4_K ? 144 : 176;
    const uint8_t *blk = (const uint8_t *)w + ((size_t)row * nb + k) * bb;
    const uint16_t *dd = (const uint16_t *)blk;
    const uint32_t *s32 = (const uint32_t *)(blk + 4);
    const int c = i / 64, hi = (i / 32) & 1, l = i % 32;
    int sc, mn;
    k4_scale_min(2 * c + hi, s32[0], s32[1], s32[2], sc, mn);
    const uint8_t *qs = blk + (type == G4_Q4_K ? 16 : 48);
    int q = hi ? (qs[32 * c + l] >> 4) : (qs[32 * c + l] & 15);
    if (type == G4_Q5_K && ((blk[16 + l] >> (2 * c + hi)) & 1)) q += 16;
    const float d1 = __fmul_rn(f16_to_f32(dd[0]), (float)sc);
    const float m1 = __fmul_rn(f16_to_f32(dd[1]), (float)mn);
    return __fsub_rn(__fmul_rn(d1, (float)q), m1);
}

__global__ void embed_kernel(const void *embd, int embd_t, int dim, size_t vocab, float emb_scale, const void *ple_tok,
                             int ple_tok_t, int ple_row, float ple_scale, const int *tokens,
                             unsigned long long *keys, float *x, float *ple_out) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x;
    int tok = tokens ? tokens[b] : argmax_key_index(keys[b]);
    if (tok < 0 || (size_t)tok >= vocab) tok = 0;  // no LM-head result yet: never index out of the table
    __syncthreads();
    if (threadIdx.x == 0) keys[b] = 0ull;  // reset for this step's LM-head argmax
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        x[(size_t)b * dim + i] = __fmul_rn(weight_elem(embd, embd_t, dim, vocab, tok, i), emb_scale);
    if (ple_out)
        for (int i = threadIdx.x; i < ple_row; i += blockDim.x)
            ple_out[(size_t)b * ple_row + i] = __fmul_rn(weight_elem(ple_tok, ple_tok_t, ple_row, vocab, tok, i), ple_scale);
}

int launch_embed_v(const void *embd, int embd_t, int dim, size_t vocab, float emb_scale, const void *ple_tok,
                   int ple_tok_t, int ple_row, float ple_scale, const int *tokens, unsigned long long *keys,
                   float *x, float *ple_out, int B, cudaStream_t st) {
    G4_CUDA(launch_pdl(embed_kernel, dim3(B), dim3(512), 0, st, embd, embd_t, dim, vocab, emb_scale, ple_tok, ple_tok_t,
                       ple_row, ple_scale, tokens, keys, x, ple_out));
    G4_LAUNCHED();
    return G4_OK;
}

// build_ple mixing (main.c:1760-1777), one CTA per (layer, sequence).
__global__ void ple_mix_kernel(const float *ple_tok, const float *ple_ctx, const float *norm_w, int pd, int L,
                               float ctx_scale, float mix_scale, float eps, float *ple_out) {
    __shared__ float red[32];
    __shared__ float cs[1024];
    pdl_trigger();
    pdl_wait();
    const int l = blockIdx.x, b = blockIdx.y;
    const size_t off = (size_t)b * L * pd + (size_t)l * pd;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < pd; i += blockDim.x) {
        const float c = __fmul_rn(ple_ctx[off + i], ctx_scale);
        cs[i] = c;
        ss = fmaf(c, c, ss);
    }
    ss = cta_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)pd + eps);
    for (int i = threadIdx.x; i < pd; i += blockDim.x) {
        const float c = __fmul_rn(__fmul_rn(cs[i], inv), norm_w[i]);
        ple_out[off + i] = __fmul_rn(__fadd_rn(ple_tok[off + i], c), mix_scale);
    }
}

int launch_ple_mix(const float *ple_tok, float *ple_ctx, const float *norm_w, int pd, int L, float ctx_scale,
                   float mix_scale, float eps, float *ple_out, int B, cudaStream_t st) {
    if (pd > 1024) { set_error(G4_ERR_ARG, "ple_dim %d > 1024", pd); return G4_ERR_ARG; }
    G4_CUDA(launch_pdl(ple_mix_kernel, dim3(L, B), dim3(256), 0, st, ple_tok, (const float *)ple_ctx, norm_w, pd, L,
                       ctx_scale, mix_scale, eps, ple_out));
    G4_LAUNCHED();
    return G4_OK;
}

__global__ void keys_to_tokens_kernel(const unsigned long long *keys, int *tokens, int B) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) tokens[b] = argmax_key_index(keys[b]);
}

int launch_keys_to_tokens(const unsigned long long *keys, int *tokens, int B, cudaStream_t st) {
    G4_CUDA(launch_pdl(keys_to_tokens_kernel, dim3((B + 127) / 128), dim3(128), 0, st, keys, tokens, B));
    G4_LAUNCHED();
    return G4_OK;
}

}  // namespace g4

namespace g4 {

__global__ void gelu_mul_kernel(float *a, const float *b, size_t n) {
    pdl_trigger();
    pdl_wait();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = gelu_f32(a[i]) * b[i];
}

int launch_gelu_mul(float *a, const float *b, size_t n, cudaStream_t st) {
    G4_CUDA(launch_pdl(gelu_mul_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, a, b, n));
    G4_LAUNCHED();
    return G4_OK;
}

// Softcap in place (main.c:1790-1795) and first-max argmax per sequence
// (sample_token temp <= 0, main.c:2045-2050) for LM heads of dense types.
__global__ void softcap_argmax_kernel(float *logits, int vocab, int ld, float cap, unsigned long long *keys) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.y;
    float *lg = logits + (size_t)b * ld;
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x) {
        float v = lg[i];
        if (cap > 0.0f) { v = cap * tanhf(v * (1.0f / cap)); lg[i] = v; }
        const unsigned long long k = argmax_key(v, i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long ok = __shfl_xor_sync(0xffffffffu, best, o);
        best = ok > best ? ok : best;
    }
    if ((threadIdx.x & 31) == 0 && best) atomicMax(keys + b, best);
}

int launch_softcap_argmax(float *logits, int vocab, int ld, float cap, unsigned long long *keys, int B,
                          cudaStream_t st) {
    G4_CUDA(launch_pdl(softcap_argmax_kernel, dim3(148, B), dim3(256), 0, st, logits, vocab, ld, cap, keys));
    G4_LAUNCHED();
    return G4_OK;
}

// GGUF Q6_K blocks (210 B) -> device rows (ql | qh | scales | d planes per row).
__global__ void repack_q6_kernel(const uint8_t *raw, size_t nblk, size_t off, uint8_t *dst, int nb) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblk) return;
    const uint8_t *b = raw + i * 210;
    const size_t gi = off + i, row = gi / nb;
    const int k = (int)(gi % nb);
    uint8_t *r = dst + row * q6_row_bytes(nb);
    uint8_t *ql = r + (size_t)k * 128, *qh = r + (size_t)nb * 128 + (size_t)k * 64, *sc = r + (size_t)nb * 192 + (size_t)k * 16;
    uint16_t *d = reinterpret_cast<uint16_t *>(r + (size_t)nb * 208) + k;
    for (int j = 0; j < 128; j++) ql[j] = b[j];
    for (int j = 0; j < 64; j++) qh[j] = b[128 + j];
    for (int j = 0; j < 16; j++) sc[j] = b[192 + j];
    *d = (uint16_t)(b[208] | (b[209] << 8));
}

int launch_repack_q6(const void *raw_dev, size_t nblk, size_t blk_offset, void *planes_dev, int nb,
                     cudaStream_t st) {
    if (!nblk) return G4_OK;
    repack_q6_kernel<<<(unsigned)((nblk + 255) / 256), 256, 0, st>>>((const uint8_t *)raw_dev, nblk, blk_offset,
                                                                     (uint8_t *)planes_dev, nb);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

}  // namespace g4

namespace g4 {

// apply_rope_neox (main.c:1725-1745) with a precomputed (cos, sin) row.
__global__ void rope_kernel(float *vec, int hd, int n_rot, const float2 *cs) {
    float *seg = vec + (size_t)blockIdx.x * hd;
    const int half = hd / 2;
    for (int j = threadIdx.x; j < n_rot / 2; j += blockDim.x) {
        const float v0 = seg[j], v1 = seg[j + half];
        const float2 c = cs[j];
        seg[j] = __fsub_rn(__fmul_rn(v0, c.x), __fmul_rn(v1, c.y));
        seg[j + half] = __fadd_rn(__fmul_rn(v0, c.y), __fmul_rn(v1, c.x));
    }
}

int launch_rope(float *vec, int n_heads, int hd, int n_rot, const float2 *cs, cudaStream_t st) {
    if (n_rot < 2) return G4_OK;
    rope_kernel<<<n_heads, 128, 0, st>>>(vec, hd, n_rot, cs);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

// mm_quant_rows for Q4_K/Q5_K (main.c:1539-1556, the --f32-matmul debug
// path): dequantize each weight with the reference expression, fp32 dot.
__global__ void gemv_deq_kernel(const void *w, int type, int n, int rows, const float *x, float *out) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    float acc = 0.0f;
    for (int e = lane; e < n; e += 32) acc = fmaf(x[e], weight_elem(w, type, n, rows, warp, e), acc);
    acc = warp_sum(acc);
    if (lane == 0) out[warp] = acc;
}

int launch_gemv_deq(const void *w, int type, int n, int rows, const float *x, float *out, cudaStream_t st) {
    gemv_deq_kernel<<<(rows + 7) / 8, 256, 0, st>>>(w, type, n, rows, x, out);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

}  // namespace g4

namespace g4 {
int prime_gemv_attrs();
int prime_attn_attrs();
int prime_kernel_attrs() {
    G4_CUDA(cudaFuncSetAttribute(resnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024));
    int rc = prime_gemv_attrs();
    if (rc) return rc;
    if ((rc = prime_tc_attrs())) return rc;
    if ((rc = prime_tc6_attrs())) return rc;
    if ((rc = prime_bf16tc_attrs())) return rc;
    return prime_attn_attrs();
}
}  // namespace g4

namespace g4 {

// Seeded values in [-1, 1) for KV rows [0, npos) of one cache (a splitmix64
// hash of the element index), so a benchmark can start decoding at a long
// context without running the prefill; a decode step's cost does not depend
// on the cached values.
__global__ void fill_kv_kernel(float *c, size_t rows_per_head, int ring, int hd, int npos, size_t total, uint64_t seed) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const size_t head_row = i / hd;                 // (b, h, slot) row index
    const int slot = (int)(head_row % ring);
    if (slot >= npos && npos < ring) return;
    uint64_t z = seed + 0x9E3779B97F4A7C15ull * (i + 1);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    c[i] = (float)(z >> 40) * (2.0f / 16777216.0f) - 1.0f;
    (void)rows_per_head;
}

int launch_fill_kv(float *c, int B, int n_kv, int ring, int hd, int npos, uint64_t seed, cudaStream_t st) {
    const size_t total = (size_t)B * n_kv * ring * hd;
    if (!total) return G4_OK;
    fill_kv_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(c, (size_t)ring, ring, hd, npos, total, seed);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

}  // namespace g4
