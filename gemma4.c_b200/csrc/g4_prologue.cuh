// g4_prologue.cuh — residual/norm glue fused into the prologue of a GEMV.
//
// At batch <= 8 every CTA of a GEMV recomputes, from the residual stream in
// L2, the activation it multiplies: x' = (x + rmsnorm(delta)*w_post) * scale,
// then act = rmsnorm(x')*w_pre (or x'), quantized to Q8_K when the weights
// are Q4_K/Q5_K (forward, main.c:1878-1886, 1959-1975, 1999-2003; rmsnorm
// 1451-1456; quantize_row_q8_K 282-340).  One CTA (the launch's writer)
// stores x' for later kernels.  The CTA issues its first weight loads before
// running this, so the glue costs no extra launch and hides under the loads.
#pragma once
#include "g4_internal.cuh"
#include "g4_quant.cuh"

namespace g4 {

struct Prologue {
    const float *x_in;    // [B][dim] residual stream (or the plain activation)
    const float *delta;   // [B][dim] sublayer output to normalise and add, or null
    const float *post_w;  // [dim] norm weight of delta
    const float *scale;   // layer_output_scale (1 float) or null
    float *x_out;         // [B][dim] x' (written by the writer CTA) or null
    const float *pre_w;   // [dim] pre-norm weight, or null: act = x'
    float *xn_out;        // [B][dim] the normalised activation (writer CTA) or null
    int dim;
    float eps;
};

// sum_i v[i]^2 in one fixed order, whatever the CTA size (>= 256 threads):
// thread t < 256 accumulates i = t, t+256, ... with fmaf, then a xor-tree
// over each warp and the 8 warp totals in order.  Every kernel that
// normalises the residual stream uses this, so results do not depend on
// which kernel (or batch size) computed them.  Returned to all threads.
__device__ __forceinline__ float canon_sumsq(const float *v, int n, float *red) {
    const int t = threadIdx.x;
    float p = 0.0f;
    if (t < 256)
        for (int i = t; i < n; i += 256) p = fmaf(v[i], v[i], p);
    p = warp_sum(p);
    __syncthreads();
    if (t < 256 && (t & 31) == 0) red[t >> 5] = p;
    __syncthreads();
    return ((red[0] + red[1]) + (red[2] + red[3])) + ((red[4] + red[5]) + (red[6] + red[7]));
}

// prologue_run for dim = 256 * nb, nb <= NBM: thread t < 256 holds elements
// t + 256k in registers (the element order of canon_sumsq), so all of a
// sequence's inputs are loaded in one trip to memory; same operations and
// rounding as the general loop below.
template <int NBM>
__device__ __forceinline__ void prologue_run_reg(const Prologue &P, int B, float *xs_all, bool writer, float *red) {
    const int dim = P.dim, t = threadIdx.x, nb = dim / 256;
    const bool own = t < 256;
    auto tree = [&](float p) {  // canon_sumsq's reduction of the 256 per-thread chains
        p = warp_sum(p);
        __syncthreads();
        if (own && (t & 31) == 0) red[t >> 5] = p;
        __syncthreads();
        return ((red[0] + red[1]) + (red[2] + red[3])) + ((red[4] + red[5]) + (red[6] + red[7]));
    };
    for (int s = 0; s < B; s++) {
        float x[NBM], d[NBM], pw[NBM], qw[NBM];
#pragma unroll
        for (int k = 0; k < NBM; k++)
            if (own && k < nb) {
                const int i = t + 256 * k;
                x[k] = P.x_in[(size_t)s * dim + i];
                d[k] = P.delta ? P.delta[(size_t)s * dim + i] : 0.0f;
                pw[k] = P.delta ? P.post_w[i] : 0.0f;
                qw[k] = P.pre_w ? P.pre_w[i] : 0.0f;
            }
        if (P.delta) {
            float p = 0.0f;
#pragma unroll
            for (int k = 0; k < NBM; k++)
                if (own && k < nb) p = fmaf(d[k], d[k], p);
            const float ss = tree(p);
            const float inv = 1.0f / sqrtf(ss / (float)dim + P.eps);
#pragma unroll
            for (int k = 0; k < NBM; k++)
                if (own && k < nb) x[k] = __fadd_rn(x[k], __fmul_rn(__fmul_rn(d[k], inv), pw[k]));
        }
        if (P.scale) {
            const float sc = *P.scale;
#pragma unroll
            for (int k = 0; k < NBM; k++)
                if (own && k < nb) x[k] = __fmul_rn(x[k], sc);
        }
        if (writer && P.x_out)
#pragma unroll
            for (int k = 0; k < NBM; k++)
                if (own && k < nb) P.x_out[(size_t)s * dim + t + 256 * k] = x[k];
        if (P.pre_w) {
            float p = 0.0f;
#pragma unroll
            for (int k = 0; k < NBM; k++)
                if (own && k < nb) p = fmaf(x[k], x[k], p);
            const float ss = tree(p);
            const float inv = 1.0f / sqrtf(ss / (float)dim + P.eps);
#pragma unroll
            for (int k = 0; k < NBM; k++)
                if (own && k < nb) {
                    x[k] = __fmul_rn(__fmul_rn(x[k], inv), qw[k]);
                    if (writer && P.xn_out) P.xn_out[(size_t)s * dim + t + 256 * k] = x[k];
                }
        }
#pragma unroll
        for (int k = 0; k < NBM; k++)
            if (own && k < nb) xs_all[(size_t)s * dim + t + 256 * k] = x[k];
    }
    __syncthreads();
}

// Whether prologue_run_reg<10> applies (dim <= 2560, whole super-blocks, >= 256 threads).
__device__ __forceinline__ bool prologue_reg_ok(const Prologue &P) {
    return P.dim % 256 == 0 && P.dim <= 10 * 256 && blockDim.x >= 256;
}

// Fills xs[B][dim] (fp32 activation) and, when q8 != null, q8[B][dim/256]
// BlockQ8_K in shared memory.  Ends with a CTA barrier.
__device__ __forceinline__ void prologue_run(const Prologue &P, int B, float *xs_all, uint8_t *q8_all, bool writer,
                                             float *red) {
    const int dim = P.dim, tid = threadIdx.x, nt = blockDim.x;
    for (int s = 0; s < B; s++) {
        float *xs = xs_all + (size_t)s * dim;
        const float *xi = P.x_in + (size_t)s * dim;
        if (P.delta) {
            const float *dl = P.delta + (size_t)s * dim;
            const float ss = canon_sumsq(dl, dim, red);
            const float inv = 1.0f / sqrtf(ss / (float)dim + P.eps);
            for (int i = tid; i < dim; i += nt) xs[i] = __fadd_rn(xi[i], __fmul_rn(__fmul_rn(dl[i], inv), P.post_w[i]));
        } else {
            for (int i = tid; i < dim; i += nt) xs[i] = xi[i];
        }
        if (P.scale) {
            const float sc = *P.scale;
            for (int i = tid; i < dim; i += nt) xs[i] = __fmul_rn(xs[i], sc);
        }
        if (P.pre_w) {
            __syncthreads();  // xs complete before the cross-thread sum
            const float ss = canon_sumsq(xs, dim, red);
            const float inv = 1.0f / sqrtf(ss / (float)dim + P.eps);
            for (int i = tid; i < dim; i += nt) {  // same thread owns element i in every loop
                if (writer && P.x_out) P.x_out[(size_t)s * dim + i] = xs[i];
                xs[i] = __fmul_rn(__fmul_rn(xs[i], inv), P.pre_w[i]);
                if (writer && P.xn_out) P.xn_out[(size_t)s * dim + i] = xs[i];
            }
        } else if (writer && P.x_out) {
            for (int i = tid; i < dim; i += nt) P.x_out[(size_t)s * dim + i] = xs[i];
        }
    }
    __syncthreads();
    if (q8_all) {
        const int nb = dim / G4_QK, warp = tid >> 5, lane = tid & 31, nw = nt >> 5;
        for (int t = warp; t < B * nb; t += nw) {
            const int s = t / nb, k = t % nb;
            uint32_t q[2];
            float d;
            int ls;
            warp_quant_block(xs_all + (size_t)s * dim + (size_t)k * G4_QK, lane, q, d, ls);
            store_q8_block(q8_all + ((size_t)s * nb + k) * G4_Q8_BYTES, lane, q, d, ls);
        }
        __syncthreads();
    }
}

}  // namespace g4
