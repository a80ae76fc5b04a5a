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
            for (int i = tid; i < dim; i += nt) xs[i] = xs[i] * sc;
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
