// k_gemv.cu — batch-1 decode GEMVs and the Q8_K activation quantizer.
//
// Kernels (all sm_100a SIMT; batch-1 decode is HBM-bound, no tensor cores):
//   quantize_q8k   quantize_row_q8_K (main.c:282-340), one warp per super-block.
//   gemv_dense     F32 / F16 / BF16 rows (mm_f32/mm_f16/mm_bf16, main.c:1494-1537).
//   qk_block_sums  per (row, block) integer sums of the K-quant dot (test tap).
// The K-quant GEMV itself lives in k_gemv_ks.cu.
#include <math.h>

#include <algorithm>

#include "g4_internal.cuh"
#include "g4_kernels.cuh"
#include "g4_prologue.cuh"
#include "g4_quant.cuh"

namespace g4 {

// ---------------------------------------------------------------- Q8_K quantize

// x: [B][ldx] floats, y: [B][nb] BlockQ8_K.  grid (nb, B), block 32.
__global__ void quantize_q8k_kernel(const float *__restrict__ x, int ldx, uint8_t *__restrict__ y, int nb) {
    pdl_trigger();
    pdl_wait();
    const int k = blockIdx.x, s = blockIdx.y, lane = threadIdx.x;
    uint32_t q[2];
    float d;
    int ls;
    warp_quant_block(x + (size_t)s * ldx + (size_t)k * G4_QK, lane, q, d, ls);
    store_q8_block(y + ((size_t)s * nb + k) * G4_Q8_BYTES, lane, q, d, ls);
}

int launch_quantize_q8k(const float *x, int ldx, void *y, int n, int B, cudaStream_t st) {
    if (n % G4_QK) { set_error(G4_ERR_ARG, "quantize_q8K: k=%d not a multiple of 256", n); return G4_ERR_ARG; }
    if (n == 0 || B == 0) return G4_OK;
    G4_CUDA(launch_pdl(quantize_q8k_kernel, dim3(n / G4_QK, B), dim3(32), 0, st, x, ldx, (uint8_t *)y, n / G4_QK));
    G4_LAUNCHED();
    return G4_OK;
}

// ---------------------------------------------------------------- K-quant GEMV

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// ---------------------------------------------------------------- dense GEMV

// One warp per row; x staged in shared memory as fp32.  Epilogues: plain
// store, or GELU(acc) * evec[row] (the PLE gate, main.c:1986-1991).
__global__ void __launch_bounds__(256) gemv_dense_kernel(const void *__restrict__ w, int type, int n, int rows,
                                                         const float *__restrict__ x, int ldx,
                                                         float *__restrict__ out, int ldo, int epi,
                                                         const float *__restrict__ evec, int ld_evec, Prologue pro,
                                                         int has_pro, int pro_writer) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ float pred[8];
    pdl_trigger();
    pdl_wait();
    float *xs = (float *)smem_raw;
    const int s = blockIdx.y;
    if (has_pro) {  // x' = x + rmsnorm(delta)*w (per sequence), computed by every CTA
        Prologue P = pro;
        P.x_in += (size_t)s * P.dim;
        if (P.delta) P.delta += (size_t)s * P.dim;
        if (P.x_out) P.x_out += (size_t)s * P.dim;
        if (P.xn_out) P.xn_out += (size_t)s * P.dim;
        prologue_run(P, 1, xs, nullptr, pro_writer && blockIdx.x == 0, pred);
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = x[(size_t)s * ldx + i];
        __syncthreads();
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + warp;
    if (row >= rows) return;
    float acc = 0.0f;
    const bool vec = (n % 8) == 0;
    if (type == G4_F32) {
        const float *r = (const float *)w + (size_t)row * n;
        if (vec) {
#pragma unroll 5
            for (int j = lane * 4; j < n; j += 128) {
                const float4 a = __ldg(reinterpret_cast<const float4 *>(r + j));
                acc = fmaf(a.x, xs[j], acc); acc = fmaf(a.y, xs[j + 1], acc);
                acc = fmaf(a.z, xs[j + 2], acc); acc = fmaf(a.w, xs[j + 3], acc);
            }
        } else {
            for (int j = lane; j < n; j += 32) acc = fmaf(__ldg(r + j), xs[j], acc);
        }
    } else {
        const uint16_t *r = (const uint16_t *)w + (size_t)row * n;
        const bool bf = type == G4_BF16;
        if (vec) {
#pragma unroll 5
            for (int j = lane * 8; j < n; j += 256) {
                const uint4 a = __ldg(reinterpret_cast<const uint4 *>(r + j));
                const uint32_t ww[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const uint16_t l = (uint16_t)(ww[i] & 0xffffu), h = (uint16_t)(ww[i] >> 16);
                    acc = fmaf(xs[j + 2 * i], bf ? bf16_to_f32(l) : f16_to_f32(l), acc);
                    acc = fmaf(xs[j + 2 * i + 1], bf ? bf16_to_f32(h) : f16_to_f32(h), acc);
                }
            }
        } else {
            for (int j = lane; j < n; j += 32) {
                const uint16_t v = __ldg(r + j);
                acc = fmaf(xs[j], bf ? bf16_to_f32(v) : f16_to_f32(v), acc);
            }
        }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
        if (epi == EPI_GELU_SCALE) acc = gelu_f32(acc) * evec[(size_t)s * ld_evec + row];
        out[(size_t)s * ldo + row] = acc;
    }
}

// Dense GEMV for many sequences: each weight row is read once per NS
// sequences (staged in shared memory) instead of once per sequence.  Every
// accumulator sees exactly the operation order of gemv_dense_kernel, so the
// result of a sequence does not depend on the batch.
template <int NS>
__global__ void __launch_bounds__(256) gemv_dense_ms_kernel(const void *__restrict__ w, int type, int n, int rows,
                                                            const float *__restrict__ x, int ldx, int B,
                                                            float *__restrict__ out, int ldo, int epi,
                                                            const float *__restrict__ evec, int ld_evec) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    pdl_trigger();
    pdl_wait();
    float *xs = (float *)smem_raw;  // [NS][n]
    const int s0 = blockIdx.y * NS, ns = min(NS, B - s0);
    if ((n % 4) == 0 && (ldx % 4) == 0) {  // 16-byte loads, 8 in flight per thread
        const int n4 = n / 4, tot = ns * n4;
        for (int i0 = threadIdx.x; i0 < tot; i0 += 8 * blockDim.x) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = i0 + u * blockDim.x;
                if (i < tot) v[u] = __ldg(reinterpret_cast<const float4 *>(x + (size_t)(s0 + i / n4) * ldx) + i % n4);
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = i0 + u * blockDim.x;
                if (i < tot) reinterpret_cast<float4 *>(xs + (size_t)(i / n4) * n)[i % n4] = v[u];
            }
        }
    } else {
        for (int i = threadIdx.x; i < ns * n; i += blockDim.x) {
            const int s = i / n, j = i % n;
            xs[(size_t)s * n + j] = x[(size_t)(s0 + s) * ldx + j];
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the staged activations serve rows blockIdx.x*8 + warp, stepping over the grid
    for (int row = blockIdx.x * (blockDim.x >> 5) + warp; row < rows; row += gridDim.x * (blockDim.x >> 5)) {
    float acc[NS];
#pragma unroll
    for (int s = 0; s < NS; s++) acc[s] = 0.0f;
    const bool vec = (n % 8) == 0;
    if (type == G4_F32) {
        const float *r = (const float *)w + (size_t)row * n;
        if (vec) {
            for (int j = lane * 4; j < n; j += 128) {
                const float4 a = __ldg(reinterpret_cast<const float4 *>(r + j));
#pragma unroll
                for (int s = 0; s < NS; s++) {
                    const float *xv = xs + (size_t)s * n + j;
                    float t = acc[s];
                    t = fmaf(a.x, xv[0], t); t = fmaf(a.y, xv[1], t); t = fmaf(a.z, xv[2], t); t = fmaf(a.w, xv[3], t);
                    acc[s] = t;
                }
            }
        } else {
            for (int j = lane; j < n; j += 32) {
                const float a = __ldg(r + j);
#pragma unroll
                for (int s = 0; s < NS; s++) acc[s] = fmaf(a, xs[(size_t)s * n + j], acc[s]);
            }
        }
    } else {
        const uint16_t *r = (const uint16_t *)w + (size_t)row * n;
        const bool bf = type == G4_BF16;
        if (vec) {
#pragma unroll 4
            for (int j = lane * 8; j < n; j += 256) {
                const uint4 a = __ldg(reinterpret_cast<const uint4 *>(r + j));
                const uint32_t ww[4] = {a.x, a.y, a.z, a.w};
                float wf[8];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const uint16_t l = (uint16_t)(ww[i] & 0xffffu), h = (uint16_t)(ww[i] >> 16);
                    wf[2 * i] = bf ? bf16_to_f32(l) : f16_to_f32(l);
                    wf[2 * i + 1] = bf ? bf16_to_f32(h) : f16_to_f32(h);
                }
#pragma unroll
                for (int s = 0; s < NS; s++) {
                    const float4 x0 = *reinterpret_cast<const float4 *>(xs + (size_t)s * n + j);
                    const float4 x1 = *reinterpret_cast<const float4 *>(xs + (size_t)s * n + j + 4);
                    float t = acc[s];
                    t = fmaf(x0.x, wf[0], t); t = fmaf(x0.y, wf[1], t); t = fmaf(x0.z, wf[2], t); t = fmaf(x0.w, wf[3], t);
                    t = fmaf(x1.x, wf[4], t); t = fmaf(x1.y, wf[5], t); t = fmaf(x1.z, wf[6], t); t = fmaf(x1.w, wf[7], t);
                    acc[s] = t;
                }
            }
        } else {
            for (int j = lane; j < n; j += 32) {
                const uint16_t v = __ldg(r + j);
                const float wv = bf ? bf16_to_f32(v) : f16_to_f32(v);
#pragma unroll
                for (int s = 0; s < NS; s++) acc[s] = fmaf(xs[(size_t)s * n + j], wv, acc[s]);
            }
        }
    }
#pragma unroll
    for (int s = 0; s < NS; s++) {
        float a = warp_sum(acc[s]);
        if (lane == 0 && s < ns) {
            if (epi == EPI_GELU_SCALE) a = gelu_f32(a) * evec[(size_t)(s0 + s) * ld_evec + row];
            out[(size_t)(s0 + s) * ldo + row] = a;
        }
    }
    }
}

int launch_gemv_dense(const void *w, int type, int n, int rows, const float *x, int ldx, float *out, int ldo,
                      int B, int epi, const float *evec, int ld_evec, cudaStream_t st, const Prologue *pro,
                      int pro_writer) {
    if (!pro && B > 1 && (type == G4_F32 || type == G4_F16 || type == G4_BF16) && rows > 0 && n > 0) {
        const size_t per = (size_t)n * 4;
        // two CTAs per SM (<= 100 KB of staged activations each), about one wave in total
        int NS = per * 8 <= 100 * 1024 ? 8 : per * 4 <= 100 * 1024 ? 4 : per * 2 <= 100 * 1024 ? 2 : 0;
        if (NS) {
            // short rows: one row per warp (staging the activations is cheap); long rows: about two
            // waves of CTAs that each stage once and loop over rows.  A matrix of few rows gets
            // fewer sequences per CTA, so that about 128 CTAs share the weight stream.
            auto grid_of = [&](int ns) {
                const int gy = (B + ns - 1) / ns;
                const int gx = n <= 1024 ? (rows + 7) / 8 : std::max(1, std::min((rows + 7) / 8, 296 / gy));
                return dim3(gx, gy);
            };
            while (NS > 2 && NS / 2 >= B) NS /= 2;
            while (NS > 2 && grid_of(NS).x * grid_of(NS).y < 128 && grid_of(NS / 2).y > grid_of(NS).y) NS /= 2;
            const dim3 grid = grid_of(NS);
            if (NS == 8) G4_CUDA(launch_pdl(gemv_dense_ms_kernel<8>, grid, dim3(256), per * 8, st, w, type, n, rows, x, ldx, B, out, ldo, epi, evec, ld_evec));
            else if (NS == 4) G4_CUDA(launch_pdl(gemv_dense_ms_kernel<4>, grid, dim3(256), per * 4, st, w, type, n, rows, x, ldx, B, out, ldo, epi, evec, ld_evec));
            else G4_CUDA(launch_pdl(gemv_dense_ms_kernel<2>, grid, dim3(256), per * 2, st, w, type, n, rows, x, ldx, B, out, ldo, epi, evec, ld_evec));
            G4_LAUNCHED();
            return G4_OK;
        }
    }
    if (type != G4_F32 && type != G4_F16 && type != G4_BF16) {
        set_error(G4_ERR_TYPE, "gemv_dense: unsupported type %d", type);
        return G4_ERR_TYPE;
    }
    if (rows <= 0 || n <= 0 || B <= 0) return G4_OK;
    const size_t smem = (size_t)n * 4;
    if (smem > 200 * 1024) { set_error(G4_ERR_ARG, "gemv_dense: n=%d too large", n); return G4_ERR_ARG; }
    if (pro && pro->dim != n) { set_error(G4_ERR_ARG, "gemv_dense: prologue dim %d != n %d", pro->dim, n); return G4_ERR_ARG; }
    Prologue P{};
    if (pro) P = *pro;
    G4_CUDA(launch_pdl(gemv_dense_kernel, dim3((rows + 7) / 8, B), dim3(256), smem, st, w, type, n, rows, x, ldx, out,
                       ldo, epi, evec, ld_evec, P, pro ? 1 : 0, pro_writer));
    G4_LAUNCHED();
    return G4_OK;
}

// ---------------------------------------------------------------- block sums tap

// Per (row, block) integer sums of Q4_K/Q5_K x Q8_K, one lane group per
// block, same unpacking as gemv_kquant.  Test tap for bit-exactness.
__global__ void qk_block_sums_kernel(const uint8_t *__restrict__ w, int type, int nb, int rows,
                                     const uint8_t *__restrict__ q8, int *__restrict__ ss, int *__restrict__ smn) {
    const int gid = (blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int c = threadIdx.x & 7;
    const int total = rows * nb;
    const int it = gid < total ? gid : total - 1;
    const int row = it / nb, k = it % nb;
    const size_t bb = type == G4_Q4_K ? 144 : 176;
    const uint8_t *blk = w + ((size_t)row * nb + k) * bb;
    const uint4 meta = *reinterpret_cast<const uint4 *>(blk);
    const int j = c >> 1, h = c & 1;
    uint4 qv, hv = make_uint4(0, 0, 0, 0);
    if (type == G4_Q4_K) qv = reinterpret_cast<const uint4 *>(blk + 16)[c];
    else { hv = reinterpret_cast<const uint4 *>(blk + 16)[h]; qv = reinterpret_cast<const uint4 *>(blk + 48)[c]; }
    const uint8_t *qb = q8 + (size_t)k * G4_Q8_BYTES;
    const uint32_t *a = reinterpret_cast<const uint32_t *>(qb + 4);
    const int16_t *bs = reinterpret_cast<const int16_t *>(qb + 260);
    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w}, hw[4] = {hv.x, hv.y, hv.z, hv.w};
    int dl = 0, dh = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint32_t lo = qw[i] & 0x0F0F0F0Fu, hi = (qw[i] >> 4) & 0x0F0F0F0Fu;
        if (type == G4_Q5_K) {
            lo |= ((hw[i] >> (2 * j)) & 0x01010101u) << 4;
            hi |= ((hw[i] >> (2 * j + 1)) & 0x01010101u) << 4;
        }
        dl = dp4a(lo, a[(64 * j + 16 * h) / 4 + i], dl);
        dh = dp4a(hi, a[(64 * j + 32 + 16 * h) / 4 + i], dh);
    }
    int sc_lo, mn_lo, sc_hi, mn_hi, sc_c, mn_c;
    k4_scale_min(2 * j, meta.y, meta.z, meta.w, sc_lo, mn_lo);
    k4_scale_min(2 * j + 1, meta.y, meta.z, meta.w, sc_hi, mn_hi);
    k4_scale_min(c, meta.y, meta.z, meta.w, sc_c, mn_c);
    int ps = sc_lo * dl + sc_hi * dh;
    int pm = mn_c * ((int)bs[2 * c] + (int)bs[2 * c + 1]);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
        ps += __shfl_xor_sync(0xffffffffu, ps, o, 8);
        pm += __shfl_xor_sync(0xffffffffu, pm, o, 8);
    }
    if (c == 0 && gid < total) { ss[it] = ps; smn[it] = pm; }
}

int launch_qk_block_sums(const void *w, int type, int n, int rows, const void *q8, int *ss, int *sm, cudaStream_t st) {
    const int nb = n / G4_QK;
    const long total = (long)rows * nb;
    if (total == 0) return G4_OK;
    const int threads = 256;
    const long blocks = (total * 8 + threads - 1) / threads;
    qk_block_sums_kernel<<<(unsigned)blocks, threads, 0, st>>>((const uint8_t *)w, type, nb, rows, (const uint8_t *)q8, ss, sm);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

}  // namespace g4

namespace g4 {
int prime_gemv_ks_attrs();
int prime_gemv_attrs() {
    G4_CUDA(cudaFuncSetAttribute(gemv_dense_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    G4_CUDA(cudaFuncSetAttribute(gemv_dense_ms_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    G4_CUDA(cudaFuncSetAttribute(gemv_dense_ms_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    G4_CUDA(cudaFuncSetAttribute(gemv_dense_ms_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    return prime_gemv_ks_attrs();
}
}  // namespace g4
