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

// Canonical order of a dense row dot (every dense kernel, any batch): the row is cut into chunks
// of kDenseChunk elements; in a chunk each lane runs an fmaf chain over its elements in order
// (vectors of 8 (16-bit weights) / 4 (fp32) at lane stride), the 32 lane sums are added by the
// warp_sum butterfly, and the chunk sums are added in chunk order, (0 + C0) + C1 + ...
constexpr int kDenseChunk = 512;
constexpr int kDenseMaxSlots = 128;  // chunk sums of one CTA (rows per CTA x chunks)

// Lane chain of chunk c of one row (weights r, activation xs in shared memory).
__device__ __forceinline__ float dense_chunk(const void *r, int type, int n, const float *xs, int c, int lane) {
    float acc = 0.0f;
    const int j0 = c * kDenseChunk, j1 = min(n, j0 + kDenseChunk);
    const bool vec = (n % 8) == 0;
    if (type == G4_F32) {
        const float *rf = (const float *)r;
        if (vec) {
#pragma unroll 4
            for (int j = j0 + lane * 4; j < j1; j += 128) {
                const float4 a = __ldg(reinterpret_cast<const float4 *>(rf + j));
                acc = fmaf(a.x, xs[j], acc); acc = fmaf(a.y, xs[j + 1], acc);
                acc = fmaf(a.z, xs[j + 2], acc); acc = fmaf(a.w, xs[j + 3], acc);
            }
        } else {
            for (int j = j0 + lane; j < j1; j += 32) acc = fmaf(__ldg(rf + j), xs[j], acc);
        }
    } else {
        const uint16_t *rh = (const uint16_t *)r;
        const bool bf = type == G4_BF16;
        if (vec) {
#pragma unroll 2
            for (int j = j0 + lane * 8; j < j1; j += 256) {
                const uint4 a = __ldg(reinterpret_cast<const uint4 *>(rh + j));
                const uint32_t ww[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const uint16_t l = (uint16_t)(ww[i] & 0xffffu), h = (uint16_t)(ww[i] >> 16);
                    acc = fmaf(xs[j + 2 * i], bf ? bf16_to_f32(l) : f16_to_f32(l), acc);
                    acc = fmaf(xs[j + 2 * i + 1], bf ? bf16_to_f32(h) : f16_to_f32(h), acc);
                }
            }
        } else {
            for (int j = j0 + lane; j < j1; j += 32) {
                const uint16_t v = __ldg(rh + j);
                acc = fmaf(xs[j], bf ? bf16_to_f32(v) : f16_to_f32(v), acc);
            }
        }
    }
    return warp_sum(acc);
}

// One sequence per blockIdx.y; a CTA takes rpc rows, a warp one (row, chunk) at a time (so a long
// row keeps several warps busy); x staged in shared memory as fp32.  Epilogues: plain store, or
// GELU(acc) * evec[row] (the PLE gate, main.c:1986-1991).
__global__ void __launch_bounds__(256) gemv_dense_kernel(const void *__restrict__ w, int type, int n, int rows,
                                                         const float *__restrict__ x, int ldx,
                                                         float *__restrict__ out, int ldo, int epi,
                                                         const float *__restrict__ evec, int ld_evec, Prologue pro,
                                                         int has_pro, int pro_writer, int rpc) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ float pred[8];
    __shared__ float csum[kDenseMaxSlots];
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
        if (prologue_reg_ok(P)) prologue_run_reg<10>(P, 1, xs, pro_writer && blockIdx.x == 0, pred);
        else prologue_run(P, 1, xs, nullptr, pro_writer && blockIdx.x == 0, pred);
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = x[(size_t)s * ldx + i];
        __syncthreads();
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int S = (n + kDenseChunk - 1) / kDenseChunk, row0 = blockIdx.x * rpc;
    const size_t rb = (size_t)n * (type == G4_F32 ? 4 : 2);
    for (int u = warp; u < rpc * S; u += nw) {
        const int rr = u / S, c = u % S, row = row0 + rr;
        if (row >= rows) continue;
        const float v = dense_chunk((const uint8_t *)w + (size_t)row * rb, type, n, xs, c, lane);
        if (lane == 0) csum[u] = v;
    }
    __syncthreads();
    if ((int)threadIdx.x < rpc) {
        const int row = row0 + threadIdx.x;
        if (row < rows) {
            float acc = 0.0f;
            for (int c = 0; c < S; c++) acc = __fadd_rn(acc, csum[threadIdx.x * S + c]);
            if (epi == EPI_GELU_SCALE) acc = gelu_f32(acc) * evec[(size_t)s * ld_evec + row];
            out[(size_t)s * ldo + row] = acc;
        }
    }
}

static int g_tm_sms_dense = 0;  // SM count, set when the kernels' attributes are primed

// Sum over the 32 lanes of each of the NV = 2^H values v[] with 31 shuffles
// in all (instead of 5 per value).  Every value goes through the butterfly of
// warp_sum (lane bit 4 first, then 3, 2, 1, 0), so each total is bitwise that
// of warp_sum.  Returns the total of value index (lane >> (5 - H)).
template <int NV>
__device__ __forceinline__ float warp_sum_many(float (&v)[NV], int lane) {
    constexpr int H = NV == 1 ? 0 : NV == 2 ? 1 : NV == 4 ? 2 : NV == 8 ? 3 : NV == 16 ? 4 : 5;
    static_assert((1 << H) == NV, "NV must be a power of two <= 32");
#pragma unroll
    for (int step = 0; step < H; step++) {
        const int o = 16 >> step, half = NV >> (step + 1);
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int k = 0; k < half; k++) {
            const float send = up ? v[k] : v[k + half];
            const float keep = up ? v[k + half] : v[k];
            v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    float r = v[0];
#pragma unroll
    for (int o = 16 >> H; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    return r;
}

// Dense GEMV for many sequences: NS sequences' activations are staged in
// shared memory once per CTA, and each warp works on RW rows at a time, so an
// activation value read from shared memory serves RW rows and a weight value
// read from memory serves NS sequences.  The CTAs loop over the rows.  Every
// (row, sequence) follows the canonical chunked order of gemv_dense_kernel
// (lane-strided fmaf chains per chunk, the warp_sum butterfly, chunk sums in
// order), so the result of a sequence does not depend on the batch.  With a
// prologue each CTA computes x + rmsnorm(delta)*w of its sequences itself
// (the same expressions as resnorm_reg_kernel), and the CTAs of column 0
// write it out (pro_writer).
template <int NS, int RW>
__global__ void __launch_bounds__(256, 2) gemv_dense_ms_kernel(const void *__restrict__ w, int type, int n, int rows,
                                                            const float *__restrict__ x, int ldx, int B,
                                                            float *__restrict__ out, int ldo, int epi,
                                                            const float *__restrict__ evec, int ld_evec, Prologue pro,
                                                            int has_pro, int pro_writer) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ float pred[8];
    pdl_trigger();
    pdl_wait();
    float *xs = (float *)smem_raw;  // [NS][n]
    const int s0 = blockIdx.y * NS, ns = min(NS, B - s0);
    if (has_pro) {  // x' = x + rmsnorm(delta)*w of this CTA's sequences (the residual glue of the batched step)
        Prologue P = pro;
        P.x_in += (size_t)s0 * P.dim;
        if (P.delta) P.delta += (size_t)s0 * P.dim;
        if (P.x_out) P.x_out += (size_t)s0 * P.dim;
        if (P.xn_out) P.xn_out += (size_t)s0 * P.dim;
        if (prologue_reg_ok(P)) prologue_run_reg<10>(P, ns, xs, pro_writer && blockIdx.x == 0, pred);
        else prologue_run(P, ns, xs, nullptr, pro_writer && blockIdx.x == 0, pred);
    } else if ((n % 4) == 0 && (ldx % 4) == 0) {  // 16-byte loads, 8 in flight per thread
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
    for (int i = ns * n + threadIdx.x; i < NS * n; i += blockDim.x) xs[i] = 0.0f;  // padding sequences
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool vec = (n % 8) == 0, f32 = type == G4_F32, bf = type == G4_BF16;
    constexpr int NV = RW * NS, LPV = 32 / NV;
    const int S = (n + kDenseChunk - 1) / kDenseChunk;
    for (int row0 = (blockIdx.x * (blockDim.x >> 5) + warp) * RW; row0 < rows; row0 += gridDim.x * (blockDim.x >> 5) * RW) {
        int rr[RW];  // rows past the end repeat the last row (computed, not stored)
#pragma unroll
        for (int r = 0; r < RW; r++) rr[r] = min(row0 + r, rows - 1);
        float vt = 0.0f;  // this lane's value (index lane / LPV): the chunk sums in chunk order
        for (int c = 0; c < S; c++) {
        const int j0 = c * kDenseChunk, j1 = min(n, j0 + kDenseChunk);
        float acc[RW][NS];
#pragma unroll
        for (int r = 0; r < RW; r++)
#pragma unroll
            for (int s = 0; s < NS; s++) acc[r][s] = 0.0f;
        if (f32 && vec) {
            for (int j = j0 + lane * 4; j < j1; j += 128) {
                float4 a[RW];
#pragma unroll
                for (int r = 0; r < RW; r++) a[r] = __ldg(reinterpret_cast<const float4 *>((const float *)w + (size_t)rr[r] * n + j));
#pragma unroll
                for (int s = 0; s < NS; s++) {
                    const float4 xv = *reinterpret_cast<const float4 *>(xs + (size_t)s * n + j);
#pragma unroll
                    for (int r = 0; r < RW; r++) {
                        float t = acc[r][s];
                        t = fmaf(a[r].x, xv.x, t); t = fmaf(a[r].y, xv.y, t); t = fmaf(a[r].z, xv.z, t); t = fmaf(a[r].w, xv.w, t);
                        acc[r][s] = t;
                    }
                }
            }
        } else if (f32) {
            for (int j = j0 + lane; j < j1; j += 32) {
                float a[RW];
#pragma unroll
                for (int r = 0; r < RW; r++) a[r] = __ldg((const float *)w + (size_t)rr[r] * n + j);
#pragma unroll
                for (int s = 0; s < NS; s++) {
                    const float xv = xs[(size_t)s * n + j];
#pragma unroll
                    for (int r = 0; r < RW; r++) acc[r][s] = fmaf(a[r], xv, acc[r][s]);
                }
            }
        } else if (vec) {
#pragma unroll 2
            for (int j = j0 + lane * 8; j < j1; j += 256) {
                float wf[RW][8];
#pragma unroll
                for (int r = 0; r < RW; r++) {
                    const uint4 a = __ldg(reinterpret_cast<const uint4 *>((const uint16_t *)w + (size_t)rr[r] * n + j));
                    const uint32_t ww[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const uint16_t l = (uint16_t)(ww[i] & 0xffffu), h = (uint16_t)(ww[i] >> 16);
                        wf[r][2 * i] = bf ? bf16_to_f32(l) : f16_to_f32(l);
                        wf[r][2 * i + 1] = bf ? bf16_to_f32(h) : f16_to_f32(h);
                    }
                }
#pragma unroll
                for (int s = 0; s < NS; s++) {
                    const float4 x0 = *reinterpret_cast<const float4 *>(xs + (size_t)s * n + j);
                    const float4 x1 = *reinterpret_cast<const float4 *>(xs + (size_t)s * n + j + 4);
#pragma unroll
                    for (int r = 0; r < RW; r++) {
                        float t = acc[r][s];
                        t = fmaf(x0.x, wf[r][0], t); t = fmaf(x0.y, wf[r][1], t); t = fmaf(x0.z, wf[r][2], t); t = fmaf(x0.w, wf[r][3], t);
                        t = fmaf(x1.x, wf[r][4], t); t = fmaf(x1.y, wf[r][5], t); t = fmaf(x1.z, wf[r][6], t); t = fmaf(x1.w, wf[r][7], t);
                        acc[r][s] = t;
                    }
                }
            }
        } else {
            for (int j = j0 + lane; j < j1; j += 32) {
                float wv[RW];
#pragma unroll
                for (int r = 0; r < RW; r++) {
                    const uint16_t v = __ldg((const uint16_t *)w + (size_t)rr[r] * n + j);
                    wv[r] = bf ? bf16_to_f32(v) : f16_to_f32(v);
                }
#pragma unroll
                for (int s = 0; s < NS; s++) {
                    const float xv = xs[(size_t)s * n + j];
#pragma unroll
                    for (int r = 0; r < RW; r++) acc[r][s] = fmaf(xv, wv[r], acc[r][s]);
                }
            }
        }
        // chunk totals: value index r * NS + s, one per lane group of 32 / (RW * NS) lanes
        float flat[RW * NS];
#pragma unroll
        for (int r = 0; r < RW; r++)
#pragma unroll
            for (int s = 0; s < NS; s++) flat[r * NS + s] = acc[r][s];
        vt = __fadd_rn(vt, warp_sum_many<NV>(flat, lane));
        }
        const float tot = vt;
        if ((lane & (LPV - 1)) == 0) {
            const int idx = lane / LPV, r = idx / NS, s = idx % NS, row = row0 + r;
            if (row < rows && s < ns) {
                float a = tot;
                if (epi == EPI_GELU_SCALE) a = gelu_f32(a) * evec[(size_t)(s0 + s) * ld_evec + row];
                out[(size_t)(s0 + s) * ldo + row] = a;
            }
        }
    }
}

int launch_gemv_dense(const void *w, int type, int n, int rows, const float *x, int ldx, float *out, int ldo,
                      int B, int epi, const float *evec, int ld_evec, cudaStream_t st, const Prologue *pro,
                      int pro_writer) {
    if (B > 1 && (type == G4_F32 || type == G4_F16 || type == G4_BF16) && rows > 0 && n > 0 && (!pro || pro->dim == n)) {
        Prologue P{};
        if (pro) P = *pro;
        const size_t per = (size_t)n * 4;
        // NS sequences per CTA (<= 100 KB of staged activations: two CTAs per SM), RW rows per warp
        int NS = per * 8 <= 100 * 1024 ? 8 : per * 4 <= 100 * 1024 ? 4 : per * 2 <= 100 * 1024 ? 2 : 0;
        while (NS > 2 && NS / 2 >= B) NS /= 2;
        if (NS) {
            // about two waves of CTAs (two per SM), each staging its sequences once and looping over
            // rows; a matrix of few rows gets fewer sequences per CTA so that more CTAs share it
            const int nsm = g_tm_sms_dense > 0 ? g_tm_sms_dense : 148;
            auto grid_of = [&](int ns, int rw) {
                const int gy = (B + ns - 1) / ns;
                const int need = (rows + 8 * rw - 1) / (8 * rw);
                return dim3(std::max(1, std::min(need, 2 * nsm / gy)), gy);
            };
            int RW = NS == 8 ? 4 : 8;
            while (NS > 2 && grid_of(NS, RW).x * grid_of(NS, RW).y < nsm && grid_of(NS / 2, RW).y > grid_of(NS, RW).y) {
                NS /= 2;
                RW = NS == 8 ? 4 : 8;
            }
            while (RW > 1 && grid_of(NS, RW).x * grid_of(NS, RW).y < nsm && grid_of(NS, RW / 2).x > grid_of(NS, RW).x) RW /= 2;
            const dim3 grid = grid_of(NS, RW);
#define G4_DMS(NSV, RWV)                                                                                          \
    if (NS == NSV && RW == RWV)                                                                                    \
        G4_CUDA(launch_pdl(gemv_dense_ms_kernel<NSV, RWV>, grid, dim3(256), per * NSV, st, w, type, n, rows, x, ldx, \
                           B, out, ldo, epi, evec, ld_evec, P, pro ? 1 : 0, pro_writer));
            G4_DMS(8, 4) else G4_DMS(8, 2) else G4_DMS(8, 1)
            else G4_DMS(4, 8) else G4_DMS(4, 4) else G4_DMS(4, 2) else G4_DMS(4, 1)
            else G4_DMS(2, 8) else G4_DMS(2, 4) else G4_DMS(2, 2) else G4_DMS(2, 1)
#undef G4_DMS
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
    // rows per CTA: every warp busy on short rows; at most about four CTAs per SM on tall matrices
    const int S = (n + kDenseChunk - 1) / kDenseChunk, nsm = g_tm_sms_dense > 0 ? g_tm_sms_dense : 148;
    int rpc = std::max(S >= 8 ? 1 : 8 / S, (rows + 4 * nsm - 1) / (4 * nsm));
    rpc = std::min(rpc, std::max(1, kDenseMaxSlots / S));
    if (rpc * S > kDenseMaxSlots) { set_error(G4_ERR_ARG, "gemv_dense: n=%d too large", n); return G4_ERR_ARG; }
    G4_CUDA(launch_pdl(gemv_dense_kernel, dim3((rows + rpc - 1) / rpc, B), dim3(256), smem, st, w, type, n, rows, x, ldx,
                       out, ldo, epi, evec, ld_evec, P, pro ? 1 : 0, pro_writer, rpc));
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
    {
        int dev = 0, nsm = 0;
        G4_CUDA(cudaGetDevice(&dev));
        G4_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
        g_tm_sms_dense = nsm;
    }
    G4_CUDA(cudaFuncSetAttribute(gemv_dense_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
#define G4_DMS_ATTR(NSV, RWV) \
    G4_CUDA(cudaFuncSetAttribute(gemv_dense_ms_kernel<NSV, RWV>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024));
    G4_DMS_ATTR(8, 4) G4_DMS_ATTR(8, 2) G4_DMS_ATTR(8, 1)
    G4_DMS_ATTR(4, 8) G4_DMS_ATTR(4, 4) G4_DMS_ATTR(4, 2) G4_DMS_ATTR(4, 1)
    G4_DMS_ATTR(2, 8) G4_DMS_ATTR(2, 4) G4_DMS_ATTR(2, 2) G4_DMS_ATTR(2, 1)
#undef G4_DMS_ATTR
    return prime_gemv_ks_attrs();
}
}  // namespace g4
