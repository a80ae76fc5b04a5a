// k_gemv.cu — batch-1 decode GEMVs and the Q8_K activation quantizer.
//
// Kernels (all sm_100a SIMT; batch-1 decode is HBM-bound, no tensor cores):
//   quantize_q8k   quantize_row_q8_K (main.c:282-340), one warp per super-block.
//   gemv_kquant    Q4_K/Q5_K x Q8_K integer dots (vec_dot_q{4,5}_K_q8_K,
//                  main.c:347-593) and the Q6_K fp32 dequant-dot of
//                  mm_quant_rows (main.c:1539-1556), with fused epilogues
//                  (GELU(gate)*up, softcap + argmax).
//   gemv_dense     F32 / F16 / BF16 rows (mm_f32/mm_f16/mm_bf16, main.c:1494-1537).
//
// Work decomposition of gemv_kquant: a CTA of 256 threads owns RT rows of one
// matrix.  Its 32 "lane groups" (8 lanes each) walk items = (row-tile of R
// rows, super-block k); the 8 lanes of a group split one 256-weight
// super-block (16 bytes of quants each, 128-bit loads), reduce their integer
// partials with width-8 shuffles and leave one float per (row, block) in
// shared memory.  Rows are then summed in block order, so a result does not
// depend on the launch shape.  For Q4_K/Q5_K each block's integer sums
// sumi_s / sumi_m are exact (bit-identical to the reference's integer
// arithmetic); the block's float contribution is d_x*d_w*sumi_s -
// d_x*dmin_w*sumi_m.  Q6_K weights are dequantized exactly as the reference
// does ((d*scale)*(q-32) in fp32) and dotted with the fp32 activation.
#include <math.h>

#include "g4_internal.cuh"
#include "g4_kernels.cuh"
#include "g4_quant.cuh"

namespace g4 {

// ---------------------------------------------------------------- Q8_K quantize

// x: [B][ldx] floats, y: [B][nb] BlockQ8_K.  grid (nb, B), block 32.
__global__ void quantize_q8k_kernel(const float *__restrict__ x, int ldx, uint8_t *__restrict__ y, int nb) {
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
    quantize_q8k_kernel<<<dim3(n / G4_QK, B), 32, 0, st>>>(x, ldx, (uint8_t *)y, n / G4_QK);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

// ---------------------------------------------------------------- K-quant GEMV

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

__device__ __forceinline__ float gelu_tanh(float x) {  // gelu_f32, main.c:1490-1492
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * x * (1.0f + 0.044715f * x * x)));
}

// byte i of w (0..63) as the float (q - 32), exact: 2^23 + q - (2^23 + 32).
__device__ __forceinline__ float q6_byte_to_f(uint32_t w, int i) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540 + i)) - 8388640.0f;
}

struct KqSmem {   // activation of one sequence staged in shared memory
    int8_t *qs;   // [n]        Q8_K quants (Q4/Q5 jobs)
    float *dx;    // [nb]       Q8_K scales
    int *bs2;     // [nb][8]    bsums[2i] + bsums[2i+1]
    float *x;     // [n]        fp32 activation (Q6 jobs)
    float *red;   // [rows_in_cta][nb] per-block partials
};

template <int R6>
__global__ void __launch_bounds__(256) gemv_kquant_kernel(GemvJobs jobs) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    int ji = 0;
#pragma unroll
    for (int i = 1; i < kMaxJobs; i++)
        if (i < jobs.njobs && (int)blockIdx.x >= jobs.j[i].cta_begin) ji = i;
    const GemvJob &J = jobs.j[ji];
    const int s = blockIdx.y;  // sequence
    const int type = J.type, n = J.n, nb = n / G4_QK, rows = J.rows;
    const int RT = J.rt;
    const int nmat = J.w2 ? 2 : 1;
    const int row0 = ((int)blockIdx.x - J.cta_begin) * RT;
    const int tid = threadIdx.x, lane = tid & 31, c = lane & 7, g = tid >> 3;

    KqSmem sm;
    uint8_t *p = smem_raw;
    const bool q8act = (type != G4_Q6_K);
    if (q8act) {
        sm.qs = (int8_t *)p; p += (size_t)n;
        sm.dx = (float *)p; p += (size_t)nb * 4;
        sm.bs2 = (int *)p; p += (size_t)nb * 32;
        sm.x = nullptr;
        // stage the Q8_K blocks of sequence s (BlockQ8_K, 292 B each, 4-byte aligned)
        const uint8_t *src = (const uint8_t *)J.act + (size_t)s * nb * G4_Q8_BYTES;
        for (int i = tid; i < nb * 64; i += 256) {
            const int k = i >> 6, w = i & 63;
            reinterpret_cast<uint32_t *>(sm.qs)[k * 64 + w] =
                *reinterpret_cast<const uint32_t *>(src + (size_t)k * G4_Q8_BYTES + 4 + 4 * w);
        }
        for (int i = tid; i < nb * 8; i += 256) {
            const int k = i >> 3, j = i & 7;
            const int16_t *bs = reinterpret_cast<const int16_t *>(src + (size_t)k * G4_Q8_BYTES + 260);
            sm.bs2[i] = (int)bs[2 * j] + (int)bs[2 * j + 1];
            if (j == 0) sm.dx[k] = *reinterpret_cast<const float *>(src + (size_t)k * G4_Q8_BYTES);
        }
    } else {
        sm.x = (float *)p; p += (size_t)n * 4;
        const float4 *src = reinterpret_cast<const float4 *>((const float *)J.act + (size_t)s * J.act_stride);
        for (int i = tid; i < n / 4; i += 256) reinterpret_cast<float4 *>(sm.x)[i] = src[i];
    }
    sm.red = (float *)p;
    __syncthreads();

    const int R = (type == G4_Q6_K) ? R6 : 1;
    const int tiles = (RT / R) * nmat;
    const int items = tiles * nb;
    // every lane of a warp runs the same number of iterations (full-mask shuffles)
    for (int it0 = g & ~3; it0 < items; it0 += 32) {
        const int it_raw = it0 + (g & 3);
        const bool valid = it_raw < items;
        const int it = valid ? it_raw : items - 1;
        const int k = it % nb, tile = it / nb;
        const int m = tile / (RT / R);                   // which matrix (gate / up)
        const int rl0 = (tile % (RT / R)) * R;           // first local row
        const uint8_t *W = (const uint8_t *)(m ? J.w2 : J.w);
        if (type == G4_Q4_K || type == G4_Q5_K) {
            const int row = min(row0 + rl0, rows - 1);
            const size_t bb = type == G4_Q4_K ? 144 : 176;
            const uint8_t *blk = W + ((size_t)row * nb + k) * bb;
            const uint4 meta = __ldg(reinterpret_cast<const uint4 *>(blk));
            const int j = c >> 1, h = c & 1;
            uint4 qv, hv = make_uint4(0, 0, 0, 0);
            if (type == G4_Q4_K) {
                qv = __ldg(reinterpret_cast<const uint4 *>(blk + 16) + c);
            } else {
                hv = __ldg(reinterpret_cast<const uint4 *>(blk + 16) + h);
                qv = __ldg(reinterpret_cast<const uint4 *>(blk + 48) + c);
            }
            const uint4 alo = *reinterpret_cast<const uint4 *>(sm.qs + k * G4_QK + 64 * j + 16 * h);
            const uint4 ahi = *reinterpret_cast<const uint4 *>(sm.qs + k * G4_QK + 64 * j + 32 + 16 * h);
            uint32_t lo[4], hi[4];
            const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
            const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                lo[i] = qw[i] & 0x0F0F0F0Fu;
                hi[i] = (qw[i] >> 4) & 0x0F0F0F0Fu;
                if (type == G4_Q5_K) {  // 5th bit: bit 2j (low nibbles) / 2j+1 (high) of qh
                    lo[i] |= ((hw[i] >> (2 * j)) & 0x01010101u) << 4;
                    hi[i] |= ((hw[i] >> (2 * j + 1)) & 0x01010101u) << 4;
                }
            }
            int dl = 0, dh = 0;
            dl = dp4a(lo[0], alo.x, dl); dl = dp4a(lo[1], alo.y, dl);
            dl = dp4a(lo[2], alo.z, dl); dl = dp4a(lo[3], alo.w, dl);
            dh = dp4a(hi[0], ahi.x, dh); dh = dp4a(hi[1], ahi.y, dh);
            dh = dp4a(hi[2], ahi.z, dh); dh = dp4a(hi[3], ahi.w, dh);
            int sc_lo, mn_lo, sc_hi, mn_hi, sc_c, mn_c;
            k4_scale_min(2 * j, meta.y, meta.z, meta.w, sc_lo, mn_lo);
            k4_scale_min(2 * j + 1, meta.y, meta.z, meta.w, sc_hi, mn_hi);
            k4_scale_min(c, meta.y, meta.z, meta.w, sc_c, mn_c);
            int ps = sc_lo * dl + sc_hi * dh;
            int pm = mn_c * sm.bs2[k * 8 + c];
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) {
                ps += __shfl_xor_sync(0xffffffffu, ps, o, 8);
                pm += __shfl_xor_sync(0xffffffffu, pm, o, 8);
            }
            if (c == 0 && valid) {
                const float dxk = sm.dx[k];
                const float dd = dxk * f16_to_f32((uint16_t)(meta.x & 0xffffu));
                const float dm = dxk * f16_to_f32((uint16_t)(meta.x >> 16));
                sm.red[(m * RT + rl0) * nb + k] = fmaf(-dm, (float)pm, dd * (float)ps);
            }
        } else {  // Q6_K, fp32 activation
            const int n6 = c >> 2, second = (c >> 1) & 1, par = c & 1;
            const int e_lo = 128 * n6 + 32 * second + 16 * par;
            float xl[16], xh[16];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 a = *reinterpret_cast<const float4 *>(sm.x + k * G4_QK + e_lo + 4 * i);
                const float4 b = *reinterpret_cast<const float4 *>(sm.x + k * G4_QK + e_lo + 64 + 4 * i);
                xl[4 * i] = a.x; xl[4 * i + 1] = a.y; xl[4 * i + 2] = a.z; xl[4 * i + 3] = a.w;
                xh[4 * i] = b.x; xh[4 * i + 1] = b.y; xh[4 * i + 2] = b.z; xh[4 * i + 3] = b.w;
            }
            const size_t nblk_total = (size_t)rows * nb;
            const Q6Planes P = q6_planes(W, nblk_total);
            uint4 qlv[R6], qhv[R6];
            uint2 scv[R6];
            uint16_t dv[R6];
#pragma unroll
            for (int r = 0; r < R6; r++) {
                const int row = min(row0 + rl0 + r, rows - 1);
                const size_t bi = (size_t)row * nb + k;
                qlv[r] = __ldg(P.ql + bi * 8 + c);
                qhv[r] = __ldg(P.qh + bi * 4 + 2 * n6 + par);
                scv[r] = __ldg(reinterpret_cast<const uint2 *>(P.sc + bi) + n6);
                dv[r] = __ldg(P.d + bi);
            }
#pragma unroll
            for (int r = 0; r < R6; r++) {
                const float d = f16_to_f32(dv[r]);
                const int sidx = 2 * second + par;  // scale index within the 8-byte half
                const uint32_t sw_lo = sidx < 4 ? scv[r].x : scv[r].y;
                const uint32_t sw_hi = scv[r].y;    // index sidx + 4 >= 4
                const int sc_lo = (int)(int8_t)((sw_lo >> (8 * (sidx & 3))) & 0xffu);
                const int sc_hi = (int)(int8_t)((sw_hi >> (8 * (sidx & 3))) & 0xffu);
                const float dsl = d * (float)sc_lo, dsh = d * (float)sc_hi;
                const uint32_t qlw[4] = {qlv[r].x, qlv[r].y, qlv[r].z, qlv[r].w};
                const uint32_t qhw[4] = {qhv[r].x, qhv[r].y, qhv[r].z, qhv[r].w};
                float acc = 0.0f;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const uint32_t lo = (qlw[i] & 0x0F0F0F0Fu) | (((qhw[i] >> (2 * second)) & 0x03030303u) << 4);
                    const uint32_t hi = ((qlw[i] >> 4) & 0x0F0F0F0Fu) | (((qhw[i] >> (4 + 2 * second)) & 0x03030303u) << 4);
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        acc = fmaf(xl[4 * i + b], dsl * q6_byte_to_f(lo, b), acc);
                        acc = fmaf(xh[4 * i + b], dsh * q6_byte_to_f(hi, b), acc);
                    }
                }
#pragma unroll
                for (int o = 4; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o, 8);
                if (c == 0 && valid) sm.red[(m * RT + rl0 + r) * nb + k] = acc;
            }
        }
    }
    __syncthreads();

    // epilogue: sum each row's blocks in order
    float best = -INFINITY;
    int besti = 0x7fffffff;
    for (int rl = tid; rl < RT; rl += 256) {
        const int row = row0 + rl;
        if (row >= rows) break;
        float a = 0.0f;
        for (int k = 0; k < nb; k++) a += sm.red[rl * nb + k];
        float* out = J.out + (size_t)s * J.out_stride;
        if (J.epi == EPI_GELU_MUL) {
            float b = 0.0f;
            for (int k = 0; k < nb; k++) b += sm.red[(RT + rl) * nb + k];
            out[row] = gelu_tanh(a) * b;
        } else if (J.epi == EPI_SOFTCAP_ARGMAX) {
            if (J.cap > 0.0f) a = J.cap * tanhf(a * (1.0f / J.cap));
            if (J.out) out[row] = a;
            if (a > best) { best = a; besti = row; }
        } else if (J.epi == EPI_GELU_SCALE) {
            out[row] = gelu_tanh(a) * J.evec[(size_t)s * J.ld_evec + row];
        } else {
            out[row] = a;
        }
    }
    if (J.epi == EPI_SOFTCAP_ARGMAX) {
        unsigned long long key = besti == 0x7fffffff ? 0ull : argmax_key(best, besti);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long ok = __shfl_xor_sync(0xffffffffu, key, o);
            key = ok > key ? ok : key;
        }
        if (lane == 0 && key) atomicMax(J.amax + s, key);
    }
}

// Shared memory bytes for one job of gemv_kquant.
static size_t kq_smem(const GemvJob &J) {
    const int nb = J.n / G4_QK;
    size_t act = J.type == G4_Q6_K ? (size_t)J.n * 4 : (size_t)J.n + (size_t)nb * 36;
    act = (act + 15) & ~(size_t)15;
    return act + (size_t)(J.w2 ? 2 : 1) * J.rt * nb * 4;
}

int launch_gemv_kquant(GemvJobs &jobs, int B, cudaStream_t st) {
    int ctas = 0;
    size_t smem = 0;
    for (int i = 0; i < jobs.njobs; i++) {
        GemvJob &J = jobs.j[i];
        if (J.type != G4_Q4_K && J.type != G4_Q5_K && J.type != G4_Q6_K) {
            set_error(G4_ERR_TYPE, "gemv_kquant: unsupported type %d", J.type);
            return G4_ERR_TYPE;
        }
        if (J.n % G4_QK || J.n <= 0 || J.rows <= 0) {
            set_error(G4_ERR_ARG, "gemv: n=%d (must be a positive multiple of 256), rows=%d", J.n, J.rows);
            return G4_ERR_ARG;
        }
        if (J.rt <= 0) J.rt = default_rt(J.type, J.n, J.rows);
        J.cta_begin = ctas;
        ctas += (J.rows + J.rt - 1) / J.rt;
        size_t b = kq_smem(J);
        smem = b > smem ? b : smem;
    }
    if (ctas == 0 || B == 0) return G4_OK;
    if (smem > 200 * 1024) {
        set_error(G4_ERR_ARG, "gemv: activation too large for shared memory (%zu bytes)", smem);
        return G4_ERR_ARG;
    }
    gemv_kquant_kernel<4><<<dim3(ctas, B), 256, smem, st>>>(jobs);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

// Rows per CTA: keep (rows-per-CTA x blocks) a multiple of the 32 lane
// groups where possible and give small matrices enough CTAs.
int default_rt(int type, int n, int rows) {
    const int nb = n / G4_QK;
    int rt;
    if (type == G4_Q6_K) rt = nb >= 32 ? 16 : 64;
    else rt = nb >= 32 ? 8 : 16;
    while (rt > 4 && (rows + rt - 1) / rt < 296) rt /= 2;  // >= 2 CTAs per SM when possible
    if (type == G4_Q6_K && rt < 4) rt = 4;
    return rt;
}

// ---------------------------------------------------------------- dense GEMV

// One warp per row; x staged in shared memory as fp32.  Epilogues: plain
// store, or GELU(acc) * evec[row] (the PLE gate, main.c:1986-1991).
__global__ void __launch_bounds__(256) gemv_dense_kernel(const void *__restrict__ w, int type, int n, int rows,
                                                         const float *__restrict__ x, int ldx,
                                                         float *__restrict__ out, int ldo, int epi,
                                                         const float *__restrict__ evec, int ld_evec) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    float *xs = (float *)smem_raw;
    const int s = blockIdx.y;
    for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = x[(size_t)s * ldx + i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + warp;
    if (row >= rows) return;
    float acc = 0.0f;
    const bool vec = (n % 8) == 0;
    if (type == G4_F32) {
        const float *r = (const float *)w + (size_t)row * n;
        if (vec) {
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
        if (epi == EPI_GELU_SCALE) acc = gelu_tanh(acc) * evec[(size_t)s * ld_evec + row];
        out[(size_t)s * ldo + row] = acc;
    }
}

int launch_gemv_dense(const void *w, int type, int n, int rows, const float *x, int ldx, float *out, int ldo,
                      int B, int epi, const float *evec, int ld_evec, cudaStream_t st) {
    if (type != G4_F32 && type != G4_F16 && type != G4_BF16) {
        set_error(G4_ERR_TYPE, "gemv_dense: unsupported type %d", type);
        return G4_ERR_TYPE;
    }
    if (rows <= 0 || n <= 0 || B <= 0) return G4_OK;
    const size_t smem = (size_t)n * 4;
    if (smem > 200 * 1024) { set_error(G4_ERR_ARG, "gemv_dense: n=%d too large", n); return G4_ERR_ARG; }
    gemv_dense_kernel<<<dim3((rows + 7) / 8, B), 256, smem, st>>>(w, type, n, rows, x, ldx, out, ldo, epi, evec, ld_evec);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
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
int prime_gemv_attrs() {
    G4_CUDA(cudaFuncSetAttribute(gemv_kquant_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    G4_CUDA(cudaFuncSetAttribute(gemv_dense_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    return G4_OK;
}
}  // namespace g4
