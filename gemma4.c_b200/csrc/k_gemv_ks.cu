// k_gemv_ks.cu — K-quant GEMV for decode (batch 1..64), "k-stationary" mapping.
//
// Computes, per activation vector s and output row r of a K-quant matrix W
// (rows of n/256 super-blocks in the GGUF layouts of main.c:95-115):
//   Q4_K / Q5_K: sum_k d_x[k]*d_w*sumi_s - d_x[k]*dmin_w*sumi_m with exact
//                int32 sumi_s = sum_j sc_j * sum_32 q*q8, sumi_m = sum_j mn_j*bsum_j
//                (vec_dot_q4_K_q8_K / q5, main.c:347-593);
//   Q6_K:        sum_e x[e] * ((d*sc)*(q-32)) in fp32, the weight dequantized
//                exactly like dequant_q6_k (mm_quant_rows, main.c:213-237, 1539-1556).
//
// Mapping.  A CTA has 40 lane groups of 8 lanes.  Group g owns ONE super-block
// column k = g % nb of the matrix for the CTA's whole life (S = 40/nb groups
// share a column and split the rows), so its slice of the activation (32 Q8_K
// values or 32 floats) is loaded once into registers.  The CTA walks row tiles
// of the matrix; for each tile a group first issues all its 128-bit weight
// loads (up to IMAX rows: 32 B of Q4_K per lane per row), then reduces.  Each
// (row, block) partial lands in shared memory and the rows are summed in block
// order, so results do not depend on the grid.  Grid = 1 CTA per SM, tiles
// dealt evenly, so the weight stream is spread over all SMs without a tail.
#include <math.h>

#include "g4_internal.cuh"
#include "g4_kernels.cuh"

namespace g4 {

constexpr int kGroups = 40;                 // lane groups per CTA
constexpr int kThreads = kGroups * 8;       // 320
constexpr int kIMax = 4;                    // rows per group per tile (Q4_K/Q5_K)
template <int TYPE> constexpr int ks_rows() { return TYPE == G4_Q6_K ? 2 : kIMax; }
constexpr int kSeqChunk = 8;                // sequences reduced per pass

__device__ __forceinline__ int dp4a_u(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

__device__ __forceinline__ float gelu_k(float x) {  // gelu_f32, main.c:1490-1492
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * x * (1.0f + 0.044715f * x * x)));
}

__device__ __forceinline__ float q6_val(uint32_t w, int i) {  // byte i (0..63) -> q - 32, exact
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540 + i)) - 8388640.0f;
}

struct KsWeights {            // one row's slice of super-block k for this lane
    uint4 a, b, c;            // Q4: a=meta b=qs   Q5: +c=qh   Q6: a=ql b=qh c.x/y=scales c.z=d
};

struct KsAct {                // this lane's slice of the activation for block k
    uint32_t lo[4], hi[4];    // Q8_K values (Q4/Q5)
    float dx;
    int bs2;
    float xl[16], xh[16];     // fp32 values (Q6)
};

__device__ __forceinline__ void ks_load_w(KsWeights &w, const uint8_t *W, int type, size_t nblk_total, size_t bi, int c) {
    if (type == G4_Q6_K) {
        const Q6Planes P = q6_planes(W, nblk_total);
        const int n6 = c >> 2, par = c & 1;
        w.a = __ldg(P.ql + bi * 8 + c);
        w.b = __ldg(P.qh + bi * 4 + 2 * n6 + par);
        const uint2 s = __ldg(reinterpret_cast<const uint2 *>(P.sc + bi) + n6);
        w.c = make_uint4(s.x, s.y, (uint32_t)__ldg(P.d + bi), 0u);
    } else if (type == G4_Q4_K) {
        const uint4 *blk = reinterpret_cast<const uint4 *>(W + bi * 144);
        w.a = __ldg(blk);
        w.b = __ldg(blk + 1 + c);
    } else {
        const uint4 *blk = reinterpret_cast<const uint4 *>(W + bi * 176);
        w.a = __ldg(blk);
        w.c = __ldg(blk + 1 + (c & 1));
        w.b = __ldg(blk + 3 + c);
    }
}

__device__ __forceinline__ void ks_load_act(KsAct &A, const void *act, int act_stride, int type, int nb, int s, int k,
                                            int c) {
    if (type == G4_Q6_K) {
        const int n6 = c >> 2, second = (c >> 1) & 1, par = c & 1;
        const float *x = (const float *)act + (size_t)s * act_stride + (size_t)k * G4_QK + 128 * n6 + 32 * second + 16 * par;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 u = __ldg(reinterpret_cast<const float4 *>(x) + i);
            const float4 v = __ldg(reinterpret_cast<const float4 *>(x + 64) + i);
            A.xl[4 * i] = u.x; A.xl[4 * i + 1] = u.y; A.xl[4 * i + 2] = u.z; A.xl[4 * i + 3] = u.w;
            A.xh[4 * i] = v.x; A.xh[4 * i + 1] = v.y; A.xh[4 * i + 2] = v.z; A.xh[4 * i + 3] = v.w;
        }
    } else {
        const int j = c >> 1, h = c & 1;
        const uint8_t *qb = (const uint8_t *)act + ((size_t)s * nb + k) * G4_Q8_BYTES;
        const uint32_t *q = reinterpret_cast<const uint32_t *>(qb + 4);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            A.lo[i] = __ldg(q + (64 * j + 16 * h) / 4 + i);
            A.hi[i] = __ldg(q + (64 * j + 32 + 16 * h) / 4 + i);
        }
        A.dx = __ldg(reinterpret_cast<const float *>(qb));
        const uint32_t bp = __ldg(reinterpret_cast<const uint32_t *>(qb + 260) + c);  // bsums[2c], bsums[2c+1]
        A.bs2 = (int)(int16_t)(bp & 0xffffu) + (int)(int16_t)(bp >> 16);
    }
}

// This lane's share of the (row, block) partial; reduced over the 8 lanes by the caller.
__device__ __forceinline__ float ks_partial(const KsWeights &w, const KsAct &A, int type, int c, int &ps, int &pm) {
    if (type == G4_Q6_K) {
        const int second = (c >> 1) & 1, par = c & 1, sidx = 2 * second + par;
        const float d = f16_to_f32((uint16_t)w.c.z);
        const int sc_lo = (int)(int8_t)((w.c.x >> (8 * sidx)) & 0xffu);
        const int sc_hi = (int)(int8_t)((w.c.y >> (8 * sidx)) & 0xffu);
        const float dsl = d * (float)sc_lo, dsh = d * (float)sc_hi;
        const uint32_t ql[4] = {w.a.x, w.a.y, w.a.z, w.a.w}, qh[4] = {w.b.x, w.b.y, w.b.z, w.b.w};
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t lo = (ql[i] & 0x0F0F0F0Fu) | (((qh[i] >> (2 * second)) & 0x03030303u) << 4);
            const uint32_t hi = ((ql[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> (4 + 2 * second)) & 0x03030303u) << 4);
#pragma unroll
            for (int b = 0; b < 4; b++) {
                acc = fmaf(A.xl[4 * i + b], dsl * q6_val(lo, b), acc);
                acc = fmaf(A.xh[4 * i + b], dsh * q6_val(hi, b), acc);
            }
        }
        return acc;
    }
    const int j = c >> 1;
    const uint32_t qw[4] = {w.b.x, w.b.y, w.b.z, w.b.w};
    const uint32_t hw[4] = {w.c.x, w.c.y, w.c.z, w.c.w};
    int dl = 0, dh = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint32_t lo = qw[i] & 0x0F0F0F0Fu, hi = (qw[i] >> 4) & 0x0F0F0F0Fu;
        if (type == G4_Q5_K) {  // 5th bit: bit 2j (low nibbles) / 2j+1 (high) of qh
            lo |= ((hw[i] >> (2 * j)) & 0x01010101u) << 4;
            hi |= ((hw[i] >> (2 * j + 1)) & 0x01010101u) << 4;
        }
        dl = dp4a_u(lo, A.lo[i], dl);
        dh = dp4a_u(hi, A.hi[i], dh);
    }
    int sc_lo, mn_lo, sc_hi, mn_hi, sc_c, mn_c;
    k4_scale_min(2 * j, w.a.y, w.a.z, w.a.w, sc_lo, mn_lo);
    k4_scale_min(2 * j + 1, w.a.y, w.a.z, w.a.w, sc_hi, mn_hi);
    k4_scale_min(c, w.a.y, w.a.z, w.a.w, sc_c, mn_c);
    ps = sc_lo * dl + sc_hi * dh;
    pm = mn_c * A.bs2;
    return 0.0f;
}

template <int TYPE, int IM = ks_rows<TYPE>()>
__device__ __forceinline__ void ks_load_rows(KsWeights (&w)[IM], bool (&rv)[IM], const GemvJob &J, int row0,
                                             int T, int RS, int S, int slot, int k, bool gact, size_t nblk_total,
                                             int c) {
#pragma unroll
    for (int i = 0; i < IM; i++) {
        const int rr = slot + S * i;  // row slot within [0, RS): first T rows from w, next T from w2
        const int m = rr >= T ? 1 : 0, rl = rr - m * T;
        rv[i] = gact && rr < RS && row0 + rl < J.rows;
        const int row = min(row0 + rl, J.rows - 1);
        if (rv[i]) ks_load_w(w[i], (const uint8_t *)(m ? J.w2 : J.w), TYPE, nblk_total, (size_t)row * (J.n / G4_QK) + k, c);
        else w[i].a = w[i].b = w[i].c = make_uint4(0, 0, 0, 0);
    }
}

// One CTA per SM (no register spills at this size); the next tile's weight
// loads are issued before the current tile's reduction barrier, so the
// weight stream keeps flowing while partials are summed.
template <int TYPE>
__global__ void __launch_bounds__(kThreads, 1) gemv_ks_kernel(GemvJobs jobs, int B) {
    extern __shared__ __align__(16) float red[];  // [kSeqChunk][nmat*T][nb]
    __shared__ unsigned long long best[kSeqChunk];
    // job of this CTA (uniform; a by-value copy keeps the parameters out of local memory)
    const int bx = (int)blockIdx.x;
    const GemvJob J = (jobs.njobs > 2 && bx >= jobs.j[2].cta_begin) ? jobs.j[2]
                    : (jobs.njobs > 1 && bx >= jobs.j[1].cta_begin) ? jobs.j[1] : jobs.j[0];
    constexpr int type = TYPE;
    const int nb = J.n / G4_QK, rows = J.rows, T = J.rt;
    const int nmat = J.w2 ? 2 : 1, RS = nmat * T;
    const int S = nb <= kGroups ? kGroups / nb : 1;              // groups per block column
    const int kchunks = (nb + kGroups - 1) / kGroups;
    const int tid = threadIdx.x, lane = tid & 31, c = lane & 7, g = tid >> 3;
    const int cta = bx - J.cta_begin, nctas = J.ctas;
    const int ntiles = (rows + T - 1) / T;
    const size_t nblk_total = (size_t)rows * nb;
    const int slot = nb <= kGroups ? g / nb : 0;

    for (int kc = 0; kc < kchunks; kc++) {
        const int kk = nb <= kGroups ? g % nb : kc * kGroups + g;
        const bool gact = (nb <= kGroups ? slot < S : kk < nb);
        const int k = gact ? kk : 0;
        KsAct A;  // batch 1: the activation stays in registers for the whole pass
        ks_load_act(A, J.act, J.act_stride, type, nb, 0, k, c);
        constexpr int IM = ks_rows<TYPE>();
        KsWeights w[IM];
        bool rv[IM];
        if (cta < ntiles) ks_load_rows<TYPE>(w, rv, J, cta * T, T, RS, S, slot, k, gact, nblk_total, c);
        for (int tile = cta; tile < ntiles; tile += nctas) {
            const int row0 = tile * T;
            for (int s0 = 0; s0 < B; s0 += kSeqChunk) {
                const int ns = min(kSeqChunk, B - s0);
                for (int si = 0; si < ns; si++) {
                    if (B > 1) ks_load_act(A, J.act, J.act_stride, type, nb, s0 + si, k, c);
#pragma unroll
                    for (int i = 0; i < IM; i++) {
                        int ps = 0, pm = 0;
                        float f = ks_partial(w[i], A, type, c, ps, pm);
#pragma unroll
                        for (int o = 4; o > 0; o >>= 1) {
                            if (type == G4_Q6_K) {
                                f += __shfl_xor_sync(0xffffffffu, f, o, 8);
                            } else {
                                ps += __shfl_xor_sync(0xffffffffu, ps, o, 8);
                                pm += __shfl_xor_sync(0xffffffffu, pm, o, 8);
                            }
                        }
                        if (c == 0 && rv[i]) {
                            if (type != G4_Q6_K) {
                                const float dd = A.dx * f16_to_f32((uint16_t)(w[i].a.x & 0xffffu));
                                const float dm = A.dx * f16_to_f32((uint16_t)(w[i].a.x >> 16));
                                f = fmaf(-dm, (float)pm, dd * (float)ps);
                            }
                            red[((size_t)si * RS + slot + S * i) * nb + k] = f;
                        }
                    }
                }
                const bool last_seq_chunk = s0 + kSeqChunk >= B;
                if (last_seq_chunk && tile + nctas < ntiles)  // prefetch the next tile before the barrier
                    ks_load_rows<TYPE>(w, rv, J, (tile + nctas) * T, T, RS, S, slot, k, gact, nblk_total, c);
                if (kc + 1 < kchunks) continue;  // more block columns of this tile to come
                if (tid < kSeqChunk) best[tid] = 0ull;
                __syncthreads();
                // epilogue: one thread per (sequence, row), blocks summed in order
                for (int idx = tid; idx < ns * T; idx += kThreads) {
                    const int si = idx / T, rl = idx % T, row = row0 + rl, s = s0 + si;
                    if (row >= rows) continue;
                    const float *rp = red + ((size_t)si * RS + rl) * nb;
                    float a = 0.0f;
                    for (int kb = 0; kb < nb; kb++) a += rp[kb];
                    float *out = J.out ? J.out + (size_t)s * J.out_stride : nullptr;
                    if (J.epi == EPI_GELU_MUL) {
                        const float *rq = red + ((size_t)si * RS + T + rl) * nb;
                        float b = 0.0f;
                        for (int kb = 0; kb < nb; kb++) b += rq[kb];
                        out[row] = gelu_k(a) * b;
                    } else if (J.epi == EPI_SOFTCAP_ARGMAX) {
                        if (J.cap > 0.0f) a = J.cap * tanhf(a * (1.0f / J.cap));
                        if (out) out[row] = a;
                        atomicMax(&best[si], argmax_key(a, row));
                    } else if (J.epi == EPI_GELU_SCALE) {
                        out[row] = gelu_k(a) * J.evec[(size_t)s * J.ld_evec + row];
                    } else {
                        out[row] = a;
                    }
                }
                __syncthreads();
                if (J.epi == EPI_SOFTCAP_ARGMAX && tid < ns && best[tid]) atomicMax(J.amax + s0 + tid, best[tid]);
            }
        }
    }
}

// Rows per tile and CTAs for one job (1 CTA per SM, tiles dealt evenly).
static void ks_plan(GemvJob &J, int sms) {
    const int nb = J.n / G4_QK;
    const int S = nb <= kGroups ? kGroups / nb : 1;
    const int nmat = J.w2 ? 2 : 1;
    const int im = J.type == G4_Q6_K ? ks_rows<G4_Q6_K>() : kIMax;
    const int tmax = (S * im) / nmat;                       // rows per matrix a tile can hold
    const int grid = sms;
    const int rpc = (J.rows + grid - 1) / grid;             // rows per CTA if all CTAs work
    const int ntile_cta = (rpc + tmax - 1) / tmax;
    int T = (rpc + ntile_cta - 1) / ntile_cta;
    if (T < 1) T = 1;
    if (T > tmax) T = tmax;
    J.rt = T;
    const int ntiles = (J.rows + T - 1) / T;
    J.ctas = ntiles < grid ? ntiles : grid;
}

static int g_sms = 0;

int launch_gemv_kquant(GemvJobs &jobs, int B, cudaStream_t st) {
    if (g_sms == 0) {
        int dev = 0;
        G4_CUDA(cudaGetDevice(&dev));
        G4_CUDA(cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev));
    }
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
        if (J.type == G4_Q6_K && J.act_stride % 4) {
            set_error(G4_ERR_ARG, "gemv: fp32 activation stride %d not a multiple of 4", J.act_stride);
            return G4_ERR_ARG;
        }
        ks_plan(J, g_sms);
        if (J.n / G4_QK > kGroups && (B > kSeqChunk || J.ctas < (J.rows + J.rt - 1) / J.rt)) {
            // rows longer than 40 super-blocks: every tile needs its own CTA and one sequence chunk
            J.ctas = (J.rows + J.rt - 1) / J.rt;
            if (B > kSeqChunk) {
                set_error(G4_ERR_ARG, "gemv: n=%d with batch %d > %d unsupported", J.n, B, kSeqChunk);
                return G4_ERR_ARG;
            }
        }
        if (i > 0 && J.type != jobs.j[0].type) {
            set_error(G4_ERR_ARG, "gemv: one launch takes one tensor type");
            return G4_ERR_ARG;
        }
        J.cta_begin = ctas;
        ctas += J.ctas;
        const int nb = J.n / G4_QK;
        const size_t b = sizeof(float) * (size_t)kSeqChunk * (J.w2 ? 2 : 1) * J.rt * nb;
        smem = b > smem ? b : smem;
    }
    if (ctas == 0 || B <= 0) return G4_OK;
    if (smem > 200 * 1024) {
        set_error(G4_ERR_ARG, "gemv: tile too large for shared memory (%zu bytes)", smem);
        return G4_ERR_ARG;
    }
    switch (jobs.j[0].type) {
    case G4_Q4_K: gemv_ks_kernel<G4_Q4_K><<<ctas, kThreads, smem, st>>>(jobs, B); break;
    case G4_Q5_K: gemv_ks_kernel<G4_Q5_K><<<ctas, kThreads, smem, st>>>(jobs, B); break;
    default: gemv_ks_kernel<G4_Q6_K><<<ctas, kThreads, smem, st>>>(jobs, B); break;
    }
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

int prime_gemv_ks_attrs() {
    G4_CUDA(cudaFuncSetAttribute(gemv_ks_kernel<G4_Q4_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    G4_CUDA(cudaFuncSetAttribute(gemv_ks_kernel<G4_Q5_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    G4_CUDA(cudaFuncSetAttribute(gemv_ks_kernel<G4_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    return G4_OK;
}

}  // namespace g4
