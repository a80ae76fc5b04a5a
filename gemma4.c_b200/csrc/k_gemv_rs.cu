// k_gemv_rs.cu — K-quant GEMV for decode (batch 1..8 per pass), row-stationary.
//
// Computes, per activation vector s and output row r of a K-quant matrix W
// (rows of n/256 super-blocks in the GGUF layouts of main.c:95-115):
//   Q4_K / Q5_K: sum_k d_x*d_w*sumi_s - d_x*dmin_w*sumi_m with the integer
//                dot structure of vec_dot_q4_K_q8_K / q5 (main.c:347-593):
//                int32 sumi_s = sum_j sc_j * sum_32 q*q8, sumi_m = sum_j mn_j*bsum_j;
//   Q6_K:        sum_e x[e] * ((d*sc)*(q-32)) in fp32, the weight dequantized
//                exactly like dequant_q6_k (mm_quant_rows, main.c:213-237, 1539-1556).
//
// Mapping.  A CTA has 40 lane groups of 8 lanes (10 warps).  1, 2 or 4
// groups of one warp own an output row (R = 1 row; 2 rows for the fused
// gate/up product), each summing a contiguous run of its super-blocks, so the
// hot loop has no barrier: the 8 lanes split each 256-weight super-block (16
// bytes of quants each), issue the 128-bit loads of KU super-blocks at once,
// accumulate per-lane fp32 partials and reduce them with 3-5 shuffles at the
// end.  The activation (Q8_K values or fp32) sits in shared memory, staged
// once per CTA or computed there by the fused prologue; the first weight
// loads are issued before that, so staging hides under them.  Rows are dealt
// round-robin over the warps of a persistent grid (2 CTAs per SM), so every
// SM streams the same share of the weights.
#include <math.h>

#include "g4_internal.cuh"
#include "g4_kernels.cuh"

namespace g4 {

constexpr int kRsGroups = 40;
constexpr int kRsThreads = kRsGroups * 8;  // 320

__device__ __forceinline__ float rs_gelu(float x) {  // gelu_f32, main.c:1490-1492
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * x * (1.0f + 0.044715f * x * x)));
}

__device__ __forceinline__ float rs_q6(uint32_t w, int i) {  // byte i (0..63) -> q - 32, exact
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540 + i)) - 8388640.0f;
}

// Activation staging in shared memory for NBc sequences.
struct RsAct {
    int8_t *qs;   // [NBc][n]      Q8_K quants           (Q4/Q5)
    float *dx;    // [NBc][nb]     Q8_K block scales
    int *bs2;     // [NBc][nb][8]  sums of 32 quants per sub-block
    float *x;     // [NBc][n]      fp32 activation       (Q6)
};

// Q4_K/Q5_K block meta (d, dmin, 12 scale bytes) -> this lane's two 6-bit
// scales (sub-blocks 2j, 2j+1) and its min (sub-block c).  The 12-byte
// packing of get_scale_min_k4 (main.c:162-170) unpacked word-wise, branch-free.
__device__ __forceinline__ void rs_scales(const uint4 &m, int j, int c, int &sc_lo, int &sc_hi, int &mn_c) {
    const uint32_t s0 = m.y, s1 = m.z, s2 = m.w;
    const uint32_t sc03 = s0 & 0x3f3f3f3fu;
    const uint32_t sc47 = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);
    const uint32_t mn03 = s1 & 0x3f3f3f3fu;
    const uint32_t mn47 = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);
    sc_lo = (int)__byte_perm(sc03, sc47, 0x4440 | (2 * j)) & 0xff;
    sc_hi = (int)__byte_perm(sc03, sc47, 0x4440 | (2 * j + 1)) & 0xff;
    mn_c = (int)__byte_perm(mn03, mn47, 0x4440 | c) & 0xff;
}

template <int TYPE> constexpr int rs_ku(int R) {  // super-blocks per load chunk (registers)
    return TYPE == G4_Q6_K ? (R == 1 ? 3 : 2) : TYPE == G4_Q5_K ? (R == 1 ? 4 : 2) : (R == 1 ? 5 : 3);
}

template <int TYPE, int KU, int R>
struct RsChunk {
    uint4 a[KU][R], b[KU][R], c[KU][R];
};

// Issue the loads of super-blocks [k0, k0+KU) (clamped to ke) of `row`.
template <int TYPE, int KU, int R>
__device__ __forceinline__ void rs_load(RsChunk<TYPE, KU, R> &w, const GemvJob &J, int row, int k0, int ke, int c) {
    const int nb = J.n / G4_QK;
    const size_t nblk_total = (size_t)J.rows * nb;
    const int n6 = c >> 2, par = c & 1, h = c & 1;
#pragma unroll
    for (int u = 0; u < KU; u++) {
        const int k = min(k0 + u, ke - 1);
#pragma unroll
        for (int r = 0; r < R; r++) {
            const uint8_t *W = (const uint8_t *)(r ? J.w2 : J.w);
            const size_t bi = (size_t)row * nb + k;
            if (TYPE == G4_Q6_K) {
                const Q6Planes P = q6_planes(W, nblk_total);
                w.a[u][r] = __ldg(P.ql + bi * 8 + c);
                w.b[u][r] = __ldg(P.qh + bi * 4 + 2 * n6 + par);
                const uint2 sc = __ldg(reinterpret_cast<const uint2 *>(P.sc + bi) + n6);
                w.c[u][r] = make_uint4(sc.x, sc.y, (uint32_t)__ldg(P.d + bi), 0u);
            } else if (TYPE == G4_Q4_K) {
                const uint4 *blk = reinterpret_cast<const uint4 *>(W + bi * 144);
                w.a[u][r] = __ldg(blk);
                w.b[u][r] = __ldg(blk + 1 + c);
            } else {
                const uint4 *blk = reinterpret_cast<const uint4 *>(W + bi * 176);
                w.a[u][r] = __ldg(blk);
                w.c[u][r] = __ldg(blk + 1 + h);
                w.b[u][r] = __ldg(blk + 3 + c);
            }
        }
    }
}

// Accumulate the loaded chunk into acc[s][r] for the staged sequences.
template <int TYPE, int KU, int R, int NB>
__device__ __forceinline__ void rs_compute(const RsChunk<TYPE, KU, R> &w, const GemvJob &J, const RsAct &A, int nbc,
                                           int k0, int ke, float (&acc)[NB][R], int c) {
    const int nb = J.n / G4_QK;
    const int j = c >> 1, h = c & 1;
    const int n6 = c >> 2, second = (c >> 1) & 1, par = c & 1;
#pragma unroll
    for (int u = 0; u < KU; u++) {
        const int k = k0 + u;
        if (k >= ke) break;
#pragma unroll
        for (int r = 0; r < R; r++) {
            if (TYPE == G4_Q6_K) {
                const int sidx = 2 * second + par;
                const float d = f16_to_f32((uint16_t)w.c[u][r].z);
                const float dsl = d * (float)(int)(int8_t)((w.c[u][r].x >> (8 * sidx)) & 0xffu);
                const float dsh = d * (float)(int)(int8_t)((w.c[u][r].y >> (8 * sidx)) & 0xffu);
                const uint32_t ql[4] = {w.a[u][r].x, w.a[u][r].y, w.a[u][r].z, w.a[u][r].w};
                const uint32_t qh[4] = {w.b[u][r].x, w.b[u][r].y, w.b[u][r].z, w.b[u][r].w};
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    lo[i] = (ql[i] & 0x0F0F0F0Fu) | (((qh[i] >> (2 * second)) & 0x03030303u) << 4);
                    hi[i] = ((ql[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> (4 + 2 * second)) & 0x03030303u) << 4);
                }
                const int e_lo = k * G4_QK + 128 * n6 + 32 * second + 16 * par;
#pragma unroll
                for (int s = 0; s < NB; s++) {
                    if (s >= nbc) break;
                    const float4 *xl = reinterpret_cast<const float4 *>(A.x + (size_t)s * J.n + e_lo);
                    float a = acc[s][r];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float4 vl = xl[i], vh = xl[16 + i];  // +64 elements
                        a = fmaf(vl.x, dsl * rs_q6(lo[i], 0), a);
                        a = fmaf(vl.y, dsl * rs_q6(lo[i], 1), a);
                        a = fmaf(vl.z, dsl * rs_q6(lo[i], 2), a);
                        a = fmaf(vl.w, dsl * rs_q6(lo[i], 3), a);
                        a = fmaf(vh.x, dsh * rs_q6(hi[i], 0), a);
                        a = fmaf(vh.y, dsh * rs_q6(hi[i], 1), a);
                        a = fmaf(vh.z, dsh * rs_q6(hi[i], 2), a);
                        a = fmaf(vh.w, dsh * rs_q6(hi[i], 3), a);
                    }
                    acc[s][r] = a;
                }
            } else {
                const uint32_t qw[4] = {w.b[u][r].x, w.b[u][r].y, w.b[u][r].z, w.b[u][r].w};
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    lo[i] = qw[i] & 0x0F0F0F0Fu;
                    hi[i] = (qw[i] >> 4) & 0x0F0F0F0Fu;
                }
                if (TYPE == G4_Q5_K) {  // 5th bit: bit 2j (low nibbles) / 2j+1 (high) of qh
                    const uint32_t hw[4] = {w.c[u][r].x, w.c[u][r].y, w.c[u][r].z, w.c[u][r].w};
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        lo[i] |= ((hw[i] >> (2 * j)) & 0x01010101u) << 4;
                        hi[i] |= ((hw[i] >> (2 * j + 1)) & 0x01010101u) << 4;
                    }
                }
                int sc_lo, sc_hi, mn_c;
                rs_scales(w.a[u][r], j, c, sc_lo, sc_hi, mn_c);
                const float dw = f16_to_f32((uint16_t)(w.a[u][r].x & 0xffffu));
                const float dmw = f16_to_f32((uint16_t)(w.a[u][r].x >> 16));
#pragma unroll
                for (int s = 0; s < NB; s++) {
                    if (s >= nbc) break;
                    const int8_t *q8 = A.qs + (size_t)s * J.n + k * G4_QK + 64 * j + 16 * h;
                    const uint4 al = *reinterpret_cast<const uint4 *>(q8);
                    const uint4 ah = *reinterpret_cast<const uint4 *>(q8 + 32);
                    int dl = __dp4a((int)lo[0], (int)al.x, 0);
                    dl = __dp4a((int)lo[1], (int)al.y, dl);
                    dl = __dp4a((int)lo[2], (int)al.z, dl);
                    dl = __dp4a((int)lo[3], (int)al.w, dl);
                    int dh = __dp4a((int)hi[0], (int)ah.x, 0);
                    dh = __dp4a((int)hi[1], (int)ah.y, dh);
                    dh = __dp4a((int)hi[2], (int)ah.z, dh);
                    dh = __dp4a((int)hi[3], (int)ah.w, dh);
                    const float dx = A.dx[s * nb + k];
                    const int ps = sc_lo * dl + sc_hi * dh;
                    const int pm = mn_c * A.bs2[(s * nb + k) * 8 + c];
                    acc[s][r] = fmaf(dx * dw, (float)ps, fmaf(-(dx * dmw), (float)pm, acc[s][r]));
                }
            }
        }
    }
}

// Stage (or compute, with the fused prologue) the activation of sequences
// [s0, s0+nbc) into shared memory.  Ends with a CTA barrier.
template <int TYPE, int NB>
__device__ __forceinline__ void rs_stage(const GemvJobs &jobs, const GemvJob &J, RsAct &A, float *pro_x, int s0,
                                         int nbc, bool writer, float *pred) {
    const int n = J.n, nb = n / G4_QK, tid = threadIdx.x, lane = tid & 31;
    if (jobs.has_pro) {
        Prologue P = jobs.pro;
        P.x_in += (size_t)s0 * P.dim;
        if (P.delta) P.delta += (size_t)s0 * P.dim;
        if (P.x_out) P.x_out += (size_t)s0 * P.dim;
        if (P.xn_out) P.xn_out += (size_t)s0 * P.dim;
        float *xs = TYPE == G4_Q6_K ? A.x : pro_x;
        prologue_run(P, nbc, xs, nullptr, writer, pred);
        if (TYPE != G4_Q6_K) {  // quantize into planes
            const int warp = tid >> 5, nw = blockDim.x >> 5;
            for (int t = warp; t < nbc * nb; t += nw) {
                const int s = t / nb, k = t % nb;
                uint32_t q[2];
                float d;
                int ls;
                warp_quant_block(xs + (size_t)s * n + (size_t)k * G4_QK, lane, q, d, ls);
                uint32_t *dst = reinterpret_cast<uint32_t *>(A.qs + (size_t)s * n + (size_t)k * G4_QK + 8 * lane);
                dst[0] = q[0];
                dst[1] = q[1];
                int sub = ls + __shfl_xor_sync(0xffffffffu, ls, 1);
                sub += __shfl_xor_sync(0xffffffffu, sub, 2);
                if ((lane & 3) == 0) A.bs2[(s * nb + k) * 8 + (lane >> 2)] = sub;
                if (lane == 0) A.dx[s * nb + k] = d;
            }
        }
    } else if (TYPE == G4_Q6_K) {
        for (int s = 0; s < nbc; s++) {
            const float4 *src = reinterpret_cast<const float4 *>((const float *)J.act + (size_t)(s0 + s) * J.act_stride);
            float4 *dst = reinterpret_cast<float4 *>(A.x + (size_t)s * n);
            for (int i = tid; i < n / 4; i += blockDim.x) dst[i] = src[i];
        }
    } else {
        const uint8_t *src = (const uint8_t *)J.act + (size_t)s0 * nb * G4_Q8_BYTES;
        for (int i = tid; i < nbc * nb * 64; i += blockDim.x) {
            const int blk = i >> 6, w = i & 63;
            reinterpret_cast<uint32_t *>(A.qs)[blk * 64 + w] =
                *reinterpret_cast<const uint32_t *>(src + (size_t)blk * G4_Q8_BYTES + 4 + 4 * w);
        }
        for (int i = tid; i < nbc * nb * 8; i += blockDim.x) {
            const int blk = i >> 3, jj = i & 7;
            const int16_t *bs = reinterpret_cast<const int16_t *>(src + (size_t)blk * G4_Q8_BYTES + 260);
            A.bs2[i] = (int)bs[2 * jj] + (int)bs[2 * jj + 1];
            if (jj == 0) A.dx[blk] = *reinterpret_cast<const float *>(src + (size_t)blk * G4_Q8_BYTES);
        }
    }
    __syncthreads();
}

// Units: a warp takes 4/GPR rows per round (GPR lane groups per row, each
// summing a contiguous run of the row's super-blocks); warp-round wu =
// cta + nctas * (warp + 10 * round).
template <int TYPE, int NB, int R>
__global__ void __launch_bounds__(kRsThreads, 2) gemv_rs_kernel(GemvJobs jobs, int B) {
    constexpr int KU = rs_ku<TYPE>(R);
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ unsigned long long best[NB];
    __shared__ float pred[8];
    const int bx = (int)blockIdx.x;
    const GemvJob J = (jobs.njobs > 2 && bx >= jobs.j[2].cta_begin) ? jobs.j[2]
                    : (jobs.njobs > 1 && bx >= jobs.j[1].cta_begin) ? jobs.j[1] : jobs.j[0];
    const int n = J.n, nb = n / G4_QK;
    const int tid = threadIdx.x, lane = tid & 31, c = lane & 7, warp = tid >> 5, q = (lane >> 3);
    const int cta = bx - J.cta_begin, nctas = J.ctas;
    const int GPR = J.rt;                      // lane groups per row (1, 2, 4)
    const int rpw = 4 / GPR;                   // rows per warp-round
    const int part = q % GPR;
    const int bpg = (nb + GPR - 1) / GPR;      // super-blocks per group
    const int kb = min(part * bpg, nb), ke = min(kb + bpg, nb);

    RsAct A;
    uint8_t *p = smem;
    if (TYPE == G4_Q6_K) {
        A.x = (float *)p;
        p += (size_t)NB * n * 4;
    } else {
        A.qs = (int8_t *)p;
        p += (size_t)NB * n;
        A.dx = (float *)p;
        p += (size_t)NB * nb * 4;
        A.bs2 = (int *)p;
        p += (size_t)NB * nb * 32;
    }
    float *pro_x = (float *)(((uintptr_t)p + 15) & ~(uintptr_t)15);  // prologue scratch [NB][n] (Q4/Q5)

    for (int s0 = 0; s0 < B; s0 += NB) {
        const int nbc = min(NB, B - s0);
        if (s0 > 0) __syncthreads();  // previous pass done with the staged activation
        if (tid < NB) best[tid] = 0ull;
        unsigned long long mykey[NB];
#pragma unroll
        for (int s = 0; s < NB; s++) mykey[s] = 0ull;
        RsChunk<TYPE, KU, R> w;
        // first chunk of round 0 is issued before the activation is staged
        int row0 = (cta + nctas * warp) * rpw + q / GPR;
        bool v0 = (long)(cta + nctas * warp) * rpw < J.rows && row0 < J.rows && kb < ke;
        if (v0) rs_load<TYPE, KU, R>(w, J, row0, kb, ke, c);
        rs_stage<TYPE, NB>(jobs, J, A, pro_x, s0, nbc, jobs.pro_writer && bx == 0, pred);
        for (int round = 0;; round++) {
            const long wu = (long)cta + (long)nctas * (warp + 10L * round);
            if (wu * rpw >= J.rows) break;  // uniform per warp
            const int row = (int)(wu * rpw) + q / GPR;
            const bool valid = row < J.rows && kb < ke;
            float acc[NB][R];
#pragma unroll
            for (int s = 0; s < NB; s++)
#pragma unroll
                for (int r = 0; r < R; r++) acc[s][r] = 0.0f;
            for (int k0 = kb; k0 < ke; k0 += KU) {
                if (!(round == 0 && k0 == kb)) {
                    if (valid) rs_load<TYPE, KU, R>(w, J, row, k0, ke, c);
                }
                if (valid) rs_compute<TYPE, KU, R, NB>(w, J, A, nbc, k0, ke, acc, c);
            }
#pragma unroll
            for (int s = 0; s < NB; s++)
#pragma unroll
                for (int r = 0; r < R; r++) {
                    float v = acc[s][r];
                    v += __shfl_xor_sync(0xffffffffu, v, 4);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    if (GPR >= 2) v += __shfl_xor_sync(0xffffffffu, v, 8);
                    if (GPR >= 4) v += __shfl_xor_sync(0xffffffffu, v, 16);
                    acc[s][r] = v;
                }
            if (c == 0 && part == 0 && row < J.rows) {
#pragma unroll
                for (int s = 0; s < NB; s++) {
                    if (s >= nbc) break;
                    float a = acc[s][0];
                    float *out = J.out ? J.out + (size_t)(s0 + s) * J.out_stride : nullptr;
                    if (J.epi == EPI_GELU_MUL) {
                        out[row] = rs_gelu(a) * acc[s][R - 1];
                    } else if (J.epi == EPI_SOFTCAP_ARGMAX) {
                        if (J.cap > 0.0f) a = J.cap * tanhf(a * (1.0f / J.cap));
                        if (out) out[row] = a;
                        const unsigned long long kk = argmax_key(a, row);
                        mykey[s] = kk > mykey[s] ? kk : mykey[s];
                    } else if (J.epi == EPI_GELU_SCALE) {
                        out[row] = rs_gelu(a) * J.evec[(size_t)(s0 + s) * J.ld_evec + row];
                    } else {
                        out[row] = a;
                    }
                }
            }
        }
        if (J.epi == EPI_SOFTCAP_ARGMAX) {
#pragma unroll
            for (int s = 0; s < NB; s++) {
                unsigned long long kk = mykey[s];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long ok = __shfl_xor_sync(0xffffffffu, kk, o);
                    kk = ok > kk ? ok : kk;
                }
                if (lane == 0 && kk) atomicMax(&best[s], kk);
            }
            __syncthreads();
            if (tid < nbc && best[tid]) atomicMax(J.amax + s0 + tid, best[tid]);
        }
    }
}

static int g_rs_sms = 0;

template <int TYPE>
static size_t rs_smem(int nb_seq, int n) {
    const int nb = n / G4_QK;
    if (TYPE == G4_Q6_K) return (size_t)nb_seq * n * 4 + 16;
    return (size_t)nb_seq * n + (size_t)nb_seq * nb * 36 + 16 + (size_t)nb_seq * n * 4;  // + prologue scratch
}

template <int TYPE, int NB>
static void rs_launch(GemvJobs &jobs, int ctas, size_t smem, int B, cudaStream_t st) {
    if (jobs.j[0].w2) gemv_rs_kernel<TYPE, NB, 2><<<ctas, kRsThreads, smem, st>>>(jobs, B);
    else gemv_rs_kernel<TYPE, NB, 1><<<ctas, kRsThreads, smem, st>>>(jobs, B);
}

template <int TYPE>
static int rs_dispatch(GemvJobs &jobs, int ctas, int B, cudaStream_t st) {
    int n = jobs.j[0].n;
    for (int i = 1; i < jobs.njobs; i++) n = jobs.j[i].n > n ? jobs.j[i].n : n;
    // sequences per pass: as many as fit in shared memory (weights are re-read per pass)
    int nbs = B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : 8;
    while (nbs > 1 && rs_smem<TYPE>(nbs, n) > 200 * 1024) nbs /= 2;
    const size_t smem = rs_smem<TYPE>(nbs, n);
    if (smem > 200 * 1024) {
        set_error(G4_ERR_ARG, "gemv: activation of n=%d does not fit in shared memory", n);
        return G4_ERR_ARG;
    }
    switch (nbs) {
    case 1: rs_launch<TYPE, 1>(jobs, ctas, smem, B, st); break;
    case 2: rs_launch<TYPE, 2>(jobs, ctas, smem, B, st); break;
    case 4: rs_launch<TYPE, 4>(jobs, ctas, smem, B, st); break;
    default: rs_launch<TYPE, 8>(jobs, ctas, smem, B, st); break;
    }
    return G4_OK;
}

int launch_gemv_kquant(GemvJobs &jobs, int B, cudaStream_t st) {
    if (g_rs_sms == 0) {
        int dev = 0;
        G4_CUDA(cudaGetDevice(&dev));
        G4_CUDA(cudaDeviceGetAttribute(&g_rs_sms, cudaDevAttrMultiProcessorCount, dev));
    }
    if (jobs.njobs < 1 || B <= 0) return G4_OK;
    const int type = jobs.j[0].type;
    if (type != G4_Q4_K && type != G4_Q5_K && type != G4_Q6_K) {
        set_error(G4_ERR_TYPE, "gemv_kquant: unsupported type %d", type);
        return G4_ERR_TYPE;
    }
    if (jobs.has_pro && (B > kFusedMaxBatch || jobs.pro.dim % G4_QK)) {
        set_error(G4_ERR_ARG, "gemv: fused prologue needs batch <= %d and dim %% 256 == 0", kFusedMaxBatch);
        return G4_ERR_ARG;
    }
    long total_work = 0;
    for (int i = 0; i < jobs.njobs; i++) total_work += (long)jobs.j[i].rows * (jobs.j[i].n / G4_QK);
    int ctas = 0;
    for (int i = 0; i < jobs.njobs; i++) {
        GemvJob &J = jobs.j[i];
        if (J.type != type) { set_error(G4_ERR_ARG, "gemv: one launch takes one tensor type"); return G4_ERR_ARG; }
        if (J.n % G4_QK || J.n <= 0 || J.rows <= 0) {
            set_error(G4_ERR_ARG, "gemv: n=%d (must be a positive multiple of 256), rows=%d", J.n, J.rows);
            return G4_ERR_ARG;
        }
        if (type == G4_Q6_K && J.act_stride % 4 && !jobs.has_pro) {
            set_error(G4_ERR_ARG, "gemv: fp32 activation stride %d not a multiple of 4", J.act_stride);
            return G4_ERR_ARG;
        }
        if (jobs.has_pro && J.n != jobs.pro.dim) {
            set_error(G4_ERR_ARG, "gemv: fused prologue dim %d != n %d", jobs.pro.dim, J.n);
            return G4_ERR_ARG;
        }
        // lane groups per row: enough that a group holds about one load chunk
        const int nbj = J.n / G4_QK;
        const int ku = type == G4_Q6_K ? 3 : type == G4_Q5_K ? 4 : 5;
        J.rt = nbj <= ku ? 1 : nbj <= 2 * ku ? 2 : 4;
        if (J.w2 && J.rt < 4 && nbj > 3) J.rt *= 2;
        // CTAs in proportion to the job's bytes (rows x super-blocks)
        const long grid = 2L * g_rs_sms;
        long cj = (grid * J.rows * nbj + total_work - 1) / total_work;
        const long warp_rounds = ((long)J.rows * J.rt + 3) / 4;
        const long need = (warp_rounds + 9) / 10;
        if (cj > need) cj = need;
        if (cj < 1) cj = 1;
        J.ctas = (int)cj;
        J.cta_begin = ctas;
        ctas += J.ctas;
    }
    int rc;
    switch (type) {
    case G4_Q4_K: rc = rs_dispatch<G4_Q4_K>(jobs, ctas, B, st); break;
    case G4_Q5_K: rc = rs_dispatch<G4_Q5_K>(jobs, ctas, B, st); break;
    default: rc = rs_dispatch<G4_Q6_K>(jobs, ctas, B, st); break;
    }
    if (rc) return rc;
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

template <int TYPE, int R>
static int rs_prime_r() {
    G4_CUDA(cudaFuncSetAttribute(gemv_rs_kernel<TYPE, 1, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    G4_CUDA(cudaFuncSetAttribute(gemv_rs_kernel<TYPE, 2, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    G4_CUDA(cudaFuncSetAttribute(gemv_rs_kernel<TYPE, 4, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    G4_CUDA(cudaFuncSetAttribute(gemv_rs_kernel<TYPE, 8, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    return G4_OK;
}
template <int TYPE>
static int rs_prime() {
    int rc = rs_prime_r<TYPE, 1>();
    return rc ? rc : rs_prime_r<TYPE, 2>();
}

int prime_gemv_ks_attrs() {
    int rc = rs_prime<G4_Q4_K>();
    rc |= rs_prime<G4_Q5_K>();
    rc |= rs_prime<G4_Q6_K>();
    return rc ? G4_ERR_CUDA : G4_OK;
}

}  // namespace g4
