// k_gemv_tma.cu — K-quant GEMV for decode (batch 1..8 per pass): weight tiles
// streamed into shared memory by bulk asynchronous copies (the TMA engine,
// cp.async.bulk) through an mbarrier ring, consumed by 16 warps.
//
// Computes, per activation vector s and output row r of a K-quant matrix W
// (rows of n/256 super-blocks in the GGUF layouts of main.c:95-115):
//   Q4_K / Q5_K: sum_k d_x*d_w*sumi_s - d_x*dmin_w*sumi_m with the integer
//                dot structure of vec_dot_q4_K_q8_K / q5 (main.c:347-593):
//                int32 sumi_s = sum_j sc_j * sum_32 q*q8, sumi_m = sum_j mn_j*bsum_j;
//   Q6_K:        sum_e x[e] * ((d*sc)*(q-32)) in fp32, the weight dequantized
//                exactly like dequant_q6_k (mm_quant_rows, main.c:213-237, 1539-1556).
//
// Batch-1 decode is a pure weight stream (0.5625 B/weight for Q4_K), so the
// kernel is built to keep HBM busy: one persistent CTA per SM; warp 8 is the
// producer and keeps S tiles (each TR contiguous rows, one bulk copy) in
// flight; warps 0-15 hold 64 lane groups of 8 lanes.  GPR groups (1, 2, 4) of
// one warp own a row of the tile and each sums a contiguous run of its
// super-blocks: the 8 lanes split a 256-weight super-block (16 bytes of
// quants each), so the reduction is 3-5 shuffles and there is no CTA barrier
// after the prologue.  The activation (Q8_K planes or fp32) is staged once in
// shared memory, or computed there by the fused residual/norm prologue while
// the first tiles are already in flight.
//
// Every wait is bounded by the global timer: after 2 s a warp records
// G4_ERR_TIMEOUT in *err, the producer drains the copies it issued, and the
// CTA returns instead of hanging the GPU.
#include <math.h>

#include <algorithm>

#include "g4_async.cuh"
#include "g4_internal.cuh"
#include "g4_kernels.cuh"

namespace g4 {

constexpr int kTmConsumerWarps = 16;
constexpr int kTmGroups = kTmConsumerWarps * 4;       // consumer lane groups
constexpr int kTmThreads = (kTmConsumerWarps + 1) * 32;  // + producer warp
constexpr int kTmMaxStages = 6;

// ---------------------------------------------------------------- activation
struct TmAct {
    int8_t *qs;   // [NB][n]      Q8_K quants           (Q4/Q5)
    float *dx;    // [NB][nb]     Q8_K block scales     (Q4/Q5)
    int *bs2;     // [NB][nb][8]  sums of 32 quants per sub-block (Q4/Q5)
    int8_t *pc;   // [NB][3][n]   fixed-point activation pieces (Q6, q6x_block)
    float *ys;    // [NB][nb]     their block scales 2^(E-22) (Q6)
};

// Q4_K/Q5_K block meta (d, dmin, 12 scale bytes) -> this lane's two 6-bit
// scales (sub-blocks 2j, 2j+1) and its min (sub-block c): the packing of
// get_scale_min_k4 (main.c:162-170) unpacked word-wise, branch-free.
__device__ __forceinline__ void tm_scales(const uint4 &m, int j, int c, int &sc_lo, int &sc_hi, int &mn_c) {
    const uint32_t s0 = m.y, s1 = m.z, s2 = m.w;
    const uint32_t sc03 = s0 & 0x3f3f3f3fu;
    const uint32_t sc47 = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);
    const uint32_t mn03 = s1 & 0x3f3f3f3fu;
    const uint32_t mn47 = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);
    sc_lo = (int)__byte_perm(sc03, sc47, 0x4440 | (2 * j)) & 0xff;
    sc_hi = (int)__byte_perm(sc03, sc47, 0x4440 | (2 * j + 1)) & 0xff;
    mn_c = (int)__byte_perm(mn03, mn47, 0x4440 | c) & 0xff;
}

// Sum over the 8 lanes of this lane's group (lanes 8q..8q+7, `mask`); exact for ints.
__device__ __forceinline__ int grp_sum(int v, unsigned mask) {
    v += __shfl_xor_sync(mask, v, 1);
    v += __shfl_xor_sync(mask, v, 2);
    v += __shfl_xor_sync(mask, v, 4);
    return v;
}

// One super-block k of one row (in shared memory) against NB activations:
// the 8 lanes of the group each cover 32 weights, their integer partial sums
// are added across the group (exact), and lane c == 0 writes the block's
// canonical term pair (a, c) of every sequence to tw[s] (RowOrder):
//   Q4_K/Q5_K: a = d_x, c = fma(d, float(sumi_s), -(dmin * sumi_m))
//              (vec_dot_q4_K_q8_K / q5, main.c:347-593, integer sums exact);
//   Q6_K:      a = float(sum_i v_i X_i), c = d * 2^(E-22)
//              (v = sc*(q-32) of dequant_q6_k, main.c:213-237; X = q6x_block).
template <int TYPE, int NB>
__device__ __forceinline__ void tm_block(const uint8_t *row, int nb, int n, int k, const TmAct &A, int nbc,
                                         float2 *tw, int c, unsigned gmask) {
    if (TYPE == G4_Q6_K) {
        const int n6 = c >> 2, second = (c >> 1) & 1, par = c & 1, sidx = 2 * second + par;
        const uint4 ql4 = reinterpret_cast<const uint4 *>(row)[k * 8 + c];
        const uint4 qh4 = reinterpret_cast<const uint4 *>(row + (size_t)nb * 128)[k * 4 + 2 * n6 + par];
        const uint2 sc = reinterpret_cast<const uint2 *>(row + (size_t)nb * 192)[k * 2 + n6];
        const float d = f16_to_f32(reinterpret_cast<const uint16_t *>(row + (size_t)nb * 208)[k]);
        const int sl = (int)(int8_t)((sc.x >> (8 * sidx)) & 0xffu);
        const int sh = (int)(int8_t)((sc.y >> (8 * sidx)) & 0xffu);
        const uint32_t ql[4] = {ql4.x, ql4.y, ql4.z, ql4.w}, qh[4] = {qh4.x, qh4.y, qh4.z, qh4.w};
        uint32_t lo[4], hi[4];  // q - 32 as signed bytes
#pragma unroll
        for (int i = 0; i < 4; i++) {
            lo[i] = __vsub4((ql[i] & 0x0F0F0F0Fu) | (((qh[i] >> (2 * second)) & 0x03030303u) << 4), 0x20202020u);
            hi[i] = __vsub4(((ql[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> (4 + 2 * second)) & 0x03030303u) << 4), 0x20202020u);
        }
        const int e_lo = k * G4_QK + 128 * n6 + 32 * second + 16 * par;
#pragma unroll
        for (int s = 0; s < NB; s++) {
            if (s >= nbc) break;
            int D[3];
#pragma unroll
            for (int j = 0; j < 3; j++) {
                const int8_t *pj = A.pc + ((size_t)s * 3 + j) * n;
                const uint4 xl = *reinterpret_cast<const uint4 *>(pj + e_lo);
                const uint4 xh = *reinterpret_cast<const uint4 *>(pj + e_lo + 64);
                int dl = __dp4a((int)lo[0], (int)xl.x, 0);
                dl = __dp4a((int)lo[1], (int)xl.y, dl);
                dl = __dp4a((int)lo[2], (int)xl.z, dl);
                dl = __dp4a((int)lo[3], (int)xl.w, dl);
                int dh = __dp4a((int)hi[0], (int)xh.x, 0);
                dh = __dp4a((int)hi[1], (int)xh.y, dh);
                dh = __dp4a((int)hi[2], (int)xh.z, dh);
                dh = __dp4a((int)hi[3], (int)xh.w, dh);
                D[j] = grp_sum(sl * dl + sh * dh, gmask);
            }
            if (c == 0) tw[s] = make_float2(q6x_dot(D[0], D[1], D[2]), __fmul_rn(d, A.ys[s * nb + k]));
        }
        return;
    }
    const int j = c >> 1, h = c & 1;
    const uint8_t *blk = row + (size_t)k * (TYPE == G4_Q4_K ? 144 : 176);
    const uint4 meta = *reinterpret_cast<const uint4 *>(blk);
    const uint4 qv = *reinterpret_cast<const uint4 *>(blk + (TYPE == G4_Q4_K ? 16 : 48) + 16 * c);
    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        lo[i] = qw[i] & 0x0F0F0F0Fu;
        hi[i] = (qw[i] >> 4) & 0x0F0F0F0Fu;
    }
    if (TYPE == G4_Q5_K) {  // 5th bit: bit 2j (low nibbles) / 2j+1 (high) of qh
        const uint4 hv = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * h);
        const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            lo[i] |= ((hw[i] >> (2 * j)) & 0x01010101u) << 4;
            hi[i] |= ((hw[i] >> (2 * j + 1)) & 0x01010101u) << 4;
        }
    }
    int sc_lo, sc_hi, mn_c;
    tm_scales(meta, j, c, sc_lo, sc_hi, mn_c);
    const float dw = f16_to_f32((uint16_t)(meta.x & 0xffffu));
    const float dmw = f16_to_f32((uint16_t)(meta.x >> 16));
#pragma unroll
    for (int s = 0; s < NB; s++) {
        if (s >= nbc) break;
        const int8_t *q8 = A.qs + (size_t)s * n + k * G4_QK + 64 * j + 16 * h;
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
        const int S = grp_sum(sc_lo * dl + sc_hi * dh, gmask);
        const int M = grp_sum(mn_c * A.bs2[(s * (n / G4_QK) + k) * 8 + c], gmask);
        if (c == 0)
            tw[s] = make_float2(A.dx[s * (n / G4_QK) + k],
                                __fmaf_rn(dw, __int2float_rn(S), __fmul_rn(-dmw, __int2float_rn(M))));
    }
}

// The canonical fold of one row's block terms (RowOrder): terms of block b of
// sequence s at t[b * NB + s].
// Segment starts are tracked with counters (the row's unit index modulo the stream-K share, and
// the block index modulo the K slice) instead of a division per block.
template <int NB>
__device__ __forceinline__ float tm_fold(const float2 *t, int nb, int s, const RowOrder &o, int row) {
    float v = 0.0f, P = 0.0f;
    int us = o.share > 0 ? (int)(((long long)(o.tile0 + row / 128) * nb) % o.share) : 0, ks = 0;
    for (int b = 0; b < nb; b++) {
        if (b > 0 && ((o.share > 0 && us == 0) || (o.kslice > 0 && ks == 0))) { v = __fadd_rn(v, P); P = 0.0f; }
        const float2 ab = t[b * NB + s];
        P = __fmaf_rn(ab.x, ab.y, P);
        if (o.share > 0 && ++us == o.share) us = 0;
        if (o.kslice > 0 && ++ks == o.kslice) ks = 0;
    }
    return __fadd_rn(v, P);
}

// Stage (or compute, with the fused prologue) the activation of sequences
// [s0, s0+nbc) into shared memory.  Ends with a CTA barrier.
template <int TYPE, int NB>
__device__ __forceinline__ void tm_stage(const GemvJobs &jobs, const GemvJob &J, TmAct &A, float *pro_x, int s0,
                                         int nbc, bool writer, float *pred) {
    const int n = J.n, nb = n / G4_QK, tid = threadIdx.x, lane = tid & 31, nt = blockDim.x;
    const int warp = tid >> 5, nw = nt >> 5;
    if (jobs.has_pro) {
        Prologue P = jobs.pro;
        P.x_in += (size_t)s0 * P.dim;
        if (P.delta) P.delta += (size_t)s0 * P.dim;
        if (P.x_out) P.x_out += (size_t)s0 * P.dim;
        if (P.xn_out) P.xn_out += (size_t)s0 * P.dim;
        if (NB == 1 && prologue_reg_ok(P)) prologue_run_reg<10>(P, nbc, pro_x, writer, pred);
        else prologue_run(P, nbc, pro_x, nullptr, writer, pred);
    }
    if (TYPE == G4_Q6_K) {  // fp32 (prologue output or the global activation) -> fixed-point pieces
        for (int t = warp; t < nbc * nb; t += nw) {
            const int s = t / nb, k = t % nb;
            const float *src = jobs.has_pro ? pro_x + (size_t)s * n + (size_t)k * G4_QK
                                            : (const float *)J.act + (size_t)(s0 + s) * J.act_stride + (size_t)k * G4_QK;
            float v[8];
            const float4 a = *reinterpret_cast<const float4 *>(src + 8 * lane);
            const float4 b = *reinterpret_cast<const float4 *>(src + 8 * lane + 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            uint32_t pw[6];
            float ys;
            q6x_block(v, pw, ys);
#pragma unroll
            for (int jj = 0; jj < 3; jj++)
                *reinterpret_cast<uint2 *>(A.pc + ((size_t)s * 3 + jj) * n + (size_t)k * G4_QK + 8 * lane) =
                    make_uint2(pw[2 * jj], pw[2 * jj + 1]);
            if (lane == 0) A.ys[s * nb + k] = ys;
        }
    } else if (jobs.has_pro) {  // quantize into planes (quantize_row_q8_K, main.c:282-340)
        for (int t = warp; t < nbc * nb; t += nw) {
            const int s = t / nb, k = t % nb;
            uint32_t q[2];
            float d;
            int ls;
            warp_quant_block(pro_x + (size_t)s * n + (size_t)k * G4_QK, lane, q, d, ls);
            uint32_t *dst = reinterpret_cast<uint32_t *>(A.qs + (size_t)s * n + (size_t)k * G4_QK + 8 * lane);
            dst[0] = q[0];
            dst[1] = q[1];
            int sub = ls + __shfl_xor_sync(0xffffffffu, ls, 1);
            sub += __shfl_xor_sync(0xffffffffu, sub, 2);
            if ((lane & 3) == 0) A.bs2[(s * nb + k) * 8 + (lane >> 2)] = sub;
            if (lane == 0) A.dx[s * nb + k] = d;
        }
    } else {
        const uint8_t *src = (const uint8_t *)J.act + (size_t)s0 * nb * G4_Q8_BYTES;
        for (int i = tid; i < nbc * nb * 64; i += nt) {
            const int blk = i >> 6, w = i & 63;
            reinterpret_cast<uint32_t *>(A.qs)[blk * 64 + w] =
                *reinterpret_cast<const uint32_t *>(src + (size_t)blk * G4_Q8_BYTES + 4 + 4 * w);
        }
        for (int i = tid; i < nbc * nb * 8; i += nt) {
            const int blk = i >> 3, jj = i & 7;
            const int16_t *bs = reinterpret_cast<const int16_t *>(src + (size_t)blk * G4_Q8_BYTES + 260);
            A.bs2[i] = (int)bs[2 * jj] + (int)bs[2 * jj + 1];
            if (jj == 0) A.dx[blk] = *reinterpret_cast<const float *>(src + (size_t)blk * G4_Q8_BYTES);
        }
    }
    __syncthreads();
}

struct TmPlan {   // per launch, computed on the host
    int gpr;      // lane groups per row (1, 2, 4)
    int tr;       // rows per tile (<= 64 / gpr)
    int stages;   // ring depth
    int row_bytes;
    int stage_bytes;  // R * tr * row_bytes, 128-aligned
    int act_bytes;    // activation staging + prologue scratch + term buffers (precedes the ring)
    int pro_off;      // offset of the fp32 prologue scratch
    int term_off;     // offset of the per-warp term buffers
    int term_warp;    // bytes of one warp's term buffer: (4/gpr) rows x R x nb x NB float2
};

template <int TYPE, int NB, int R>
__global__ void __launch_bounds__(kTmThreads, 1) gemv_tma_kernel(GemvJobs jobs, int B, TmPlan plan) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kTmMaxStages], empty[kTmMaxStages];
    __shared__ unsigned long long best[NB];
    __shared__ float pred[8];
    __shared__ int abort_flag;
    const int bx = (int)blockIdx.x;
    const GemvJob J = (jobs.njobs > 2 && bx >= jobs.j[2].cta_begin) ? jobs.j[2]
                    : (jobs.njobs > 1 && bx >= jobs.j[1].cta_begin) ? jobs.j[1] : jobs.j[0];
    const int n = J.n, nb = n / G4_QK;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, c = lane & 7, q = lane >> 3;
    const int cta = bx - J.cta_begin, nctas = J.ctas;
    const int TR = plan.tr, GPR = plan.gpr, S = plan.stages;
    const int ntiles = (J.rows + TR - 1) / TR;
    const size_t rb = (size_t)plan.row_bytes;
    uint8_t *ring = smem + plan.act_bytes;
    const bool producer = warp == kTmConsumerWarps;
    pdl_trigger();

    TmAct A{};
    if (TYPE == G4_Q6_K) {
        A.pc = (int8_t *)smem;
        A.ys = (float *)(smem + (((size_t)NB * 3 * n + 15) & ~(size_t)15));
    } else {
        A.qs = (int8_t *)smem;
        A.dx = (float *)(smem + (size_t)NB * n);
        A.bs2 = (int *)(smem + (size_t)NB * n + (size_t)NB * nb * 4);
    }
    float *pro_x = (float *)(smem + plan.pro_off);

    for (int s0 = 0; s0 < B; s0 += NB) {
        const int nbc = min(NB, B - s0);
        if (tid == 0) {
            for (int st = 0; st < S; st++) {
                mbar_init(&full[st], 1);
                mbar_init(&empty[st], kTmConsumerWarps);
            }
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            abort_flag = 0;
        }
        if (tid < NB) best[tid] = 0ull;
        __syncthreads();
        // producer: first S tiles in flight before the activation is staged
        int issued = 0;
        auto issue = [&](int i) {
            const int tile = cta + i * nctas;
            const int st = i % S;
            const int rows_t = min(TR, J.rows - tile * TR);
            const uint32_t bytes = (uint32_t)(rows_t * rb);
            mbar_expect_tx(&full[st], bytes * R);
            uint8_t *dst = ring + (size_t)st * plan.stage_bytes;
            bulk_g2s(dst, (const uint8_t *)J.w + (size_t)tile * TR * rb, bytes, &full[st]);
            if (R == 2) bulk_g2s(dst + (size_t)TR * rb, (const uint8_t *)J.w2 + (size_t)tile * TR * rb, bytes, &full[st]);
        };
        const int my_tiles = cta < ntiles ? (ntiles - cta + nctas - 1) / nctas : 0;
        if (producer && lane == 0)
            for (; issued < my_tiles && issued < S; issued++) issue(issued);
        pdl_wait();  // activation / residual from the previous kernel; weights above do not depend on it
        tm_stage<TYPE, NB>(jobs, J, A, pro_x, s0, nbc, jobs.pro_writer && bx == 0, pred);

        if (producer) {
            if (lane == 0) {
                bool ok = true;
                for (; issued < my_tiles; issued++) {
                    const int st = issued % S;
                    // slot st was last used by tile issued-S: wait until all consumer warps released it
                    if (!mbar_wait_sleep(&empty[st], ((issued / S) - 1) & 1)) { ok = false; break; }
                    if (abort_flag) break;
                    issue(issued);
                }
                if (!ok) {
                    atomicExch(&abort_flag, 1);
                    if (jobs.err) atomicExch(jobs.err, G4_ERR_TIMEOUT);
                }
                // drain: every issued copy must land before the CTA can exit
                const int first = issued > S ? issued - S : 0;
                for (int i = first; i < issued; i++) (void)mbar_wait(&full[i % S], (i / S) & 1);
            }
        } else {
            unsigned long long mykey[NB];
#pragma unroll
            for (int s = 0; s < NB; s++) mykey[s] = 0ull;
            const int g = warp * 4 + q;               // consumer lane group
            const int rl = g / GPR, part = g % GPR;  // tile row, block run
            const int bpg = (nb + GPR - 1) / GPR;
            const int kb = min(part * bpg, nb), ke = min(kb + bpg, nb);
            const bool grp_on = rl < TR;             // long rows: fewer tile rows than groups
            const unsigned gmask = 0xffu << (lane & 24);
            // this row's term buffer: [R][nb][NB] float2, one per tile row of this warp
            float2 *terms = reinterpret_cast<float2 *>(smem + plan.term_off + (size_t)warp * plan.term_warp) +
                            (size_t)(q / GPR) * R * nb * NB;
            for (int i = 0; i < my_tiles; i++) {
                const int tile = cta + i * nctas, st = i % S;
                if (!mbar_wait_sleep(&full[st], (i / S) & 1)) {
                    atomicExch(&abort_flag, 1);
                    if (jobs.err) atomicExch(jobs.err, G4_ERR_TIMEOUT);
                    break;
                }
                const uint8_t *stage = ring + (size_t)st * plan.stage_bytes;
                const int row = tile * TR + rl;
                const bool valid = grp_on && row < J.rows;
                if (valid) {
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        const uint8_t *rowp = stage + (size_t)(r * TR + rl) * rb;
                        for (int k = kb; k < ke; k++)
                            tm_block<TYPE, NB>(rowp, nb, n, k, A, nbc, terms + ((size_t)r * nb + k) * NB, c, gmask);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the slot
                if (c == 0 && part == 0 && valid) {
#pragma unroll
                    for (int s = 0; s < NB; s++) {
                        if (s >= nbc) break;
                        float a = tm_fold<NB>(terms, nb, s, J.ord, row);
                        float *out = J.out ? J.out + (size_t)(s0 + s) * J.out_stride : nullptr;
                        if (J.epi == EPI_GELU_MUL) {
                            out[row] = gelu_f32(a) * tm_fold<NB>(terms + (size_t)nb * NB, nb, s, J.ord2, row);
                        } else if (J.epi == EPI_SOFTCAP_ARGMAX) {
                            if (J.cap > 0.0f) a = J.cap * tanhf(a * (1.0f / J.cap));
                            if (out) out[row] = a;
                            const unsigned long long kk = argmax_key(a, row);
                            mykey[s] = kk > mykey[s] ? kk : mykey[s];
                        } else if (J.epi == EPI_GELU_SCALE) {
                            out[row] = gelu_f32(a) * J.evec[(size_t)(s0 + s) * J.ld_evec + row];
                        } else {
                            out[row] = a;
                        }
                    }
                }
                __syncwarp();  // the fold has read the terms before the next tile rewrites them
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
            }
        }
        __syncthreads();
        if (J.epi == EPI_SOFTCAP_ARGMAX && tid < nbc && best[tid]) atomicMax(J.amax + s0 + tid, best[tid]);
        if (tid == 0)
            for (int st = 0; st < S; st++) {
                asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[st])) : "memory");
                asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(&empty[st])) : "memory");
            }
        __syncthreads();
        if (abort_flag) return;
    }
}

// ---------------------------------------------------------------- batch-1 row-owner GEMV (Q4_K / Q5_K)
//
// At batch 1 the GEMV is bounded by instruction issue and by the latency of
// its first weight bytes more than by HBM bandwidth, so this variant keeps
// the work per weight small: each warp owns tiles of 8 row units (a row of a
// matrix; for a gate/up pair 4 rows of each) and streams them through two
// shared-memory buffers of its own (8 bulk copies of KC super-blocks per row,
// one mbarrier per buffer, no CTA-wide synchronisation after the activation
// is staged).  4 lanes share a super-block (64 weights each: 16 dp4a, two
// shuffle levels per integer sum), and lane group g folds its row's block
// terms in registers in the canonical row order (RowOrder), so the result is
// bit-identical to gemv_tma_kernel and to the tensor-core GEMMs.  The first
// two chunks of every warp are requested before griddepcontrol.wait.
constexpr int kRoWarps = 16;
constexpr int kRoThreads = kRoWarps * 32;
constexpr int kRoBufs = 2;

struct RoPlan {
    int row_bytes;
    int kc;           // super-blocks per chunk
    int chunk_bytes;  // kc * block bytes (one row unit)
    int unit_stride;  // bytes between the row units of a buffer (chunk padded to 16 mod 32: no bank conflicts)
    int stage_bytes;  // 8 row units
    int act_bytes;    // activation staging (+ prologue scratch) before the warp buffers
    int pro_off;
    int tiles;        // tiles of all jobs
    int tile_begin[kMaxJobs + 1];
};

// Scales and mins of sub-blocks 2j and 2j+1 of a Q4_K/Q5_K block (get_scale_min_k4, main.c:162-170).
__device__ __forceinline__ void ro_scales(const uint4 &m, int j, int &sc0, int &sc1, int &mn0, int &mn1) {
    const uint32_t s0 = m.y, s1 = m.z, s2 = m.w;
    const uint32_t sc03 = s0 & 0x3f3f3f3fu;
    const uint32_t sc47 = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);
    const uint32_t mn03 = s1 & 0x3f3f3f3fu;
    const uint32_t mn47 = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);
    sc0 = (int)__byte_perm(sc03, sc47, 0x4440 | (2 * j)) & 0xff;
    sc1 = (int)__byte_perm(sc03, sc47, 0x4440 | (2 * j + 1)) & 0xff;
    mn0 = (int)__byte_perm(mn03, mn47, 0x4440 | (2 * j)) & 0xff;
    mn1 = (int)__byte_perm(mn03, mn47, 0x4440 | (2 * j + 1)) & 0xff;
}

// Term (a, c) of super-block b of one row (blk in shared memory) for this lane's 64 weights
// (32-byte chunk j = lane & 3 of the quants): the integer sums S and M of the whole block
// (exact, over the 4 lanes of the group), then a = d_x, c = fma(d, S, -dmin*M) as in tm_block.
template <int TYPE>
__device__ __forceinline__ float2 ro_block(const uint8_t *blk, int b, int j, const TmAct &A) {
    constexpr int QOFF = TYPE == G4_Q4_K ? 16 : 48;
    const uint4 meta = *reinterpret_cast<const uint4 *>(blk);
    const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + QOFF + 32 * j);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + QOFF + 32 * j + 16);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        lo[i] = w[i] & 0x0F0F0F0Fu;
        hi[i] = (w[i] >> 4) & 0x0F0F0F0Fu;
    }
    if (TYPE == G4_Q5_K) {  // 5th bit: bit 2j (low nibbles) / 2j+1 (high) of qh[l]
        const uint4 h0 = *reinterpret_cast<const uint4 *>(blk + 16);
        const uint4 h1 = *reinterpret_cast<const uint4 *>(blk + 32);
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            lo[i] |= ((hw[i] >> (2 * j)) & 0x01010101u) << 4;
            hi[i] |= ((hw[i] >> (2 * j + 1)) & 0x01010101u) << 4;
        }
    }
    const int8_t *q8 = A.qs + (size_t)b * G4_QK + 64 * j;
    const uint4 a0 = *reinterpret_cast<const uint4 *>(q8), a1 = *reinterpret_cast<const uint4 *>(q8 + 16);
    const uint4 a2 = *reinterpret_cast<const uint4 *>(q8 + 32), a3 = *reinterpret_cast<const uint4 *>(q8 + 48);
    int dl = __dp4a((int)lo[0], (int)a0.x, 0);
    dl = __dp4a((int)lo[1], (int)a0.y, dl);
    dl = __dp4a((int)lo[2], (int)a0.z, dl);
    dl = __dp4a((int)lo[3], (int)a0.w, dl);
    dl = __dp4a((int)lo[4], (int)a1.x, dl);
    dl = __dp4a((int)lo[5], (int)a1.y, dl);
    dl = __dp4a((int)lo[6], (int)a1.z, dl);
    dl = __dp4a((int)lo[7], (int)a1.w, dl);
    int dh = __dp4a((int)hi[0], (int)a2.x, 0);
    dh = __dp4a((int)hi[1], (int)a2.y, dh);
    dh = __dp4a((int)hi[2], (int)a2.z, dh);
    dh = __dp4a((int)hi[3], (int)a2.w, dh);
    dh = __dp4a((int)hi[4], (int)a3.x, dh);
    dh = __dp4a((int)hi[5], (int)a3.y, dh);
    dh = __dp4a((int)hi[6], (int)a3.z, dh);
    dh = __dp4a((int)hi[7], (int)a3.w, dh);
    int sc0, sc1, mn0, mn1;
    ro_scales(meta, j, sc0, sc1, mn0, mn1);
    const int *bs = A.bs2 + (size_t)b * 8 + 2 * j;  // 4-byte aligned only (nb may be odd)
    int S = sc0 * dl + sc1 * dh, M = mn0 * bs[0] + mn1 * bs[1];
    S += __shfl_xor_sync(0xffffffffu, S, 1);
    M += __shfl_xor_sync(0xffffffffu, M, 1);
    S += __shfl_xor_sync(0xffffffffu, S, 2);
    M += __shfl_xor_sync(0xffffffffu, M, 2);
    const float dw = f16_to_f32((uint16_t)(meta.x & 0xffffu));
    const float dmw = f16_to_f32((uint16_t)(meta.x >> 16));
    return make_float2(A.dx[b], __fmaf_rn(dw, __int2float_rn(S), __fmul_rn(-dmw, __int2float_rn(M))));
}

// The fields of job jb that a tile needs (selected without indexing the parameter array).
struct RoJob {
    const uint8_t *w, *w2;
    float *out;
    int rows;
    RowOrder ord, ord2;
};
__device__ __forceinline__ RoJob ro_job(const GemvJobs &jobs, int jb) {
    const GemvJob &J = jb == 0 ? jobs.j[0] : jb == 1 ? jobs.j[1] : jobs.j[2];
    return RoJob{(const uint8_t *)J.w, (const uint8_t *)J.w2, J.out, J.rows, J.ord, J.ord2};
}

template <int TYPE, int R>
__global__ void __launch_bounds__(kRoThreads, 1) gemv_rows_kernel(GemvJobs jobs, RoPlan plan) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kRoWarps][kRoBufs];
    __shared__ float pred[8];
    constexpr int BLK = TYPE == G4_Q4_K ? 144 : 176;
    constexpr int UPR = 8 / R;  // rows per tile
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, j = lane & 3;
    pdl_trigger();
    const int n = jobs.j[0].n, nb = n / G4_QK, KC = plan.kc, nck = (nb + KC - 1) / KC;
    TmAct A{};
    A.qs = (int8_t *)smem;
    A.dx = (float *)(smem + (size_t)n);
    A.bs2 = (int *)(smem + (size_t)n + (size_t)nb * 4);
    float *pro_x = (float *)(smem + plan.pro_off);
    uint8_t *stage = smem + plan.act_bytes + (size_t)warp * kRoBufs * plan.stage_bytes;
    const int nwarps = gridDim.x * kRoWarps, gw = warp * gridDim.x + (int)blockIdx.x;
    const int my_tiles = gw < plan.tiles ? (plan.tiles - gw + nwarps - 1) / nwarps : 0;
    const int nchunks = my_tiles * nck;
    auto job_of = [&](int T, int &lt) {
        int jb = 0;
        if (jobs.njobs > 1 && T >= plan.tile_begin[1]) jb = 1;
        if (jobs.njobs > 2 && T >= plan.tile_begin[2]) jb = 2;
        lt = T - (jb == 0 ? 0 : jb == 1 ? plan.tile_begin[1] : plan.tile_begin[2]);
        return jb;
    };
    auto issue = [&](int ci) {  // lane 0: the chunk's bulk copies, one per row unit
        const int T = gw + (ci / nck) * nwarps, kc = ci % nck, kb0 = kc * KC, kcnt = min(KC, nb - kb0);
        int lt;
        const RoJob Jt = ro_job(jobs, job_of(T, lt));
        const int r0 = lt * UPR, vr = min(UPR, Jt.rows - r0);  // valid rows of the tile
        uint64_t *bar = &full[warp][ci % kRoBufs];
        uint8_t *dst = stage + (ci % kRoBufs) * plan.stage_bytes;
        const uint32_t cb = (uint32_t)(kcnt * BLK);
        mbar_expect_tx(bar, cb * (uint32_t)(vr * R));
        const size_t off = (size_t)r0 * plan.row_bytes + (size_t)kb0 * BLK;
        for (int u = 0; u < vr; u++) {
            bulk_g2s(dst + (size_t)u * plan.unit_stride, Jt.w + off + (size_t)u * plan.row_bytes, cb, bar);
            if (R == 2) bulk_g2s(dst + (size_t)(u + 4) * plan.unit_stride, Jt.w2 + off + (size_t)u * plan.row_bytes, cb, bar);
        }
    };
    if (lane == 0) {
        for (int b = 0; b < kRoBufs; b++) mbar_init(&full[warp][b], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int ci = 0; ci < kRoBufs && ci < nchunks; ci++) issue(ci);
    }
    __syncwarp();
    pdl_wait();  // activation / residual from the previous kernel; the weights above do not depend on it
    tm_stage<TYPE, 1>(jobs, jobs.j[0], A, pro_x, 0, 1, jobs.pro_writer && blockIdx.x == 0, pred);

    float v = 0.0f, P = 0.0f;
    int us = 0, ks = 0, row = 0;
    RowOrder o{};
    RoJob Jt{};
    int ci = 0;
    for (; ci < nchunks; ci++) {
        const int kc = ci % nck, kb0 = kc * KC, kcnt = min(KC, nb - kb0);
        if (!mbar_wait_sleep(&full[warp][ci % kRoBufs], (ci / kRoBufs) & 1)) {
            if (jobs.err && lane == 0) atomicExch(jobs.err, G4_ERR_TIMEOUT);
            break;
        }
        if (kc == 0) {  // a new tile: this group's row and its canonical order
            int lt;
            Jt = ro_job(jobs, job_of(gw + (ci / nck) * nwarps, lt));
            row = lt * UPR + (R == 2 ? (g & 3) : g);
            o = (R == 2 && g >= 4) ? Jt.ord2 : Jt.ord;
            v = 0.0f;
            P = 0.0f;
            us = o.share > 0 ? (int)(((long long)(o.tile0 + row / 128) * nb) % o.share) : 0;
            ks = 0;
        }
        const uint8_t *rowp = stage + (ci % kRoBufs) * plan.stage_bytes + (size_t)g * plan.unit_stride;
#pragma unroll 2
        for (int kk = 0; kk < kcnt; kk++) {
            const int b = kb0 + kk;
            const float2 t = ro_block<TYPE>(rowp + (size_t)kk * BLK, b, j, A);
            if (b > 0 && ((o.share > 0 && us == 0) || (o.kslice > 0 && ks == 0))) { v = __fadd_rn(v, P); P = 0.0f; }
            P = __fmaf_rn(t.x, t.y, P);
            if (o.share > 0 && ++us == o.share) us = 0;
            if (o.kslice > 0 && ++ks == o.kslice) ks = 0;
        }
        if (kc == nck - 1) {
            const float fin = __fadd_rn(v, P);
            if (R == 2) {
                const float up = __shfl_xor_sync(0xffffffffu, fin, 16);  // group g + 4: the up row
                if (g < 4 && j == 0 && row < Jt.rows) Jt.out[row] = gelu_f32(fin) * up;
            } else if (j == 0 && row < Jt.rows) {
                Jt.out[row] = fin;
            }
        }
        __syncwarp();  // every lane is done with this buffer before it is refilled
        if (lane == 0 && ci + kRoBufs < nchunks) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(ci + kRoBufs);
        }
    }
    if (ci < nchunks && lane == 0)  // gave up: drain this warp's copies in flight (bounded) before the CTA exits
        for (int k = ci; k < nchunks && k < ci + kRoBufs; k++) (void)mbar_wait(&full[warp][k % kRoBufs], (k / kRoBufs) & 1);
}

static int g_tm_sms = 0;
static int g_ro_off = 0;  // 1: batch 1 takes gemv_tma_kernel as well (g4_set_gemv_rows)
static constexpr int kTmSmemBudget = 220 * 1024;

// Activation staging bytes of nbs sequences (Q4/Q5: Q8_K planes; Q6: fixed-point pieces), then the
// fp32 prologue scratch when the launch runs the fused prologue.
template <int TYPE>
static size_t tm_stage_bytes(int nbs, int n) {
    const int nb = n / G4_QK;
    if (TYPE == G4_Q6_K) return (((size_t)nbs * 3 * n + 15) & ~(size_t)15) + (size_t)nbs * nb * 4;
    return (size_t)nbs * n + (size_t)nbs * nb * 36;
}
template <int TYPE>
static size_t tm_act_bytes(int nbs, int n, bool pro, int gpr, int R) {
    const size_t a = (tm_stage_bytes<TYPE>(nbs, n) + 15) & ~(size_t)15;
    const size_t p = pro ? (size_t)nbs * n * 4 : 0;
    const size_t t = (size_t)kTmConsumerWarps * (4 / gpr) * R * (n / G4_QK) * nbs * sizeof(float2);
    return a + p + t;
}

template <int TYPE, int NB, int R>
static void tm_launch(GemvJobs &jobs, int ctas, size_t smem, int B, const TmPlan &plan, cudaStream_t st) {
    (void)launch_pdl(gemv_tma_kernel<TYPE, NB, R>, dim3(ctas), dim3(kTmThreads), smem, st, jobs, B, plan);
}

template <int TYPE, int NB>
static void tm_launch_r(GemvJobs &jobs, int ctas, size_t smem, int B, const TmPlan &plan, cudaStream_t st) {
    if (jobs.j[0].w2) tm_launch<TYPE, NB, 2>(jobs, ctas, smem, B, plan, st);
    else tm_launch<TYPE, NB, 1>(jobs, ctas, smem, B, plan, st);
}

template <int TYPE>
static int tm_dispatch(GemvJobs &jobs, int ctas, int B, cudaStream_t st, int tr_cap) {
    const GemvJob &J0 = jobs.j[0];
    const int n = J0.n, nb = n / G4_QK, R = J0.w2 ? 2 : 1;
    for (int i = 1; i < jobs.njobs; i++)
        if (jobs.j[i].n != n || (jobs.j[i].w2 != nullptr) != (R == 2)) {
            set_error(G4_ERR_ARG, "gemv: jobs of one launch must share n and the gate/up form");
            return G4_ERR_ARG;
        }
    TmPlan plan{};
    plan.gpr = nb <= 6 ? 1 : nb <= 12 ? 2 : 4;
    plan.row_bytes = (int)device_row_bytes(TYPE, n);
    const bool pro = jobs.has_pro != 0;
    int nbs = B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : 8;
    while (nbs > 1 && tm_act_bytes<TYPE>(nbs, n, pro, plan.gpr, R) > (size_t)kTmSmemBudget / 3) nbs /= 2;
    const size_t stage_a = (tm_stage_bytes<TYPE>(nbs, n) + 15) & ~(size_t)15;
    plan.pro_off = (int)stage_a;
    plan.term_off = (int)(stage_a + (pro ? (size_t)nbs * n * 4 : 0));
    plan.term_warp = (int)((size_t)(4 / plan.gpr) * R * nb * nbs * sizeof(float2));
    plan.act_bytes = (int)((tm_act_bytes<TYPE>(nbs, n, pro, plan.gpr, R) + 127) & ~(size_t)127);
    // rows per tile: one row per GPR groups, at most what lets >= 3 stages fit
    int tr = std::min(kTmGroups / plan.gpr, tr_cap);
    const int fit = (kTmSmemBudget - plan.act_bytes) / (3 * R * plan.row_bytes);
    if (tr > fit) tr = fit > 1 ? fit : 1;
    plan.tr = tr;
    plan.stage_bytes = (int)(((size_t)R * plan.tr * plan.row_bytes + 127) & ~(size_t)127);
    int stages = (kTmSmemBudget - plan.act_bytes) / plan.stage_bytes;
    if (stages > kTmMaxStages) stages = kTmMaxStages;
    if (stages < 2) {
        set_error(G4_ERR_ARG, "gemv: tile of n=%d does not fit in shared memory", n);
        return G4_ERR_ARG;
    }
    plan.stages = stages;
    const size_t smem = (size_t)plan.act_bytes + (size_t)stages * plan.stage_bytes;
    switch (nbs) {
    case 1: tm_launch_r<TYPE, 1>(jobs, ctas, smem, B, plan, st); break;
    case 2: tm_launch_r<TYPE, 2>(jobs, ctas, smem, B, plan, st); break;
    case 4: tm_launch_r<TYPE, 4>(jobs, ctas, smem, B, plan, st); break;
    default: tm_launch_r<TYPE, 8>(jobs, ctas, smem, B, plan, st); break;
    }
    return G4_OK;
}

// The batch-1 row-owner GEMV, when it applies: one sequence, Q4_K/Q5_K, plain or gate/up epilogues,
// one activation for all jobs.  Returns 1 if launched, 0 if not applicable, < 0 on error.
template <int TYPE>
static int ro_dispatch(GemvJobs &jobs, cudaStream_t st) {
    const GemvJob &J0 = jobs.j[0];
    const int n = J0.n, nb = n / G4_QK, R = J0.w2 ? 2 : 1;
    constexpr int BLK = TYPE == G4_Q4_K ? 144 : 176;
    for (int i = 0; i < jobs.njobs; i++) {
        const GemvJob &J = jobs.j[i];
        if (J.epi != EPI_STORE && J.epi != EPI_GELU_MUL) return 0;
        if ((J.epi == EPI_GELU_MUL) != (J.w2 != nullptr) || !J.out) return 0;
        if (!jobs.has_pro && J.act != J0.act) return 0;
    }
    RoPlan plan{};
    plan.row_bytes = nb * BLK;
    size_t act = ((tm_stage_bytes<TYPE>(1, n) + 15) & ~(size_t)15);
    plan.pro_off = (int)act;
    if (jobs.has_pro) act += (size_t)n * 4;
    plan.act_bytes = (int)((act + 127) & ~(size_t)127);
    const long room = (long)kTmSmemBudget - plan.act_bytes;
    int kc = (int)(room / ((long)kRoWarps * kRoBufs * 8 * BLK));
    if (kc > nb) kc = nb;
    if (kc < 1) return 0;
    plan.kc = kc;
    plan.chunk_bytes = kc * BLK;
    plan.unit_stride = plan.chunk_bytes % 32 ? plan.chunk_bytes : plan.chunk_bytes + 16;
    plan.stage_bytes = 8 * plan.unit_stride;
    if ((size_t)plan.act_bytes + (size_t)kRoWarps * kRoBufs * plan.stage_bytes > (size_t)kTmSmemBudget) {
        kc = (int)(room / ((long)kRoWarps * kRoBufs * 8 * (BLK + 16)));
        if (kc < 1) return 0;
        plan.kc = kc;
        plan.chunk_bytes = kc * BLK;
        plan.unit_stride = plan.chunk_bytes % 32 ? plan.chunk_bytes : plan.chunk_bytes + 16;
        plan.stage_bytes = 8 * plan.unit_stride;
    }
    const int upr = 8 / R;
    int tiles = 0;
    for (int i = 0; i < jobs.njobs; i++) {
        plan.tile_begin[i] = tiles;
        tiles += (jobs.j[i].rows + upr - 1) / upr;
    }
    plan.tile_begin[jobs.njobs] = tiles;
    plan.tiles = tiles;
    const int ctas = tiles < g_tm_sms ? tiles : g_tm_sms;
    const size_t smem = (size_t)plan.act_bytes + (size_t)kRoWarps * kRoBufs * plan.stage_bytes;
    cudaError_t e = R == 2 ? launch_pdl(gemv_rows_kernel<TYPE, 2>, dim3(ctas), dim3(kRoThreads), smem, st, jobs, plan)
                           : launch_pdl(gemv_rows_kernel<TYPE, 1>, dim3(ctas), dim3(kRoThreads), smem, st, jobs, plan);
    if (e != cudaSuccess) {
        set_error(G4_ERR_CUDA, "gemv_rows launch: %s", cudaGetErrorString(e));
        return -1;
    }
    return 1;
}

int launch_gemv_kquant(GemvJobs &jobs, int B, cudaStream_t st) {
    if (g_tm_sms == 0) {
        int dev = 0;
        G4_CUDA(cudaGetDevice(&dev));
        G4_CUDA(cudaDeviceGetAttribute(&g_tm_sms, cudaDevAttrMultiProcessorCount, dev));
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
    int ctas = 0, tr_cap = kTmGroups;
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
        if (((uintptr_t)J.w & 15) || ((uintptr_t)J.w2 & 15)) {  // bulk copies need 16-byte aligned sources
            set_error(G4_ERR_ARG, "gemv: weight pointer not 16-byte aligned");
            return G4_ERR_ARG;
        }
        if (!J.explicit_order) {  // w alone in its own tensor-core launch
            if (type == G4_Q4_K) J.ord = q4_row_order(J.rows, 0, J.n, g_tm_sms, 0);
            else if (type == G4_Q5_K) J.ord = q5_row_order(J.rows, J.n, g_tm_sms);
            else J.ord = q6_row_order(J.rows, J.n, g_tm_sms, J.epi == EPI_SOFTCAP_ARGMAX);
            J.ord2 = J.ord;
            if (J.w2 && type == G4_Q4_K) {  // a gate/up pair shares one launch
                J.ord = q4_row_order(J.rows, J.rows, J.n, g_tm_sms, 0);
                J.ord2 = q4_row_order(J.rows, J.rows, J.n, g_tm_sms, 1);
            }
        }
        // persistent CTAs (1 per SM) shared out in proportion to the job's bytes
        const int nbj = J.n / G4_QK;
        const int gpr = nbj <= 6 ? 1 : nbj <= 12 ? 2 : 4;
        // rows per tile: a single small matrix gets smaller tiles, so that about half of the SMs
        // (or more) stream it instead of a few (fewer lane groups per tile, more tiles in flight)
        int trj = kTmGroups / gpr;
        if (jobs.njobs == 1)
            while (trj > 1 && (J.rows + trj - 1) / trj < g_tm_sms / 2) trj /= 2;
        tr_cap = std::min(tr_cap, trj);
        const long tiles = (J.rows + trj - 1) / trj;
        long cj = ((long)g_tm_sms * J.rows * nbj + total_work - 1) / total_work;
        if (cj > tiles) cj = tiles;
        if (cj < 1) cj = 1;
        J.ctas = (int)cj;
        J.cta_begin = ctas;
        ctas += J.ctas;
    }
    if (B == 1 && !g_ro_off && (type == G4_Q4_K || type == G4_Q5_K)) {
        const int r = type == G4_Q4_K ? ro_dispatch<G4_Q4_K>(jobs, st) : ro_dispatch<G4_Q5_K>(jobs, st);
        if (r < 0) return G4_ERR_CUDA;
        if (r > 0) {
            G4_LAUNCHED();
            return G4_OK;
        }
    }
    int rc;
    switch (type) {
    case G4_Q4_K: rc = tm_dispatch<G4_Q4_K>(jobs, ctas, B, st, tr_cap); break;
    case G4_Q5_K: rc = tm_dispatch<G4_Q5_K>(jobs, ctas, B, st, tr_cap); break;
    default: rc = tm_dispatch<G4_Q6_K>(jobs, ctas, B, st, tr_cap); break;
    }
    if (rc) return rc;
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

template <int TYPE, int R>
static int tm_prime_r() {
    G4_CUDA(cudaFuncSetAttribute(gemv_tma_kernel<TYPE, 1, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTmSmemBudget));
    G4_CUDA(cudaFuncSetAttribute(gemv_tma_kernel<TYPE, 2, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTmSmemBudget));
    G4_CUDA(cudaFuncSetAttribute(gemv_tma_kernel<TYPE, 4, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTmSmemBudget));
    G4_CUDA(cudaFuncSetAttribute(gemv_tma_kernel<TYPE, 8, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTmSmemBudget));
    return G4_OK;
}
template <int TYPE>
static int tm_prime() {
    int rc = tm_prime_r<TYPE, 1>();
    return rc ? rc : tm_prime_r<TYPE, 2>();
}

int set_gemv_rows(int on) {
    const int prev = g_ro_off ? 0 : 1;
    g_ro_off = on ? 0 : 1;
    return prev;
}

int prime_gemv_ks_attrs() {
    G4_CUDA(cudaFuncSetAttribute(gemv_rows_kernel<G4_Q4_K, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTmSmemBudget));
    G4_CUDA(cudaFuncSetAttribute(gemv_rows_kernel<G4_Q4_K, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTmSmemBudget));
    G4_CUDA(cudaFuncSetAttribute(gemv_rows_kernel<G4_Q5_K, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTmSmemBudget));
    G4_CUDA(cudaFuncSetAttribute(gemv_rows_kernel<G4_Q5_K, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTmSmemBudget));
    int rc = tm_prime<G4_Q4_K>();
    rc |= tm_prime<G4_Q5_K>();
    rc |= tm_prime<G4_Q6_K>();
    return rc ? G4_ERR_CUDA : G4_OK;
}

}  // namespace g4
