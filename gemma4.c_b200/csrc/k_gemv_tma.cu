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
                    if (!mbar_wait(&empty[st], ((issued / S) - 1) & 1)) { ok = false; break; }
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
                if (!mbar_wait(&full[st], (i / S) & 1)) {
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

static int g_tm_sms = 0;
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
static int tm_dispatch(GemvJobs &jobs, int ctas, int B, cudaStream_t st) {
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
    int tr = kTmGroups / plan.gpr;
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
        const long tiles = (J.rows + kTmGroups / gpr - 1) / (kTmGroups / gpr);
        long cj = ((long)g_tm_sms * J.rows * nbj + total_work - 1) / total_work;
        if (cj > tiles) cj = tiles;
        if (cj < 1) cj = 1;
        J.ctas = (int)cj;
        J.cta_begin = ctas;
        ctas += J.ctas;
    }
    int rc;
    switch (type) {
    case G4_Q4_K: rc = tm_dispatch<G4_Q4_K>(jobs, ctas, B, st); break;
    case G4_Q5_K: rc = tm_dispatch<G4_Q5_K>(jobs, ctas, B, st); break;
    default: rc = tm_dispatch<G4_Q6_K>(jobs, ctas, B, st); break;
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

int prime_gemv_ks_attrs() {
    int rc = tm_prime<G4_Q4_K>();
    rc |= tm_prime<G4_Q5_K>();
    rc |= tm_prime<G4_Q6_K>();
    return rc ? G4_ERR_CUDA : G4_OK;
}

}  // namespace g4
