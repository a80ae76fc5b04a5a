// k_gemm_q6tc.cu — batched Q6_K GEMM on the tensor cores (tcgen05.mma
// kind::f16, accumulators and the A operand in tensor memory), for decode
// steps with 16..64 sequences per GPU: the FFN down projection, V, and the
// tied LM head (with the softcap + argmax epilogue).
//
// The reference computes Q6_K rows as an fp32 dequant-dot against the fp32
// activation (mm_quant_rows, gemma4-4b/cpu-blas/main.c:1539-1556; the weight
// of element k of block b is d * sc_j * (q_k - 32), dequant_q6_k, main.c:
// 213-237).  Here, per row r, sequence s and super-block b:
//   v_k = sc_j * (q_k - 32)             integer in [-4064, 4096]
//       = 64 * (h_k + l_k),  h_k = (v_k + 4096) / 64 - 64 in [-64, 64],
//                            l_k = ((v_k + 4096) mod 64) / 64
//   (both exact in fp16), and the activation of block b of sequence s is
//   scaled by a power of two 2^e (largest |x| in [2^13, 2^14)) and split
//   into two fp16 parts, x * 2^e = x1 + x2 (to 2^-22 relative).
//   out[s][r] += 64 * d * 2^-e * sum_k (h_k + l_k) * (x1_k + x2_k).
// The MMA B operand stacks x1 (rows 0..NP-1) and x2 (rows NP..2NP-1), so
// every MMA is N = 2*NP (128 at 64 sequences, full tensor rate) and the two
// halves of the accumulator are added in the epilogue.  All products are
// exact in fp32; the float sum differs from the reference's sequential
// fp32 dot only in order and rounding (checked at 1e-5 of the term scale).
//
// CTA layout (one per SM, persistent) as in the Q4_K kernel: warp 0 bulk
// tensor copies (TMA) of 128-row x 1-super-block weight tiles and bulk copies
// of the B operand; warp 1 owns TMEM, one lane issues the MMAs; warps 2..9
// expand the 6-bit quants into the A operand in TMEM (tcgen05.st), warp
// group e = half e of the block; warps 10..17 run the per-block epilogue
// for half of the sequences each.  Every wait is bounded (2 s).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include "g4_async.cuh"
#include "g4_internal.cuh"
#include "g4_kernels.cuh"
#include "g4_tc.cuh"

namespace g4 {

namespace {

constexpr int kQ6Threads = 576;
constexpr int kQ6RawStages = 3;

// The device row of a Q6_K matrix is stored as planes: ql (128 B per
// super-block), qh (64 B), scales (16 B), d (2 B).  A raw tile (128 rows x
// one super-block) is three tensor copies into [ql 16 KB | qh 8 KB | sc 2 KB];
// ql and qh land with the 128-byte / 64-byte swizzles so that 32 rows read
// the same 16-byte column without bank conflicts.
struct Q6Maps {
    CUtensorMap ql, qh, sc;
};
constexpr int kQ6QhOff = 16384, kQ6ScOff = 24576;

template <int NP>
struct Q6Smem {
    static constexpr int raw = 128 * 208;            // ql, qh, sc of one super-block for 128 rows
    static constexpr int bst = 1024 * NP;            // 256 x 2*NP fp16
    static constexpr int bstages = NP == 64 ? 2 : 3;
    static constexpr int b_off = kQ6RawStages * raw;
    static constexpr int total = b_off + bstages * bst + 1024;
};
// TMEM columns: two accumulators of N = 2*NP, then four quarters of A
// (64 weights: 32 columns of h, 32 of l).
template <int NP>
struct Q6Tmem {
    static constexpr uint32_t a = 4 * NP;
    static_assert(a + 256 <= 512, "TMEM columns");
};

struct Q6State {
    uint64_t raw_full[kQ6RawStages], raw_empty[kQ6RawStages], b_full[3], b_empty[3];
    uint64_t a_full[4], a_empty[4], acc_full[2], acc_empty[2], mma_done;
    uint32_t tmem_base;
    volatile int abort;
    float ys[8][2][32];  // per epilogue warp: 64*d-free activation scales 2^-e of its sequences, by parity
};

__device__ __forceinline__ bool q6_wait(Q6State &S, uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
        if (S.abort) return false;
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
}
__device__ __forceinline__ void q6_fail(Q6State &S, int *err) {
    S.abort = 1;
    if (err) atomicExch(err, G4_ERR_TIMEOUT);
}

// 4 quants (bytes of qb, values 0..63) of one sub-block with scale sc ->
// columns (h, l) for the byte pairs (0, 2) and (1, 3).
__device__ __forceinline__ void q6_expand4(uint32_t qb, int sc, uint32_t C, uint32_t &h0, uint32_t &h1, uint32_t &l0,
                                           uint32_t &l1) {
    // u = sc*(q-32) + 4096 in [32, 8192], two 16-bit lanes per word (exact: the sum of the lanes is
    // non-negative and below 2^32 even when sc*q borrows)
    const uint32_t u0 = (qb & 0x00FF00FFu) * (uint32_t)sc + C;
    const uint32_t u1 = ((qb >> 8) & 0x00FF00FFu) * (uint32_t)sc + C;
    // h = (1024 + u/64) - 1088; l = (1024 + u%64)/64 - 16   (fp16, exact)
    h0 = hadd2_u(((u0 >> 6) & 0x00FF00FFu) | 0x64006400u, 0xE440E440u);
    h1 = hadd2_u(((u1 >> 6) & 0x00FF00FFu) | 0x64006400u, 0xE440E440u);
    l0 = hfma2_u((u0 & 0x003F003Fu) | 0x64006400u, 0x24002400u, 0xCC00CC00u);
    l1 = hfma2_u((u1 & 0x003F003Fu) | 0x64006400u, 0x24002400u, 0xCC00CC00u);
}

template <int NP>
__global__ void __launch_bounds__(kQ6Threads, 1) gemm_q6tc_kernel(const __grid_constant__ Q6Maps maps, TcArgs a) {
    constexpr int RAW = Q6Smem<NP>::raw, BST = Q6Smem<NP>::bst, BS = Q6Smem<NP>::bstages, RS = kQ6RawStages;
    constexpr int SP = NP / 2;  // sequences per epilogue warp
    using TM = Q6Tmem<NP>;
    extern __shared__ uint8_t smem_dyn[];
    __shared__ Q6State S;
    uint8_t *smem = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
    uint8_t *raw = smem, *bst = smem + Q6Smem<NP>::b_off;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_trigger();
    if (tid == 0) {
        for (int i = 0; i < RS; i++) {
            mbar_init(&S.raw_full[i], 1);
            mbar_init(&S.raw_empty[i], 8);
        }
        for (int i = 0; i < BS; i++) {
            mbar_init(&S.b_full[i], 1);
            mbar_init(&S.b_empty[i], 1);
        }
        for (int i = 0; i < 4; i++) {
            mbar_init(&S.a_full[i], 4);
            mbar_init(&S.a_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&S.acc_full[i], 1);
            mbar_init(&S.acc_empty[i], 8);
        }
        mbar_init(&S.mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.abort = 0;
    }
    if (warp == 1) tc_alloc(&S.tmem_base, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = S.tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int i = 0, nb_issued = 0;
            bool ok = true, dep = false;
            for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
                const int rt = u / a.ksplit, b0 = (u % a.ksplit) * a.kslice, b1 = min(a.nb, b0 + a.kslice);
                for (int b = b0; b < b1; b++, i++) {
                    const int rs = i % RS;
                    if (!q6_wait(S, &S.raw_empty[rs], ((i / RS) & 1) ^ 1)) { ok = false; break; }
                    mbar_expect_tx(&S.raw_full[rs], RAW);
                    tma_load_2d(raw + rs * RAW, &maps.ql, b * 128, rt * 128, &S.raw_full[rs]);
                    tma_load_2d(raw + rs * RAW + kQ6QhOff, &maps.qh, a.nb * 128 + b * 64, rt * 128, &S.raw_full[rs]);
                    tma_load_2d(raw + rs * RAW + kQ6ScOff, &maps.sc, a.nb * 192 + b * 16, rt * 128, &S.raw_full[rs]);
                    if (!dep) { pdl_wait(); dep = true; }
                    const int bs = i % BS;
                    if (!q6_wait(S, &S.b_empty[bs], ((i / BS) & 1) ^ 1)) { ok = false; i++; break; }
                    mbar_expect_tx(&S.b_full[bs], BST);
                    bulk_g2s(bst + bs * BST, a.bq + (size_t)b * BST, BST, &S.b_full[bs]);
                    nb_issued = i + 1;
                }
            }
            if (!dep) pdl_wait();
            if (!ok) {
                q6_fail(S, a.err);
                for (int k = max(0, i - RS); k < i; k++) {
                    const unsigned long long t0 = global_ns();
                    while (!mbar_try_wait(&S.raw_full[k % RS], (k / RS) & 1) && global_ns() - t0 < kWaitLimitNs) {}
                }
                for (int k = max(0, nb_issued - BS); k < nb_issued; k++) {
                    const unsigned long long t0 = global_ns();
                    while (!mbar_try_wait(&S.b_full[k % BS], (k / BS) & 1) && global_ns() - t0 < kWaitLimitNs) {}
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc(1, 0, 0, 2 * NP);  // f32 += f16 * f16, N = 2*NP
            int i = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
                const int b0 = (u % a.ksplit) * a.kslice, b1 = min(a.nb, b0 + a.kslice);
                for (int b = b0; b < b1 && ok; b++, i++) {
                    const int abuf = i & 1, bs = i % BS;
                    const uint32_t pa = i & 1;
                    {   // accumulator and B stage tested together; each A quarter just before its MMAs
                        const bool r0 = mbar_try_wait(&S.acc_empty[abuf], ((i >> 1) & 1) ^ 1);
                        const bool r1 = mbar_try_wait(&S.b_full[bs], (i / BS) & 1);
                        if (!(r0 && r1)) {
                            if (!q6_wait(S, &S.acc_empty[abuf], ((i >> 1) & 1) ^ 1) ||
                                !q6_wait(S, &S.b_full[bs], (i / BS) & 1)) { ok = false; break; }
                        }
                    }
                    const uint32_t bsa = smem_u32(bst + bs * BST);
                    const uint32_t d = tbase + abuf * 2 * NP;
                    for (int qi = 0; qi < 4; qi++) {
                        const int q = ((qi & 1) << 1) | (qi >> 1);  // 0, 2, 1, 3: the order the expand warps finish
                        if (!mbar_try_wait(&S.a_full[q], pa) && !q6_wait(S, &S.a_full[q], pa)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t acol = tbase + TM::a + 64 * q;
#pragma unroll
                        for (int ks = 0; ks < 4; ks++) {
                            const uint64_t bd = umma_desc(bsa + (8 * q + 2 * ks) * (2 * NP) * 16, 2 * NP * 16, 128);
                            tc_mma_f16_ts(d, acol + 8 * ks, bd, idesc, (qi | ks) != 0);  // h
                            tc_mma_f16_ts(d, acol + 32 + 8 * ks, bd, idesc, 1);           // l
                        }
                        tc_commit(&S.a_empty[q]);
                    }
                    if (!ok) break;
                    tc_commit(&S.b_empty[bs]);
                    tc_commit(&S.acc_full[abuf]);
                }
            }
            if (!ok) q6_fail(S, a.err);
            tc_commit(&S.mma_done);
            const unsigned long long t0 = global_ns();
            while (!mbar_try_wait(&S.mma_done, 0) && global_ns() - t0 < kWaitLimitNs) {}
        }
        __syncwarp();
    } else if (warp < 10) {
        // ------------------------------------------------------------ expand warps: half e of every block
        const int quad = warp & 3, e = (warp - 2) >> 2, r = 32 * quad + lane;
        const uint32_t tl = tbase + ((uint32_t)(32 * quad) << 16);
        const uint32_t raw_s = smem_u32(raw);
        int i = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
            const int b0 = (u % a.ksplit) * a.kslice, b1 = min(a.nb, b0 + a.kslice);
            for (int b = b0; b < b1; b++, i++) {
                const int rs = i % RS;
                if (!q6_wait(S, &S.raw_full[rs], (i / RS) & 1)) { ok = false; break; }
                const uint32_t st0 = raw_s + rs * RAW;
                // half e: ql[64e .. 64e+63], qh[32e .. 32e+31], sc[8e .. 8e+7]  (dequant_q6_k, main.c:213-237);
                // 16-byte chunk c of row r sits at chunk c ^ (r & 7) (ql, 128-B swizzle) / c ^ ((r >> 1) & 3) (qh, 64-B)
                uint32_t ql[16], qh[8];
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const uint4 v = lds128(st0 + r * 128 + (((4 * e + k) ^ (r & 7)) << 4));
                    ql[4 * k] = v.x; ql[4 * k + 1] = v.y; ql[4 * k + 2] = v.z; ql[4 * k + 3] = v.w;
                }
#pragma unroll
                for (int k = 0; k < 2; k++) {
                    const uint4 v = lds128(st0 + kQ6QhOff + r * 64 + (((2 * e + k) ^ ((r >> 1) & 3)) << 4));
                    qh[4 * k] = v.x; qh[4 * k + 1] = v.y; qh[4 * k + 2] = v.z; qh[4 * k + 3] = v.w;
                }
                const uint4 scv = lds128(st0 + kQ6ScOff + r * 16);
                const uint32_t sw0 = e ? scv.z : scv.x, sw1 = e ? scv.w : scv.y;  // sc[8e .. 8e+7]
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.raw_empty[rs]);
#pragma unroll
                for (int qq = 0; qq < 2; qq++) {
                    const int q = 2 * e + qq;
                    // qq = 0: weights l, l+32 (low nibbles, qh bits 0-1 / 2-3), scales sc[0..3] of the half;
                    // qq = 1: weights l+64, l+96 (high nibbles, qh bits 4-5 / 6-7), scales sc[4..7]
                    const uint32_t swq = qq ? sw1 : sw0;
                    int scs[4];
                    uint32_t cs[4];
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        scs[t] = (int)(int8_t)(swq >> (8 * t));
                        cs[t] = (uint32_t)(4096 - 32 * scs[t]) * 0x00010001u;
                    }
                    if (!q6_wait(S, &S.a_empty[q], (i & 1) ^ 1)) { ok = false; break; }
#pragma unroll
                    for (int set = 0; set < 2; set++) {  // set 0: weights l (scales t=0,1); set 1: l+32 (t=2,3)
#pragma unroll
                        for (int hf = 0; hf < 2; hf++) {  // 16 weights of scale t = 2*set + hf: 8 columns of h, of l
                            const int t = 2 * set + hf;
                            uint32_t ch[8], cl[8];
#pragma unroll
                            for (int ww = 0; ww < 4; ww++) {
                                const int w = 4 * hf + ww;
                                const uint32_t lw = ql[8 * set + w], hw = qh[w];
                                uint32_t qb;
                                if (qq == 0) qb = (lw & 0x0F0F0F0Fu) | ((set ? (hw << 2) : (hw << 4)) & 0x30303030u);
                                else qb = ((lw >> 4) & 0x0F0F0F0Fu) | ((set ? (hw >> 2) : hw) & 0x30303030u);
                                q6_expand4(qb, scs[t], cs[t], ch[2 * ww], ch[2 * ww + 1], cl[2 * ww], cl[2 * ww + 1]);
                            }
                            tc_st8(tl + TM::a + 64 * q + 16 * set + 8 * hf, ch);
                            tc_st8(tl + TM::a + 64 * q + 32 + 16 * set + 8 * hf, cl);
                        }
                    }
                    tc_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.a_full[q]);
                }
                if (!ok) break;
            }
        }
        if (!ok) q6_fail(S, a.err);
    } else {
        // ------------------------------------------------------------ epilogue warps
        const int quad = warp & 3, p = (warp - 10) >> 2, pw = warp - 10, r = 32 * quad + lane;
        const uint32_t tl = tbase + ((uint32_t)(32 * quad) << 16);
        pdl_wait();
        unsigned long long acc[SP / 2];
#pragma unroll
        for (int s = 0; s < SP / 2; s++) acc[s] = 0ull;
        int i = 0;
        bool ok = true;
        // per block: d of row r (fp16 after the quant planes of the row) and the activation scale of
        // sequence p*SP + lane, loaded one block ahead and converted only when used, so the load
        // latency overlaps the current block
        auto fetch = [&](int u, int b, uint16_t &hd, float &yl) {
            const int row = (u / a.ksplit) * 128 + r;
            hd = 0;
            if (row < a.rows) hd = __ldg(reinterpret_cast<const uint16_t *>(a.w + (size_t)row * a.row_bytes + (size_t)a.nb * 208) + b);
            yl = lane < SP ? __ldg(a.yd + (size_t)b * NP + p * SP + lane) : 0.0f;
        };
        // final values of sequences p*SP + 2s, +1 for row `row`
        auto emit = [&](int row, int s, float v0, float v1) {
            const int seq = p * SP + 2 * s;
            if (a.epi == EPI_SOFTCAP_ARGMAX) {  // logits softcap (main.c:1780-1796), then argmax over rows
                if (a.cap > 0.0f) {
                    v0 = a.cap * tanhf(v0 / a.cap);
                    v1 = a.cap * tanhf(v1 / a.cap);
                }
                unsigned long long k0 = row < a.rows ? argmax_key(v0, row) : 0ull;
                unsigned long long k1 = row < a.rows ? argmax_key(v1, row) : 0ull;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long t0 = __shfl_xor_sync(0xffffffffu, k0, o);
                    const unsigned long long t1 = __shfl_xor_sync(0xffffffffu, k1, o);
                    k0 = t0 > k0 ? t0 : k0;
                    k1 = t1 > k1 ? t1 : k1;
                }
                if (lane == 0) {
                    if (seq < a.B) atomicMax(a.keys + seq, k0);
                    if (seq + 1 < a.B) atomicMax(a.keys + seq + 1, k1);
                }
                if (!a.out) return;
            }
            if (row < a.rows) {
                if (seq < a.B) a.out[(size_t)seq * a.ldo + row] = v0;
                if (seq + 1 < a.B) a.out[(size_t)(seq + 1) * a.ldo + row] = v1;
            }
        };
        auto finish = [&](int u) {  // final values, or this K slice's partial (summed by tc_merge_kernel)
            const int ks = u % a.ksplit, row = (u / a.ksplit) * 128 + r;
            if (a.ksplit == 1) {
#pragma unroll
                for (int s = 0; s < SP / 2; s++) {
                    const float2 f = f2_unpack(acc[s]);
                    emit(row, s, f.x, f.y);
                    acc[s] = 0ull;
                }
                return;
            }
            if (row < a.rows) {  // all NP slots of the partial exist: no per-sequence bound
                float *dst = a.part + ((size_t)ks * NP + p * SP) * a.rows + row;
                const size_t st = (size_t)a.rows;
#pragma unroll
                for (int s = 0; s < SP / 2; s++) {
                    const float2 f = f2_unpack(acc[s]);
                    dst[(size_t)(2 * s) * st] = f.x;
                    dst[(size_t)(2 * s + 1) * st] = f.y;
                }
            }
#pragma unroll
            for (int s = 0; s < SP / 2; s++) acc[s] = 0ull;
        };
        int u = blockIdx.x, b = u < a.units ? (u % a.ksplit) * a.kslice : 0;
        uint16_t nhd = 0;
        float nyl = 0.f;
        if (u < a.units) fetch(u, b, nhd, nyl);
        while (u < a.units && ok) {
            const int b1 = min(a.nb, (u % a.ksplit) * a.kslice + a.kslice);
            const uint16_t hd = nhd;
            if (lane < SP) S.ys[pw][i & 1][lane] = nyl;
            __syncwarp();
            int nu = u, nbk = b + 1;
            if (nbk >= b1) { nu = u + gridDim.x; nbk = nu < a.units ? (nu % a.ksplit) * a.kslice : 0; }
            if (nu < a.units) fetch(nu, nbk, nhd, nyl);
            if (!q6_wait(S, &S.acc_full[i & 1], (i >> 1) & 1)) { ok = false; break; }
            const float dw = 64.0f * f16_to_f32(hd);
            tc_fence_after();
            const float *yv = S.ys[pw][i & 1];
            const unsigned long long dw2 = f2_pack(dw, dw);
#pragma unroll
            for (int c = 0; c < SP / 8; c++) {
                uint32_t v1[8], v2[8];
                tc_ld8(tl + (i & 1) * 2 * NP + p * SP + 8 * c, v1);       // products with x1
                tc_ld8(tl + (i & 1) * 2 * NP + NP + p * SP + 8 * c, v2);  // products with x2
                tc_wait_ld();
                if (c == SP / 8 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.acc_empty[i & 1]);
                }
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const unsigned long long t = f2_add(f2_pack_u(v1[2 * k], v1[2 * k + 1]), f2_pack_u(v2[2 * k], v2[2 * k + 1]));
                    const float2 y = *reinterpret_cast<const float2 *>(yv + 8 * c + 2 * k);
                    acc[4 * c + k] = f2_fma(f2_mul(dw2, f2_pack(y.x, y.y)), t, acc[4 * c + k]);
                }
            }
            if (nu != u) finish(u);
            u = nu; b = nbk; i++;
        }
        if (!ok) q6_fail(S, a.err);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tc_dealloc(tbase, 512);
    }
}

// B operand of gemm_q6tc for super-block k: the activation of every sequence
// scaled by 2^e_s (largest |x| of the block in [2^13, 2^14)) and split into
// fp16 x1 + x2, as 2*NP rows (x1 of sequence s in row s, x2 in row NP+s) of
// K-major core matrices: byte (k'/8)*(2*NP*16) + row*16 + (k'%8)*2, with
// k' = weight index with positions 1 and 2 of every 4 swapped (the order the
// expand warps write A in).  ys[k][s] = 2^-e_s (0 for padding sequences).
// grid (nb, NP/8), 256 threads: warp w handles sequence 8*blockIdx.y + w.
__global__ void tc6_split_kernel(const float *__restrict__ x, int ldx, int B, int NP, uint8_t *__restrict__ bq,
                                 float *__restrict__ ys) {
    pdl_trigger();
    pdl_wait();
    const int k = blockIdx.x, lane = threadIdx.x & 31, s = blockIdx.y * 8 + (threadIdx.x >> 5);
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = 0.0f;
    if (s < B) {
        const float4 *p = reinterpret_cast<const float4 *>(x + (size_t)s * ldx + (size_t)k * G4_QK + 8 * lane);
        const float4 a0 = p[0], a1 = p[1];
        v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w; v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
    }
    tc6_store_block(bq, ys, k, NP, s, lane, v, s < B);
}

template <int NP>
void *q6tc_kernel_ptr() { return (void *)gemm_q6tc_kernel<NP>; }

PFN_cuTensorMapEncodeTiled_v12000 g_enc6 = nullptr;

int q6_map(CUtensorMap *m, const void *w, size_t row_bytes, int rows, uint32_t box_x, CUtensorMapSwizzle sw) {
    const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {box_x, 128u}, es[2] = {1u, 1u};
    const CUresult rc = g_enc6(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(w), dims, strides, box, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) { set_error(G4_ERR_CUDA, "cuTensorMapEncodeTiled (Q6_K planes) failed (%d)", (int)rc); return G4_ERR_CUDA; }
    return G4_OK;
}

}  // namespace

// Tensor maps of a Q6_K device matrix (plane layout) for gemm_q6tc.
int tc6_weight_maps(void *maps_out, const void *w, int n, int rows) {
    if (!g_enc6) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        G4_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn) { set_error(G4_ERR_CUDA, "cuTensorMapEncodeTiled not available"); return G4_ERR_CUDA; }
        g_enc6 = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }
    if (((uintptr_t)w & 15u) != 0) { set_error(G4_ERR_ARG, "q6 tc: weight pointer not 16-byte aligned"); return G4_ERR_ARG; }
    Q6Maps *M = (Q6Maps *)maps_out;
    const size_t rb = device_row_bytes(G4_Q6_K, n);
    if (const int rc = q6_map(&M->ql, w, rb, rows, 128u, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    if (const int rc = q6_map(&M->qh, w, rb, rows, 64u, CU_TENSOR_MAP_SWIZZLE_64B)) return rc;
    return q6_map(&M->sc, w, rb, rows, 16u, CU_TENSOR_MAP_SWIZZLE_NONE);
}
size_t tc6_maps_bytes() { return sizeof(Q6Maps); }

size_t tc6_operand_bytes(int n) { return (size_t)(n / G4_QK) * (1024 * 64 + 64 * 4); }
size_t tc6_ys_offset(int n) { return (size_t)(n / G4_QK) * 1024 * 64; }

int launch_tc6_split(const float *x, int ldx, int B, int n, int np, uint8_t *bq, float *ys, cudaStream_t st) {
    if (n % G4_QK || (ldx % 4) || ((uintptr_t)x & 15u)) { set_error(G4_ERR_ARG, "tc6 split: bad shape/alignment"); return G4_ERR_ARG; }
    G4_CUDA(launch_pdl(tc6_split_kernel, dim3(n / G4_QK, np / 8), dim3(256), 0, st, x, ldx, B, np, bq, ys));
    G4_LAUNCHED();
    return G4_OK;
}

int launch_gemm_q6tc(const void *maps, const void *w, int n, int rows, const uint8_t *bq, const float *ys, int B,
                     int np, float *out, int ldo, float *part, size_t part_bytes, int *err, int nsm,
                     int epi, float cap, unsigned long long *keys, cudaStream_t st) {
    if (B < 1 || B > np || (np != 16 && np != 32 && np != 64)) { set_error(G4_ERR_ARG, "q6 tc gemm: batch %d / %d", B, np); return G4_ERR_ARG; }
    if (epi != EPI_STORE && epi != EPI_SOFTCAP_ARGMAX) { set_error(G4_ERR_ARG, "q6 tc gemm: epilogue %d", epi); return G4_ERR_ARG; }
    if (epi == EPI_SOFTCAP_ARGMAX && !keys) { set_error(G4_ERR_ARG, "q6 tc gemm: argmax keys missing"); return G4_ERR_ARG; }
    const int nb = n / G4_QK;
    TcPlan p = tc_plan(rows, nb, nsm);
    if (epi == EPI_SOFTCAP_ARGMAX) {  // the argmax epilogue needs whole rows: no K split
        const int tiles = (rows + 127) / 128;
        p = TcPlan{1, nb, tiles, tiles < nsm ? tiles : nsm};
    }
    if (p.ksplit > 1 && (size_t)p.ksplit * np * rows * sizeof(float) > part_bytes) {
        set_error(G4_ERR_ARG, "q6 tc gemm: partial buffer too small");
        return G4_ERR_ARG;
    }
    TcArgs a{(const uint8_t *)w, device_row_bytes(G4_Q6_K, n), bq, ys, out, part, err, nb, rows, B, ldo,
             p.ksplit, p.kslice, p.units, epi, cap, keys};
#define G4_Q6TC_CASE(N)                                                                             \
    if (np == N) {                                                                                   \
        const size_t smem = Q6Smem<N>::total;                                                        \
        G4_CUDA(launch_pdl(gemm_q6tc_kernel<N>, dim3(p.grid), dim3(kQ6Threads), smem, st, *(const Q6Maps *)maps, a)); \
    }
    G4_Q6TC_CASE(16) else G4_Q6TC_CASE(32) else G4_Q6TC_CASE(64)
#undef G4_Q6TC_CASE
    G4_LAUNCHED();
    if (p.ksplit > 1) return launch_tc_merge(part, p.ksplit, np, rows, B, out, ldo, EPI_STORE, nullptr, 0, st);
    return G4_OK;
}

int prime_tc6_attrs() {
    G4_CUDA(cudaFuncSetAttribute(q6tc_kernel_ptr<16>(), cudaFuncAttributeMaxDynamicSharedMemorySize, Q6Smem<16>::total));
    G4_CUDA(cudaFuncSetAttribute(q6tc_kernel_ptr<32>(), cudaFuncAttributeMaxDynamicSharedMemorySize, Q6Smem<32>::total));
    G4_CUDA(cudaFuncSetAttribute(q6tc_kernel_ptr<64>(), cudaFuncAttributeMaxDynamicSharedMemorySize, Q6Smem<64>::total));
    return G4_OK;
}

}  // namespace g4
