// k_gemm_tc.cu — batched K-quant GEMM on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory) for decode steps that carry
// 16..64 sequences per GPU.  At batch 1..8 the SIMT GEMV streams the weights
// once per step; with tens of sequences the same weight bytes feed a real
// contraction, so the weights are expanded once per CTA into MMA operands and
// multiplied against every sequence at once.
//
// Q4_K / Q5_K x Q8_K (vec_dot_q4_K_q8_K / vec_dot_q5_K_q8_K,
// gemma4-4b/cpu-blas/main.c:347-593), per padded sequence s and row r:
//   out[s][r] = sum_blk yd[s,blk] * (d[r,blk] * S - dmin[r,blk] * M)
// with the integer super-block sums of the reference
//   S = sum_j sc_j * sum_{i in j} q_i * q8_i      M = sum_j mn_j * bsum_j
// (j = 8 sub-blocks of 32, bsum_j = sum of the 32 q8 of sub-block j).  Both
// are formed exactly by kind::i8 MMAs with int32 accumulation:
//   * sc_j = 8*sh_j + sl_j with sh, sl in [0,7], so A_h = sh_j*q and
//     A_l = sl_j*q fit in u8 (<= 7*31); S = 8*D_h + D_l.
//   * bsum_j = 64*bh_j + bl_j with bh in [-64,63], bl in [0,63]: a second B
//     operand with 2*NP rows (bh of every sequence, then bl) against A = mn_j
//     (K = 32, zero padded) gives M = 64*D_mh + D_ml.
// The float epilogue runs once per super-block on the four int32
// accumulators read back from TMEM (exact int -> float conversions), so the
// integer partial sums are those of the reference and the float sum differs
// only in summation order.
//
// That is the Q5_K kernel (gemm_tc_kernel).  Q4_K uses gemm_q4tc_kernel
// below: kind::f16 with exact fp16 integer operands, fewer MMAs per block.
//
// CTA (one per SM, persistent): warp 0 issues the bulk tensor copies (TMA) of
// 128-row x 1-super-block weight tiles and of the pre-laid-out B operand;
// warp 1 owns TMEM and one lane issues the MMAs; warps 2..9 expand the raw
// weight tile into the A operands (core-matrix layout, no swizzle) and run the
// epilogue of the previous super-block.  Work units are (128-row tile,
// K-slice); the slices of a tile leave fp32 partials that are summed in slice
// order: inside the GEMM by the CTA that completes the tile when the caller
// passes tickets (the engine), else by tc_merge_kernel / sk_merge_kernel
// (Q4_K: stream-K units).
//
// Every mbarrier wait is bounded (2 s): on expiry the kernel records
// G4_ERR_TIMEOUT in *err, the producer waits for its copies in flight, the
// MMA lane for its MMAs, TMEM is freed and the CTA returns.
#include <algorithm>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <mutex>

#include "g4_async.cuh"
#include "g4_internal.cuh"
#include "g4_kernels.cuh"
#include "g4_quant.cuh"
#include "g4_tc.cuh"

namespace g4 {

namespace {

constexpr int kTcThreads = 320;      // warp 0 producer, warp 1 MMA, warps 2..9 math
constexpr int kTcMathWarps = 8;
constexpr int kASlotBytes = 2 * 16384 + 4096;  // A_h, A_l (128 rows x 128 weights), A_bs (128 x 32)
constexpr int kASlots = 3;
constexpr int kBStages = 2;

template <int TYPE>
struct TcQ;
template <>
struct TcQ<G4_Q4_K> {
    static constexpr int blk = 144, qs_off = 16, raw_stages = 4;
};
template <>
struct TcQ<G4_Q5_K> {
    static constexpr int blk = 176, qs_off = 48, raw_stages = 3;
};

template <int TYPE, int NP>
struct TcSmem {
    static constexpr int raw = 128 * TcQ<TYPE>::blk;
    static constexpr int bst = 320 * NP;
    static constexpr int b_off = TcQ<TYPE>::raw_stages * raw;
    static constexpr int a_off = b_off + kBStages * bst;
    static constexpr int total = a_off + kASlots * kASlotBytes + 1024;  // + alignment slack
};

// exact int -> float for |v| < 2^22 (two full-rate ops)
__device__ __forceinline__ float i2f_small(int v) { return __int_as_float(v + 0x4B400000) - 12582912.0f; }

struct TcState {  // shared-memory control block
    uint64_t raw_full[4], raw_empty[4], b_full[kBStages], b_empty[kBStages];
    uint64_t a_full[kASlots], a_empty[kASlots], acc_full[2], acc_empty[2], mma_done;
    uint32_t tmem_base;
    volatile int abort;
};

__device__ __forceinline__ void tc_fail(TcState &S, int *err) {
    S.abort = 1;
    if (err) atomicExch(err, G4_ERR_TIMEOUT);
}
// bounded wait that also gives up once another role has aborted
__device__ __forceinline__ bool tc_wait(TcState &S, uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
        if (S.abort) return false;
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
}


template <int TYPE, int NP>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmw, TcArgs a) {
    constexpr int BLK = TcQ<TYPE>::blk, RS = TcQ<TYPE>::raw_stages, QOFF = TcQ<TYPE>::qs_off;
    constexpr int RAW = TcSmem<TYPE, NP>::raw, BST = TcSmem<TYPE, NP>::bst;
    constexpr int HALF = NP / 2, CH = HALF < 16 ? HALF : 16;
    extern __shared__ uint8_t smem_dyn[];
    __shared__ TcState S;
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
    uint8_t *raw = smem, *bst = smem + TcSmem<TYPE, NP>::b_off, *ast = smem + TcSmem<TYPE, NP>::a_off;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_trigger();
    if (tid == 0) {
        for (int i = 0; i < RS; i++) {
            mbar_init(&S.raw_full[i], 1);
            mbar_init(&S.raw_empty[i], kTcMathWarps);
        }
        for (int i = 0; i < kBStages; i++) {
            mbar_init(&S.b_full[i], 1);
            mbar_init(&S.b_empty[i], 1);
        }
        for (int i = 0; i < kASlots; i++) {
            mbar_init(&S.a_full[i], kTcMathWarps);
            mbar_init(&S.a_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&S.acc_full[i], 1);
            mbar_init(&S.acc_empty[i], kTcMathWarps);
        }
        mbar_init(&S.mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.abort = 0;
    }
    if (warp == 1) tc_alloc(&S.tmem_base, 8 * NP);
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
                    if (!tc_wait(S, &S.raw_empty[rs], ((i / RS) & 1) ^ 1)) { ok = false; break; }
                    mbar_expect_tx(&S.raw_full[rs], RAW);
                    tma_load_2d(raw + rs * RAW, &tmw, b * BLK, rt * 128, &S.raw_full[rs]);
                    if (!dep) { pdl_wait(); dep = true; }  // the B operand comes from the previous kernel
                    const int bs = i % kBStages;
                    if (!tc_wait(S, &S.b_empty[bs], ((i / kBStages) & 1) ^ 1)) { ok = false; i++; break; }
                    mbar_expect_tx(&S.b_full[bs], BST);
                    bulk_g2s(bst + bs * BST, a.bq + (size_t)b * BST, BST, &S.b_full[bs]);
                    nb_issued = i + 1;
                }
            }
            if (!dep) pdl_wait();
            if (!ok) {
                tc_fail(S, a.err);
                // wait (bounded) for the copies still in flight before the CTA can exit
                for (int k = max(0, i - RS); k < i; k++) {
                    const unsigned long long t0 = global_ns();
                    while (!mbar_try_wait(&S.raw_full[k % RS], (k / RS) & 1) && global_ns() - t0 < kWaitLimitNs) {}
                }
                for (int k = max(0, nb_issued - kBStages); k < nb_issued; k++) {
                    const unsigned long long t0 = global_ns();
                    while (!mbar_try_wait(&S.b_full[k % kBStages], (k / kBStages) & 1) && global_ns() - t0 < kWaitLimitNs) {}
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc(2, 0, 1, NP), idesc_bs = umma_idesc(2, 0, 1, 2 * NP);
            int i = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
                const int b0 = (u % a.ksplit) * a.kslice, b1 = min(a.nb, b0 + a.kslice);
                for (int b = b0; b < b1 && ok; b++, i++) {
                    const int abuf = i & 1, bs = i % kBStages;
                    if (!tc_wait(S, &S.acc_empty[abuf], ((i >> 1) & 1) ^ 1)) { ok = false; break; }
                    if (!tc_wait(S, &S.b_full[bs], (i / kBStages) & 1)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t bsa = smem_u32(bst + bs * BST);
                    const uint32_t dh = tbase + abuf * 4 * NP, dl = dh + NP, dbs = dh + 2 * NP;
                    for (int h = 0; h < 2; h++) {
                        const int ai = 2 * i + h, sl = ai % kASlots;
                        if (!tc_wait(S, &S.a_full[sl], (ai / kASlots) & 1)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t asa = smem_u32(ast + sl * kASlotBytes);
#pragma unroll
                        for (int ks = 0; ks < 4; ks++) {
                            const uint64_t bd = umma_desc(bsa + (8 * h + 2 * ks) * NP * 16, NP * 16, 128);
                            const uint32_t acc = (h | ks) != 0;
                            tc_mma_i8(dh, umma_desc(asa + 2 * ks * 2048, 2048, 128), bd, idesc, acc);
                            tc_mma_i8(dl, umma_desc(asa + 16384 + 2 * ks * 2048, 2048, 128), bd, idesc, acc);
                        }
                        if (h == 0)
                            tc_mma_i8(dbs, umma_desc(asa + 32768, 2048, 128), umma_desc(bsa + NP * 256, 2 * NP * 16, 128),
                                      idesc_bs, 0);
                        tc_commit(&S.a_empty[sl]);
                    }
                    if (!ok) break;
                    tc_commit(&S.b_empty[bs]);
                    tc_commit(&S.acc_full[abuf]);
                }
            }
            if (!ok) tc_fail(S, a.err);
            // every MMA issued has completed before TMEM is released
            tc_commit(&S.mma_done);
            const unsigned long long t0 = global_ns();
            while (!mbar_try_wait(&S.mma_done, 0) && global_ns() - t0 < kWaitLimitNs) {}
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ math warps
        const int mw = warp - 2, quad = warp & 3, cb = mw >> 2, r = 32 * quad + lane;
        const uint32_t tl = tbase + ((uint32_t)(32 * quad) << 16);
        pdl_wait();
        float acc[HALF];
#pragma unroll
        for (int s = 0; s < HALF; s++) acc[s] = 0.0f;
        float dw_c = 0.f, dm_c = 0.f;  // scales of the block being expanded
        int i = 0;
        bool ok = true;
        // epilogue of item ei (block eb of unit eu)
        auto epilogue = [&](int ei, int eb, float dw, float dm) -> bool {
            float yv[HALF];
            const float4 *yp = reinterpret_cast<const float4 *>(a.yd + (size_t)eb * NP + cb * HALF);
#pragma unroll
            for (int s = 0; s < HALF / 4; s++) {
                const float4 t = __ldg(yp + s);
                yv[4 * s] = t.x; yv[4 * s + 1] = t.y; yv[4 * s + 2] = t.z; yv[4 * s + 3] = t.w;
            }
            if (!tc_wait(S, &S.acc_full[ei & 1], (ei >> 1) & 1)) return false;
            tc_fence_after();
            const uint32_t t0 = tl + (ei & 1) * 4 * NP + cb * HALF;
#pragma unroll
            for (int c = 0; c < HALF / CH; c++) {
                uint32_t vh[CH], vl[CH], vmh[CH], vml[CH];
                if constexpr (CH == 16) {
                    tc_ld16(t0 + c * CH, vh); tc_ld16(t0 + NP + c * CH, vl);
                    tc_ld16(t0 + 2 * NP + c * CH, vmh); tc_ld16(t0 + 3 * NP + c * CH, vml);
                } else {
                    tc_ld8(t0 + c * CH, vh); tc_ld8(t0 + NP + c * CH, vl);
                    tc_ld8(t0 + 2 * NP + c * CH, vmh); tc_ld8(t0 + 3 * NP + c * CH, vml);
                }
                tc_wait_ld();
                if (c == HALF / CH - 1) {  // accumulator buffer free for the MMA two blocks ahead
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.acc_empty[ei & 1]);
                }
#pragma unroll
                for (int s = 0; s < CH; s++) {
                    float sf;
                    if (TYPE == G4_Q4_K) sf = fmaf(8.0f, i2f_small((int)vh[s]), i2f_small((int)vl[s]));
                    else sf = (float)(8 * (int)vh[s] + (int)vl[s]);
                    const float mf = i2f_small(64 * (int)vmh[s] + (int)vml[s]);
                    const float t = fmaf(dw, sf, -(dm * mf));
                    acc[c * CH + s] = fmaf(yv[c * CH + s], t, acc[c * CH + s]);
                }
            }
            return true;
        };
        // slices of one 128-row tile: store, or write this K slice's partial (summed by tc_merge_kernel)
        auto finish = [&](int u) {
            const int ks = u % a.ksplit, row = (u / a.ksplit) * 128 + r;
            float *dst = a.ksplit == 1 ? a.out : a.part + (size_t)ks * NP * a.rows;
            const size_t ld = a.ksplit == 1 ? (size_t)a.ldo : (size_t)a.rows;
            if (row < a.rows)
#pragma unroll
                for (int s = 0; s < HALF; s++) {
                    const int seq = cb * HALF + s;
                    if (seq < a.B) dst[(size_t)seq * ld + row] = acc[s];
                }
#pragma unroll
            for (int s = 0; s < HALF; s++) acc[s] = 0.0f;
        };
        int pu = -1, pb = 0, pi = -1;
        bool p_last = false;
        float pdw = 0.f, pdm = 0.f;
        for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
            const int b0 = (u % a.ksplit) * a.kslice, b1 = min(a.nb, b0 + a.kslice);
            for (int b = b0; b < b1; b++, i++) {
                // ---- expand block b of this tile into the A operands
                const int rs = i % RS;
                if (!tc_wait(S, &S.raw_full[rs], (i / RS) & 1)) { ok = false; break; }
                const uint8_t *rw = raw + rs * RAW + r * BLK;
                const uint4 meta = *reinterpret_cast<const uint4 *>(rw);
                dw_c = f16_to_f32((uint16_t)(meta.x & 0xffffu));
                dm_c = f16_to_f32((uint16_t)(meta.x >> 16));
                const uint32_t sc03 = meta.y & 0x3f3f3f3fu;
                const uint32_t sc47 = (meta.w & 0x0f0f0f0fu) | ((meta.y >> 2) & 0x30303030u);
                const uint32_t mn03 = meta.z & 0x3f3f3f3fu;
                const uint32_t mn47 = ((meta.w >> 4) & 0x0f0f0f0fu) | ((meta.z >> 2) & 0x30303030u);
                uint32_t hw[8];
                if (TYPE == G4_Q5_K) {
                    const uint4 h0 = *reinterpret_cast<const uint4 *>(rw + 16);
                    const uint4 h1 = *reinterpret_cast<const uint4 *>(rw + 32);
                    hw[0] = h0.x; hw[1] = h0.y; hw[2] = h0.z; hw[3] = h0.w;
                    hw[4] = h1.x; hw[5] = h1.y; hw[6] = h1.z; hw[7] = h1.w;
                }
                for (int h = 0; h < 2; h++) {
                    const int j = 2 * h + cb;  // 64-weight group: sub-blocks 2j (low nibbles), 2j+1 (high)
                    const uint4 q0 = *reinterpret_cast<const uint4 *>(rw + QOFF + 32 * j);
                    const uint4 q1 = *reinterpret_cast<const uint4 *>(rw + QOFF + 32 * j + 16);
                    const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                    const uint32_t sc_lo = __byte_perm(sc03, sc47, 0x4440 | (2 * j)) & 0xffu;
                    const uint32_t sc_hi = __byte_perm(sc03, sc47, 0x4440 | (2 * j + 1)) & 0xffu;
                    uint32_t lo[8], hi[8];
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        lo[k] = qw[k] & 0x0F0F0F0Fu;
                        hi[k] = (qw[k] >> 4) & 0x0F0F0F0Fu;
                        if (TYPE == G4_Q5_K) {
                            lo[k] |= ((hw[k] >> (2 * j)) & 0x01010101u) << 4;
                            hi[k] |= ((hw[k] >> (2 * j + 1)) & 0x01010101u) << 4;
                        }
                    }
                    const int ai = 2 * i + h, sl = ai % kASlots;
                    if (!tc_wait(S, &S.a_empty[sl], ((ai / kASlots) & 1) ^ 1)) { ok = false; break; }
                    uint8_t *As = ast + sl * kASlotBytes + r * 16;
                    // local sub-blocks 2cb (low) and 2cb+1 (high): 16-weight chunks 4cb .. 4cb+3
                    const uint32_t shl = sc_lo >> 3, sll = sc_lo & 7u, shh = sc_hi >> 3, slh = sc_hi & 7u;
#pragma unroll
                    for (int c = 0; c < 2; c++) {
                        *reinterpret_cast<uint4 *>(As + (4 * cb + c) * 2048) =
                            make_uint4(lo[4 * c] * shl, lo[4 * c + 1] * shl, lo[4 * c + 2] * shl, lo[4 * c + 3] * shl);
                        *reinterpret_cast<uint4 *>(As + (4 * cb + 2 + c) * 2048) =
                            make_uint4(hi[4 * c] * shh, hi[4 * c + 1] * shh, hi[4 * c + 2] * shh, hi[4 * c + 3] * shh);
                        *reinterpret_cast<uint4 *>(As + 16384 + (4 * cb + c) * 2048) =
                            make_uint4(lo[4 * c] * sll, lo[4 * c + 1] * sll, lo[4 * c + 2] * sll, lo[4 * c + 3] * sll);
                        *reinterpret_cast<uint4 *>(As + 16384 + (4 * cb + 2 + c) * 2048) =
                            make_uint4(hi[4 * c] * slh, hi[4 * c + 1] * slh, hi[4 * c + 2] * slh, hi[4 * c + 3] * slh);
                    }
                    if (h == 0)  // mins against the bsum operand: K = 32, bytes 8..31 zero
                        *reinterpret_cast<uint4 *>(As + 32768 + cb * 2048) =
                            cb == 0 ? make_uint4(mn03, mn47, 0u, 0u) : make_uint4(0u, 0u, 0u, 0u);
                    fence_proxy_async_smem();  // generic-proxy stores -> tensor-core reads
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.a_full[sl]);
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.raw_empty[rs]);
                // ---- epilogue of the previous block
                if (pi >= 0) {
                    if (!epilogue(pi, pb, pdw, pdm)) { ok = false; break; }
                    if (p_last) finish(pu);
                }
                pu = u; pb = b; pi = i; p_last = b == b1 - 1; pdw = dw_c; pdm = dm_c;
            }
        }
        if (ok && pi >= 0) {
            if (epilogue(pi, pb, pdw, pdm)) finish(pu);
            else ok = false;
        }
        if (!ok) tc_fail(S, a.err);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tc_dealloc(tbase, 8 * NP);
    }
}

// ---------------------------------------------------------------- B operand

// The activation of NP sequences (padding sequences zero) as the MMA B
// operand of super-block k, written where the producer copies it from:
//   [0, 256*NP)        q8 quants, core-matrix layout: byte (k/16)*(NP*16) + s*16 + k%16
//   [256*NP, 320*NP)   bsum operand, rows t < NP: bh of sequence t, t >= NP: bl of t-NP;
//                      K = 32 (bytes 0..7 = sub-blocks 0..7, the rest zero)
//   yd[k][s]           the Q8_K block scale d
__device__ __forceinline__ void tc_store_q8(uint8_t *blk, float *ydk, int NP, int s, int lane, const uint32_t q[2],
                                            float d, int ls) {
    *reinterpret_cast<uint2 *>(blk + (lane >> 1) * (NP * 16) + s * 16 + 8 * (lane & 1)) = make_uint2(q[0], q[1]);
    int sub = ls + __shfl_xor_sync(0xffffffffu, ls, 1);
    sub += __shfl_xor_sync(0xffffffffu, sub, 2);                          // lanes 4j..4j+3: sum of sub-block j
    const int sj = __shfl_sync(0xffffffffu, sub, (lane & 7) * 4);         // lane l < 8: sub-block l
    uint8_t *bsb = blk + NP * 256;
    if (lane < 16) {
        bsb[s * 16 + lane] = lane < 8 ? (uint8_t)(int8_t)(sj >> 6) : 0;          // bh in [-64, 63]
        bsb[(NP + s) * 16 + lane] = lane < 8 ? (uint8_t)(sj & 63) : 0;            // bl in [0, 63]
    } else if (lane == 16) {
        *reinterpret_cast<uint4 *>(bsb + 2 * NP * 16 + s * 16) = make_uint4(0u, 0u, 0u, 0u);
    } else if (lane == 17) {
        *reinterpret_cast<uint4 *>(bsb + 2 * NP * 16 + (NP + s) * 16) = make_uint4(0u, 0u, 0u, 0u);
    }
    if (lane == 0) ydk[s] = d;
}

// grid (nb, NP/8), 256 threads: warp w quantizes sequence 8*blockIdx.y + w
// (quantize_row_q8_K, main.c:282-340) straight into the B operand layout.
__global__ void tc_quant_kernel(const float *__restrict__ x, int ldx, int B, int NP, uint8_t *__restrict__ bq,
                                float *__restrict__ yd) {
    pdl_trigger();
    pdl_wait();
    const int k = blockIdx.x, lane = threadIdx.x & 31, s = blockIdx.y * 8 + (threadIdx.x >> 5);
    uint32_t q[2] = {0u, 0u};
    float d = 0.0f;
    int ls = 0;
    if (s < B) warp_quant_block(x + (size_t)s * ldx + (size_t)k * G4_QK, lane, q, d, ls);
    tc_store_q8(bq + (size_t)k * 320 * NP, yd + (size_t)k * NP, NP, s, lane, q, d, ls);
}

// Same operand from BlockQ8_K rows already quantized by the caller
// (q8: [B][nb] blocks of 292 bytes).
__global__ void tc_from_q8_kernel(const uint8_t *__restrict__ q8, int nb, int B, int NP, uint8_t *__restrict__ bq,
                                  float *__restrict__ yd) {
    pdl_trigger();
    pdl_wait();
    const int k = blockIdx.x, lane = threadIdx.x & 31, s = blockIdx.y * 8 + (threadIdx.x >> 5);
    uint32_t q[2] = {0u, 0u};
    float d = 0.0f;
    int ls = 0;
    if (s < B) {
        const uint8_t *blk = q8 + ((size_t)s * nb + k) * G4_Q8_BYTES;
        d = *reinterpret_cast<const float *>(blk);
        q[0] = *reinterpret_cast<const uint32_t *>(blk + 4 + 8 * lane);
        q[1] = *reinterpret_cast<const uint32_t *>(blk + 8 + 8 * lane);
        for (int b = 0; b < 4; b++) ls += (int)(int8_t)(q[0] >> (8 * b)) + (int)(int8_t)(q[1] >> (8 * b));
    }
    tc_store_q8(bq + (size_t)k * 320 * NP, yd + (size_t)k * NP, NP, s, lane, q, d, ls);
}

// ---------------------------------------------------------------- Q4_K: fp16 MMA, A operand in TMEM
//
// The same products for Q4_K with kind::f16 operands that hold exact small
// integers: A = sc_j * q (<= 63*15 = 945) and mins mn_j, B = q8 and the
// 16-element sums bsums[k] of Q8_K (|.| <= 2048).  Every product is exact in
// fp32 and every partial sum is an integer below 2^24 in magnitude as long
// as it spans at most 128 weights (945*128*128 < 2^24), so the fp32
// accumulators hold the exact integers: S0 (weights 0..127), S1 (128..255)
// and M.  S0 + S1 rounds once, exactly like (float)sumi in the reference.
// The expanded weights go straight from registers into TMEM (tcgen05.st) and
// the MMA reads A from there, so shared memory only carries the raw weight
// tile and the B operand.
//
// K order inside each group of 4 weights is (0, 2, 1, 3): two nibbles of
// one 16-bit lane pair become one 32-bit TMEM column with one mask.  The B
// operand is written in the same order, so the dot product is unchanged.

constexpr int kQ4Threads = 608;  // warp 0 producer, warps 1 and 18 MMA, warps 2..17 expand + epilogue
constexpr int kQ4RawStages = 5;

template <int NP>
struct Q4Smem {
    static constexpr int raw = 128 * 144;
    static constexpr int bst = 544 * NP;  // 256*NP fp16 quants + 16*NP fp16 bsums
    static constexpr int bstages = NP == 64 ? 3 : 4;
    static constexpr int b_off = kQ4RawStages * raw;
    // A operand of the mins MMA, two slots: 128 rows x 16 fp16, K-major core matrices
    // (byte (k/8)*2048 + r*16 + (k%8)*2)
    static constexpr int mins_off = b_off + bstages * bst;
    static constexpr int total = mins_off + 2 * 4096 + 1024;
};
// TMEM columns: [D_s0 | D_s1] and D_m for two blocks in flight (slot i&1 of
// block i is released by the epilogue through acc_empty), then the four
// 64-weight quarters of A (32 columns each).
template <int NP>
struct Q4Tmem {
    static constexpr uint32_t dm = 4 * NP, a = 6 * NP;
    static_assert(a + 128 <= 512, "TMEM columns");
};

struct Q4State {
    uint64_t raw_full[kQ4RawStages], raw_empty[kQ4RawStages], b_full[4], b_empty[4];
    uint64_t a_full[4], a_empty[4], acc_full[2], acc_empty[2], mma_done;
    uint32_t tmem_base;
    volatile int abort;
    int mcount;               // split row tiles this CTA finished last (merged after its units)
    int mlist[kTcMergeCap];
    alignas(16) float yd[8][2][32];  // per epilogue warp (read as float2): block scales of its sequences, by block parity
};

// Waiting warps sleep in the barrier (1 ms suspend hint) instead of
// spinning, so they leave the issue slots of their SMSP to working warps.
__device__ __forceinline__ bool q4_wait(Q4State &S, uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
        if (S.abort) return false;
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
}
__device__ __forceinline__ void q4_fail(Q4State &S, int *err) {
    S.abort = 1;
    if (err) atomicExch(err, G4_ERR_TIMEOUT);
}
// Merge of a split row tile t (this thread: row r of the tile, sequences p*SP ..) from its partial
// slots, summed in slot order (0 + P0 + P1 ...), then stored; for a gate/up pair (a.all_part) the
// gate tile tg and its up tile give GELU(gate) * up (main.c:1973-1978).  Kept out of line: it runs
// once per split tile, by the CTA that finishes it last.
template <int G>
__device__ __forceinline__ void q4_merge_tile(const TcArgs &a, int NP, int SP, int p, int r, int t, int tg) {
    const size_t prow = (size_t)a.prow;
    auto sums = [&](int tt, int s0, float (&v)[G]) {
        const int ns = ((tt + 1) * a.nb - 1) / a.share - (tt * a.nb) / a.share + 1;
        slot_sums<G>(a.part + (size_t)s0 * prow + (size_t)tt * 128 + r, (size_t)NP * prow, prow, ns, v);
    };
    if (a.all_part) {
        const int rw = tg * 128 + r;
        if (rw >= a.rows) return;
        for (int s0 = p * SP; s0 < p * SP + SP && s0 < a.B; s0 += G) {
            float g[G], u[G];
            sums(tg, s0, g);
            sums(a.tiles0 + tg, s0, u);
#pragma unroll
            for (int s = 0; s < G; s++)
                if (s0 + s < a.B) a.out[(size_t)(s0 + s) * a.ldo + rw] = gelu_f32(g[s]) * u[s];
        }
        return;
    }
    const bool m2 = t >= a.tiles0;
    const int row = (m2 ? t - a.tiles0 : t) * 128 + r;
    if (row >= (m2 ? a.rows2 : a.rows)) return;
    float *dst = (m2 ? a.out2 : a.out) + row;
    const size_t ld = m2 ? (size_t)a.ldo2 : (size_t)a.ldo;
    for (int s0 = p * SP; s0 < p * SP + SP && s0 < a.B; s0 += G) {
        float v[G];
        sums(t, s0, v);
#pragma unroll
        for (int s = 0; s < G; s++)
            if (s0 + s < a.B) dst[(size_t)(s0 + s) * ld] = v[s];
    }
}

// Warp roles.  Warps 2..17 work on TMEM lane quadrant (warp & 3), i.e. 32
// weight rows each (a warp may only touch its own quadrant):
//   warps 2..9   expand: warp-group e = (warp-2)/4 expands the quarters 2e
//                and 2e+1 (weights 128e .. 128e+127) of every super-block;
//   warps 10..17 epilogue: group p = (warp-10)/4 owns sequences
//                [p*NP/2, (p+1)*NP/2) and runs the per-block float epilogue.
// Expansion of block i+1 and the epilogue of block i then run concurrently
// on every SMSP.
template <int NP>
__global__ void __launch_bounds__(kQ4Threads, 1) gemm_q4tc_kernel(const __grid_constant__ CUtensorMap tmw,
                                                                  const __grid_constant__ CUtensorMap tmw2, TcArgs a) {
    constexpr int RAW = Q4Smem<NP>::raw, BST = Q4Smem<NP>::bst, BS = Q4Smem<NP>::bstages, RS = kQ4RawStages;
    constexpr int SP = NP / 2;  // sequences per epilogue warp
    using TM = Q4Tmem<NP>;
    extern __shared__ uint8_t smem_dyn[];
    __shared__ Q4State S;
    uint8_t *smem = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
    uint8_t *raw = smem, *bst = smem + Q4Smem<NP>::b_off, *mins_s = smem + Q4Smem<NP>::mins_off;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_trigger();
    if (tid == 0) {
        for (int i = 0; i < RS; i++) {
            mbar_init(&S.raw_full[i], 1);
            mbar_init(&S.raw_empty[i], 8);  // expand warps
        }
        for (int i = 0; i < BS; i++) {
            mbar_init(&S.b_full[i], 1);
            mbar_init(&S.b_empty[i], 2);  // both MMA issuers
        }
        for (int i = 0; i < 4; i++) {
            mbar_init(&S.a_full[i], 4);  // the four lane quadrants of quarter i
            mbar_init(&S.a_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&S.acc_full[i], 2);   // both MMA issuers
            mbar_init(&S.acc_empty[i], 8);  // epilogue warps
        }
        mbar_init(&S.mma_done, 2);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.abort = 0;
        S.mcount = 0;
    }
    if (warp == 1) tc_alloc(&S.tmem_base, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = S.tmem_base;
    // this CTA's units [g0, g1): unit g = (row tile g / nb, super-block g % nb)
    const int g0 = blockIdx.x * a.share, g1 = min(a.total, g0 + a.share);

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int i = 0, nb_issued = 0;
            bool ok = true, dep = false;
            for (int g = g0; g < g1; g++, i++) {
                const int t = g / a.nb, b = g - t * a.nb;
                const bool m2 = t >= a.tiles0;
                const int rs = i % RS;
                if (!q4_wait(S, &S.raw_empty[rs], ((i / RS) & 1) ^ 1)) { ok = false; break; }
                mbar_expect_tx(&S.raw_full[rs], RAW);
                tma_load_2d(raw + rs * RAW, m2 ? &tmw2 : &tmw, b * 144, (m2 ? t - a.tiles0 : t) * 128, &S.raw_full[rs]);
                if (!dep) { pdl_wait(); dep = true; }
                const int bs = i % BS;
                if (!q4_wait(S, &S.b_empty[bs], ((i / BS) & 1) ^ 1)) { ok = false; i++; break; }
                mbar_expect_tx(&S.b_full[bs], BST);
                bulk_g2s(bst + bs * BST, a.bq + (size_t)b * BST, BST, &S.b_full[bs]);
                nb_issued = i + 1;
            }
            if (!dep) pdl_wait();
            if (!ok) {
                q4_fail(S, a.err);
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
    } else if (warp == 1 || warp == kQ4Threads / 32 - 1) {
        // ------------------------------------------------------------ MMA issuers
        // Two threads issue MMAs: warp 1 the quarters 0, 1 (S0) and the mins, the last warp the
        // quarters 2, 3 (S1), each right after the expand warp group of its quarters.  Each
        // issuer's commits track its own MMAs; acc_full, b_empty and mma_done count both.
        const int h = warp == 1 ? 0 : 1;
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc(1, 0, 0, NP);  // f32 += f16 * f16
            int i = 0;
            bool ok = true;
            for (int g = g0; g < g1 && ok; g++, i++) {
                const int abuf = i & 1, bs = i % BS;
                const uint32_t pa = i & 1;
                {   // the accumulator pair and the B stage tested together (the tests overlap)
                    const bool r0 = mbar_try_wait(&S.acc_empty[abuf], ((i >> 1) & 1) ^ 1);
                    const bool r1 = mbar_try_wait(&S.b_full[bs], (i / BS) & 1);
                    if (!(r0 && r1)) {
                        if (!q4_wait(S, &S.acc_empty[abuf], ((i >> 1) & 1) ^ 1) ||
                            !q4_wait(S, &S.b_full[bs], (i / BS) & 1)) { ok = false; break; }
                    }
                }
                const uint32_t bsa = smem_u32(bst + bs * BST);
                const uint32_t dq = tbase + abuf * 2 * NP + h * NP;  // S0: weights 0..127, S1: 128..255
                for (int qq = 0; qq < 2; qq++) {
                    const int q = 2 * h + qq;
                    if (!mbar_try_wait(&S.a_full[q], pa) && !q4_wait(S, &S.a_full[q], pa)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t acol = tbase + TM::a + 32 * q;
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        tc_mma_f16_ts(dq, acol + 8 * ks, umma_desc(bsa + (8 * q + 2 * ks) * NP * 16, NP * 16, 128), idesc,
                                      (ks | qq) != 0);
                    tc_commit(&S.a_empty[q]);
                }
                if (!ok) break;
                if (h == 0) {
                    // mins x bsums (K = 16) into D_m slot i&1 (free: acc_empty above).  The mins of block
                    // i sit in shared-memory slot i&1 (written with quarter 0); the expand warps rewrite
                    // it for block i+2 only after quarter 0 of block i+1 was consumed, i.e. after this
                    // MMA (issued by the same thread before that quarter) completed.
                    tc_mma_f16(tbase + TM::dm + NP * abuf, umma_desc(smem_u32(mins_s) + 4096 * abuf, 2048, 128),
                               umma_desc(bsa + 512 * NP, NP * 16, 128), idesc, 0);
                }
                tc_commit(&S.b_empty[bs]);
                tc_commit(&S.acc_full[abuf]);
            }
            if (!ok) q4_fail(S, a.err);
            tc_commit(&S.mma_done);
            const unsigned long long t0 = global_ns();
            while (!mbar_try_wait(&S.mma_done, 0) && global_ns() - t0 < kWaitLimitNs) {}
        }
        __syncwarp();
    } else if (warp < 10) {
        // ------------------------------------------------------------ expand warps
        const int quad = warp & 3, e = (warp - 2) >> 2, r = 32 * quad + lane;
        const uint32_t tl = tbase + ((uint32_t)(32 * quad) << 16);
        const uint32_t raw_s = smem_u32(raw);
        int i = 0;
        bool ok = true;
        {
            for (int g = g0; g < g1; g++, i++) {
                const int rs = i % RS;
                if (!q4_wait(S, &S.raw_full[rs], (i / RS) & 1)) { ok = false; break; }
                const uint32_t rw = raw_s + rs * RAW + r * 144;
                const uint4 meta = lds128(rw);
                const uint4 qa = lds128(rw + 16 + 64 * e), qb = lds128(rw + 32 + 64 * e);
                const uint4 qc = lds128(rw + 48 + 64 * e), qd = lds128(rw + 64 + 64 * e);
                const uint32_t sc03 = meta.y & 0x3f3f3f3fu;
                const uint32_t sc47 = (meta.w & 0x0f0f0f0fu) | ((meta.y >> 2) & 0x30303030u);
                uint32_t mc[8];
                if (e == 0) {  // mins of sub-blocks 0..7, each twice (against the bsums of 16)
                    const uint32_t mn03 = meta.z & 0x3f3f3f3fu;
                    const uint32_t mn47 = ((meta.w >> 4) & 0x0f0f0f0fu) | ((meta.z >> 2) & 0x30303030u);
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        const uint32_t m = __byte_perm(mn03, mn47, 0x4440 | c) & 0xffu;
                        mc[c] = hadd2_u(m | (m << 16) | 0x64006400u, 0xE400E400u);  // (1024+m) - 1024
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.raw_empty[rs]);  // everything needed is in registers
#pragma unroll
                for (int qq = 0; qq < 2; qq++) {
                    const int q = 2 * e + qq;  // quarter: 64-weight group q, sub-blocks 2q (low nibbles), 2q+1 (high)
                    const uint32_t qw[8] = {qq ? qc.x : qa.x, qq ? qc.y : qa.y, qq ? qc.z : qa.z, qq ? qc.w : qa.w,
                                            qq ? qd.x : qb.x, qq ? qd.y : qb.y, qq ? qd.z : qb.z, qq ? qd.w : qb.w};
                    if (!q4_wait(S, &S.a_empty[q], (i & 1) ^ 1)) { ok = false; break; }
                    // low nibble q at bits 0..3 of a 16-bit lane: fp16 bits 0x6400|q = 1024+q, and
                    //   fma(1024+q, sc, -1024*sc) = sc*q exactly (fused, |sc*q| <= 945);
                    // high nibble at bits 4..7: 0x6400|16q = 1024+16q, fma(1024+16q, sc/16, -64*sc) = sc*q.
                    const int scl = (int)(__byte_perm(sc03, sc47, 0x4440 | (2 * q)) & 0xffu);
                    const int sch = (int)(__byte_perm(sc03, sc47, 0x4440 | (2 * q + 1)) & 0xffu);
                    uint32_t hl = h_of_int(scl), hlc = h_of_int(-1024 * scl);
                    uint32_t hh = (uint32_t)__half_as_ushort(__float2half_rn((float)sch * 0.0625f)), hhc = h_of_int(-64 * sch);
                    const uint32_t sl2 = hl | (hl << 16), cl2 = hlc | (hlc << 16);
                    const uint32_t sh2 = hh | (hh << 16), ch2 = hhc | (hhc << 16);
                    uint32_t col[16], coh[16];
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        const uint32_t x = qw[k], y = __byte_perm(x, 0u, 0x4341);  // bytes 1, 3 -> lanes 0, 1
                        col[2 * k] = hfma2_u((x & 0x000F000Fu) | 0x64006400u, sl2, cl2);
                        col[2 * k + 1] = hfma2_u((y & 0x000F000Fu) | 0x64006400u, sl2, cl2);
                        coh[2 * k] = hfma2_u((x & 0x00F000F0u) | 0x64006400u, sh2, ch2);
                        coh[2 * k + 1] = hfma2_u((y & 0x00F000F0u) | 0x64006400u, sh2, ch2);
                    }
                    tc_st16(tl + TM::a + 32 * q, col);
                    tc_st16(tl + TM::a + 32 * q + 16, coh);
                    if (q == 0) {  // mins of row r for the mins MMA (generic-proxy stores, then proxy fence)
                        uint8_t *mrow = mins_s + 4096 * (i & 1) + r * 16;
                        *reinterpret_cast<uint4 *>(mrow) = make_uint4(mc[0], mc[1], mc[2], mc[3]);
                        *reinterpret_cast<uint4 *>(mrow + 2048) = make_uint4(mc[4], mc[5], mc[6], mc[7]);
                        fence_proxy_async_smem();
                    }
                    tc_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.a_full[q]);
                }
                if (!ok) break;
            }
        }
        if (!ok) q4_fail(S, a.err);
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
        // scales of unit g: the (d, dmin) word of row r of its super-block (weights, just streamed
        // through L2) and the Q8_K d of sequence p*SP + lane, loaded one unit ahead and converted
        // only when used, so the load latency overlaps the current unit
        auto fetch = [&](int g, uint32_t &mw, float &yl) {
            const int t = g / a.nb, b = g - t * a.nb;
            const bool m2 = t >= a.tiles0;
            const int row = (m2 ? t - a.tiles0 : t) * 128 + r;
            mw = 0;
            if (row < (m2 ? a.rows2 : a.rows))
                mw = __ldg(reinterpret_cast<const uint32_t *>((m2 ? a.w2 : a.w) + (size_t)row * a.row_bytes + (size_t)b * 144));
            yl = lane < SP ? __ldg(a.yd + (size_t)b * NP + p * SP + lane) : 0.0f;
        };
        // End of this CTA's units of row tile t.  A tile wholly inside this CTA is stored (unless
        // a.all_part); a tile shared by several CTAs leaves its partial in slot (CTA - first CTA of
        // the tile), and the slots are summed in slot order: by the CTA that completes the tile (tickets)
        // or by sk_merge_kernel.
        auto finish = [&](int t) {
            const bool m2 = t >= a.tiles0;
            const int row = (m2 ? t - a.tiles0 : t) * 128 + r;
            const int first = (t * a.nb) / a.share;
            const int nseg = ((t + 1) * a.nb - 1) / a.share - first + 1;
            if (nseg == 1 && !a.all_part) {
                float *dst = (m2 ? a.out2 : a.out) + row;
                const size_t ld = m2 ? (size_t)a.ldo2 : (size_t)a.ldo;
                if (row < (m2 ? a.rows2 : a.rows))
#pragma unroll
                    for (int s = 0; s < SP / 2; s++) {
                        const float2 f = f2_unpack(acc[s]);
                        const int seq = p * SP + 2 * s;
                        if (seq < a.B) dst[(size_t)seq * ld] = f.x;
                        if (seq + 1 < a.B) dst[(size_t)(seq + 1) * ld] = f.y;
                    }
            } else {
                const size_t prow = (size_t)a.prow;
                float *mine = a.part + (size_t)(blockIdx.x - first) * NP * prow + (size_t)t * 128 + r +
                              (size_t)(p * SP) * prow;
#pragma unroll
                for (int s = 0; s < SP / 2; s++) {
                    const float2 f = f2_unpack(acc[s]);
                    mine[(size_t)(2 * s) * prow] = f.x;
                    mine[(size_t)(2 * s + 1) * prow] = f.y;
                }
                if (a.tickets) {
                    // Count this CTA's part in; the CTA that completes the tile (for a gate/up pair: both
                    // tiles of the pair) merges it after its units, in slot order 0 + P0 + P1 + ...
                    __threadfence();
                    asm volatile("bar.sync 1, 256;" ::: "memory");  // the 8 epilogue warps
                    if (warp == 10 && lane == 0) {
                        auto nseg_of = [&](int tt) { return ((tt + 1) * a.nb - 1) / a.share - (tt * a.nb) / a.share + 1; };
                        const int tg = m2 ? t - a.tiles0 : t;
                        const int tk = a.all_part ? tg : t;
                        const int expect = a.all_part ? nseg_of(tg) + nseg_of(a.tiles0 + tg) : nseg;
                        if (atomicAdd(a.tickets + tk, 1) == expect - 1) {
                            if (S.mcount < kTcMergeCap) S.mlist[S.mcount++] = t;
                            else if (a.err) atomicExch(a.err, G4_ERR_STATE);
                        }
                    }
                }
            }
#pragma unroll
            for (int s = 0; s < SP / 2; s++) acc[s] = 0ull;
        };
        uint32_t nmw = 0;
        float nyl = 0.f;
        if (g0 < g1) fetch(g0, nmw, nyl);
        for (int g = g0; g < g1; g++, i++) {
            const uint32_t mw = nmw;
            if (lane < SP) S.yd[pw][i & 1][lane] = nyl;
            __syncwarp();
            if (g + 1 < g1) fetch(g + 1, nmw, nyl);  // prefetch the next unit's scales
            // ---- epilogue of block i
            if (!q4_wait(S, &S.acc_full[i & 1], (i >> 1) & 1)) { ok = false; break; }
            tc_fence_after();
            const float *yv = S.yd[pw][i & 1];
            const float dw = f16_to_f32((uint16_t)(mw & 0xffffu)), dm = f16_to_f32((uint16_t)(mw >> 16));
            const unsigned long long dw2 = f2_pack(dw, dw), ndm2 = f2_pack(-dm, -dm);
#pragma unroll
            for (int c = 0; c < SP / 8; c++) {
                uint32_t v0[8], v1[8], vm[8];
                tc_ld8(tl + (i & 1) * 2 * NP + p * SP + 8 * c, v0);
                tc_ld8(tl + (i & 1) * 2 * NP + NP + p * SP + 8 * c, v1);
                tc_ld8(tl + TM::dm + (i & 1) * NP + p * SP + 8 * c, vm);
                tc_wait_ld();
                if (c == SP / 8 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.acc_empty[i & 1]);
                }
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    // t = dw*(S0 + S1) - dm*M; acc += yd*t, two sequences per instruction
                    const unsigned long long sf = f2_add(f2_pack_u(v0[2 * k], v0[2 * k + 1]), f2_pack_u(v1[2 * k], v1[2 * k + 1]));
                    const unsigned long long mt = f2_mul(ndm2, f2_pack_u(vm[2 * k], vm[2 * k + 1]));
                    const unsigned long long t = f2_fma(dw2, sf, mt);
                    const float2 y = *reinterpret_cast<const float2 *>(yv + 8 * c + 2 * k);
                    acc[4 * c + k] = f2_fma(f2_pack(y.x, y.y), t, acc[4 * c + k]);
                }
            }
            if (g + 1 == g1 || (g + 1) % a.nb == 0) finish(g / a.nb);
        }
        if (!ok) {
            q4_fail(S, a.err);
        } else if (a.tickets) {
            asm volatile("bar.sync 1, 256;" ::: "memory");  // S.mlist complete
            const int nm = S.mcount;
            if (nm) __threadfence();
            for (int m = 0; m < nm; m++) {
                const int t = S.mlist[m];
                q4_merge_tile<(SP < 16 ? SP : 16)>(a, NP, SP, p, r, t, t >= a.tiles0 ? t - a.tiles0 : t);
            }
            if (warp == 10 && lane < nm) {  // ready for the next launch
                const int t = S.mlist[lane];
                a.tickets[a.all_part ? (t >= a.tiles0 ? t - a.tiles0 : t) : t] = 0;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tc_dealloc(tbase, 512);
    }
}

__global__ void tc4_quant_kernel(const float *__restrict__ x, int ldx, int B, int NP, uint8_t *__restrict__ bq,
                                 float *__restrict__ yd) {
    pdl_trigger();
    pdl_wait();
    const int k = blockIdx.x, lane = threadIdx.x & 31, s = blockIdx.y * 8 + (threadIdx.x >> 5);
    uint32_t q[2] = {0u, 0u};
    float d = 0.0f;
    int ls = 0;
    if (s < B) warp_quant_block(x + (size_t)s * ldx + (size_t)k * G4_QK, lane, q, d, ls);
    tc4_store_q8(bq + (size_t)k * 544 * NP, yd + (size_t)k * NP, NP, s, lane, q, d, ls);
}

__global__ void tc4_from_q8_kernel(const uint8_t *__restrict__ q8, int nb, int B, int NP, uint8_t *__restrict__ bq,
                                   float *__restrict__ yd) {
    pdl_trigger();
    pdl_wait();
    const int k = blockIdx.x, lane = threadIdx.x & 31, s = blockIdx.y * 8 + (threadIdx.x >> 5);
    uint32_t q[2] = {0u, 0u};
    float d = 0.0f;
    int ls = 0;
    if (s < B) {
        const uint8_t *blk = q8 + ((size_t)s * nb + k) * G4_Q8_BYTES;
        d = *reinterpret_cast<const float *>(blk);
        q[0] = *reinterpret_cast<const uint32_t *>(blk + 4 + 8 * lane);
        q[1] = *reinterpret_cast<const uint32_t *>(blk + 8 + 8 * lane);
        for (int b = 0; b < 4; b++) ls += (int)(int8_t)(q[0] >> (8 * b)) + (int)(int8_t)(q[1] >> (8 * b));
    }
    tc4_store_q8(bq + (size_t)k * 544 * NP, yd + (size_t)k * NP, NP, s, lane, q, d, ls);
}

template <int NP>
void *q4tc_kernel_ptr() { return (void *)gemm_q4tc_kernel<NP>; }

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_encode_mu;

int get_encode() {
    std::lock_guard<std::mutex> lk(g_encode_mu);
    if (g_encode) return G4_OK;
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    G4_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn) {
        set_error(G4_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
        return G4_ERR_CUDA;
    }
    g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    return G4_OK;
}

template <int TYPE, int NP>
void *tc_kernel_ptr() { return (void *)gemm_tc_kernel<TYPE, NP>; }

}  // namespace

int tc_np(int B) { return B <= 16 ? 16 : B <= 32 ? 32 : 64; }

// per super-block: the larger (Q4_K fp16) operand layout at NP = 64, then the block scales
size_t tc_operand_bytes(int n) { return (size_t)(n / G4_QK) * (544 * 64 + 64 * 4); }
size_t tc_yd_offset(int n) { return (size_t)(n / G4_QK) * 544 * 64; }

// Weight rows as a 2-D byte tensor [rows][row_bytes]; one box = 128 rows x
// one super-block.
int tc_weight_map(CUtensorMap *m, const void *w, int type, int n, int rows) {
    if (const int rc = get_encode()) return rc;
    if (((uintptr_t)w & 15u) != 0) { set_error(G4_ERR_ARG, "tc: weight pointer not 16-byte aligned"); return G4_ERR_ARG; }
    const cuuint64_t dims[2] = {(cuuint64_t)device_row_bytes(type, n), (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)device_row_bytes(type, n)};
    const cuuint32_t box[2] = {(cuuint32_t)(type == G4_Q4_K ? 144 : type == G4_Q5_K ? 176 : 208), 128u};
    const cuuint32_t es[2] = {1u, 1u};
    const CUresult rc = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(w), dims, strides, box, es,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) { set_error(G4_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)rc); return G4_ERR_CUDA; }
    return G4_OK;
}

TcPlan tc_plan(int rows, int nb, int nsm) {
    const int tiles = (rows + 127) / 128;
    TcPlan best{1, nb, tiles, min(tiles, nsm)};
    double best_cost = 1e30;
    for (int ks = 1; ks <= nb; ks++) {
        const int ksplit = (nb + ks - 1) / ks;
        const int units = tiles * ksplit, grid = min(units, nsm), waves = (units + grid - 1) / grid;
        // in block times: per unit pipeline fill and partial store, per split one merge pass
        const double cost = waves * (ks + 1.5) + (ksplit > 1 ? 3.0 : 0.0);
        if (cost < best_cost - 1e-9 || (fabs(cost - best_cost) < 1e-9 && ks > best.kslice)) {
            best_cost = cost;
            best = TcPlan{ksplit, ks, units, grid};
        }
    }
    return best;
}

int launch_tc_quant(int type, const float *x, int ldx, int B, int n, int np, uint8_t *bq, float *yd, cudaStream_t st) {
    if (type == G4_Q4_K) G4_CUDA(launch_pdl(tc4_quant_kernel, dim3(n / G4_QK, np / 8), dim3(256), 0, st, x, ldx, B, np, bq, yd));
    else G4_CUDA(launch_pdl(tc_quant_kernel, dim3(n / G4_QK, np / 8), dim3(256), 0, st, x, ldx, B, np, bq, yd));
    G4_LAUNCHED();
    return G4_OK;
}

int launch_tc_from_q8(int type, const void *q8, int B, int n, int np, uint8_t *bq, float *yd, cudaStream_t st) {
    if (type == G4_Q4_K)
        G4_CUDA(launch_pdl(tc4_from_q8_kernel, dim3(n / G4_QK, np / 8), dim3(256), 0, st, (const uint8_t *)q8,
                           n / G4_QK, B, np, bq, yd));
    else G4_CUDA(launch_pdl(tc_from_q8_kernel, dim3(n / G4_QK, np / 8), dim3(256), 0, st, (const uint8_t *)q8, n / G4_QK,
                       B, np, bq, yd));
    G4_LAUNCHED();
    return G4_OK;
}

// Stream-K split of the Q4_K GEMM: `share` consecutive (row tile, super-block) units per CTA,
// chosen to minimise waves * (share + per-CTA fixed cost) + the fix-up of split tiles, all in
// super-block times.  nseg_max = most CTAs sharing one tile (partial slots needed).
Q4Plan q4_plan(int tiles, int nb, int nsm) {
    const int total = tiles * nb;
    Q4Plan best{1, 0, 1};
    if (total <= 0 || nsm <= 0) return best;
    best.share = total;
    best.grid = 1;
    double best_cost = 1e30;
    for (int share = 1; share <= total; share++) {
        const int ctas = (total + share - 1) / share, waves = (ctas + nsm - 1) / nsm;
        // some CTA boundary falls inside a tile unless every boundary is a multiple of nb
        const bool split = share < total && share % nb != 0;
        const double cost = waves * (share + 2.5) + (split ? 0.5 : 0.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best.share = share;
            best.grid = ctas;
        }
    }
    best.nseg_max = 1;
    for (int t = 0; t < tiles; t++)
        best.nseg_max = max(best.nseg_max, ((t + 1) * nb - 1) / best.share - (t * nb) / best.share + 1);
    return best;
}

RowOrder q4_row_order(int rows_a, int rows_b, int n, int nsm, int which) {
    const int nb = n / G4_QK, ta = (rows_a + 127) / 128, tb = rows_b > 0 ? (rows_b + 127) / 128 : 0;
    const Q4Plan p = q4_plan(ta + tb, nb, nsm);
    return RowOrder{which ? ta : 0, p.share, 0};
}

RowOrder q5_row_order(int rows, int n, int nsm) {
    const TcPlan p = tc_plan(rows, n / G4_QK, nsm);
    return RowOrder{0, 0, p.ksplit > 1 ? p.kslice : 0};
}

size_t tc_part_bytes(int rows, int n, int nsm) {
    const TcPlan p = tc_plan(rows, n / G4_QK, nsm);
    const int tiles = (rows + 127) / 128;
    const Q4Plan q = q4_plan(tiles, n / G4_QK, nsm);
    const size_t uni = p.ksplit > 1 ? (size_t)p.ksplit * 64 * rows * sizeof(float) : 0;
    const size_t sk = (size_t)q.nseg_max * 64 * tiles * 128 * sizeof(float);  // split tiles, or a merge epilogue
    return std::max(uni, sk);
}

// Sum of the partial slots of gemm_q4tc (slot order) for the row tiles that several CTAs shared,
// or for every tile (all_part), then the epilogue: store, or GELU(gate) * up for a gate/up pair
// (matrix 1 = gate, matrix 2 = up, same rows; main.c:1973-1978).  One thread per (row, sequence).
__global__ void sk_merge_kernel(const float *__restrict__ part, int prow, int NP, int nb, int share, int tiles0,
                                int rows, float *__restrict__ out, int ldo, int rows2, float *__restrict__ out2,
                                int ldo2, int B, int epi, int all_part) {
    pdl_trigger();
    pdl_wait();
    const int grow = blockIdx.x * blockDim.x + threadIdx.x, s = blockIdx.y;
    if (grow >= prow || s >= B) return;
    auto sum = [&](int t, int gr) {
        const int first = (t * nb) / share, nseg = ((t + 1) * nb - 1) / share - first + 1;
        float v = 0.0f;
        for (int k = 0; k < nseg; k++) v += part[((size_t)k * NP + s) * prow + gr];
        return v;
    };
    const int t = grow / 128;
    if (epi == EPI_GELU_MUL) {  // grid covers the gate tiles only
        if (grow >= rows) return;
        const float g = sum(t, grow), u = sum(tiles0 + t, tiles0 * 128 + grow);
        out[(size_t)s * ldo + grow] = gelu_f32(g) * u;
        return;
    }
    if (!all_part && ((t + 1) * nb - 1) / share == (t * nb) / share) return;  // stored by its CTA
    const bool m2 = t >= tiles0;
    const int row = grow - (m2 ? tiles0 * 128 : 0);
    if (row >= (m2 ? rows2 : rows)) return;
    (m2 ? out2 : out)[(size_t)s * (m2 ? ldo2 : ldo) + row] = sum(t, grow);
}

int launch_gemm_q4tc2(const CUtensorMap *tm, const void *w, int rows, float *out, int ldo, const CUtensorMap *tm2,
                      const void *w2, int rows2, float *out2, int ldo2, int n, const uint8_t *bq, const float *yd, int B,
                      int np, float *part, size_t part_bytes, int *err, int nsm, cudaStream_t st,
                      int epi, int *tickets) {
    if (B < 1 || B > np || (np != 16 && np != 32 && np != 64)) { set_error(G4_ERR_ARG, "tc gemm: batch %d / %d", B, np); return G4_ERR_ARG; }
    if (epi != EPI_STORE && !(epi == EPI_GELU_MUL && w2 && rows2 == rows)) {
        set_error(G4_ERR_ARG, "tc gemm: epilogue %d needs a gate/up pair of equal shape", epi);
        return G4_ERR_ARG;
    }
    const int nb = n / G4_QK, tiles0 = (rows + 127) / 128, tiles = tiles0 + (w2 ? (rows2 + 127) / 128 : 0);
    const Q4Plan p = q4_plan(tiles, nb, nsm);
    const bool all_part = epi == EPI_GELU_MUL, merge = all_part || p.nseg_max > 1;
    if (merge && (size_t)p.nseg_max * np * tiles * 128 * sizeof(float) > part_bytes) {
        set_error(G4_ERR_ARG, "tc gemm: partial buffer too small");
        return G4_ERR_ARG;
    }
    // in-kernel merges: a CTA keeps at most kTcMergeCap tiles to merge (its first and last tile, or
    // for a gate/up pair every tile it touches)
    if (tickets && all_part && (p.share + nb - 1) / nb + 1 > kTcMergeCap) tickets = nullptr;
    TcArgs a{(const uint8_t *)w, device_row_bytes(G4_Q4_K, n), bq, yd, out, part, err, nb, rows, B, ldo,
             1, nb, tiles, EPI_STORE, 0.0f, nullptr};
    a.w2 = (const uint8_t *)w2; a.out2 = out2; a.rows2 = rows2; a.ldo2 = ldo2; a.tiles0 = w2 ? tiles0 : tiles;
    a.share = p.share; a.total = tiles * nb; a.prow = tiles * 128; a.all_part = all_part ? 1 : 0;
    a.tickets = tickets;
    const CUtensorMap *m2 = w2 ? tm2 : tm;
#define G4_Q4TC_CASE(N)                                                                                  \
    if (np == N)                                                                                           \
        G4_CUDA(launch_pdl(gemm_q4tc_kernel<N>, dim3(p.grid), dim3(kQ4Threads), (size_t)Q4Smem<N>::total, st, *tm, \
                           *m2, a));
    G4_Q4TC_CASE(16) else G4_Q4TC_CASE(32) else G4_Q4TC_CASE(64)
#undef G4_Q4TC_CASE
    G4_LAUNCHED();
    if (!merge || tickets) return G4_OK;  // with tickets the kernel merges split tiles itself
    const int mrows = all_part ? tiles0 * 128 : tiles * 128;
    G4_CUDA(launch_pdl(sk_merge_kernel, dim3((unsigned)(mrows / 128), (unsigned)B), dim3(128), 0, st, (const float *)part,
                       tiles * 128, np, nb, p.share, a.tiles0, rows, out, ldo, rows2, out2, ldo2, B, epi, a.all_part));
    G4_LAUNCHED();
    return G4_OK;
}

int launch_gemm_tc(const CUtensorMap *tm, const void *w, int type, int n, int rows, const uint8_t *bq, const float *yd, int B, int np,
                   float *out, int ldo, float *part, size_t part_bytes, int *err, int nsm,
                   cudaStream_t st, int *tickets) {
    if (type != G4_Q4_K && type != G4_Q5_K) { set_error(G4_ERR_TYPE, "tc gemm: type %d", type); return G4_ERR_TYPE; }
    if (type == G4_Q4_K)
        return launch_gemm_q4tc2(tm, w, rows, out, ldo, nullptr, nullptr, 0, nullptr, 0, n, bq, yd, B, np, part, part_bytes,
                                 err, nsm, st, EPI_STORE, tickets);
    if (B < 1 || B > np || (np != 16 && np != 32 && np != 64)) { set_error(G4_ERR_ARG, "tc gemm: batch %d / %d", B, np); return G4_ERR_ARG; }
    const int nb = n / G4_QK;
    const TcPlan p = tc_plan(rows, nb, nsm);
    if (p.ksplit > 1 && (size_t)p.ksplit * np * rows * sizeof(float) > part_bytes) {
        set_error(G4_ERR_ARG, "tc gemm: partial buffer too small");
        return G4_ERR_ARG;
    }
    TcArgs a{(const uint8_t *)w, device_row_bytes(type, n), bq, yd, out, part, err, nb, rows, B, ldo,
             p.ksplit, p.kslice, p.units, EPI_STORE, 0.0f, nullptr};
    void *k = nullptr;
    size_t smem = 0;
#define G4_TC_CASE(T, N)                                                          \
    if (type == T && np == N) {                                                    \
        k = tc_kernel_ptr<T, N>();                                                 \
        smem = TcSmem<T, N>::total;                                                \
        G4_CUDA(launch_pdl(gemm_tc_kernel<T, N>, dim3(p.grid), dim3(kTcThreads), smem, st, *tm, a)); \
    }
    G4_TC_CASE(G4_Q5_K, 16) else G4_TC_CASE(G4_Q5_K, 32) else G4_TC_CASE(G4_Q5_K, 64)
#undef G4_TC_CASE
    (void)k;
    (void)smem;
    G4_LAUNCHED();
    if (p.ksplit > 1) return launch_tc_merge(part, p.ksplit, np, rows, B, out, ldo, EPI_STORE, nullptr, 0, st);
    return G4_OK;
}

// Sum of the K-slice partials part[k][s][row] in slice order, then the
// epilogue (store, or GELU(acc) * evec for the per-layer-embedding gate):
// one thread per (sequence, row).
__global__ void tc_merge_kernel(const float *__restrict__ part, int ksplit, int NP, int rows, int B,
                                float *__restrict__ out, int ldo, int epi, const float *__restrict__ evec, int ld_evec) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x * blockDim.x + threadIdx.x, s = blockIdx.y;
    if (row >= rows || s >= B) return;
    float v = 0.0f;
    for (int k = 0; k < ksplit; k++) v += part[((size_t)k * NP + s) * rows + row];
    if (epi == EPI_GELU_SCALE)
        v = gelu_f32(v) * evec[(size_t)s * ld_evec + row];
    out[(size_t)s * ldo + row] = v;
}

int launch_tc_merge(const float *part, int ksplit, int np, int rows, int B, float *out, int ldo, int epi,
                    const float *evec, int ld_evec, cudaStream_t st) {
    G4_CUDA(launch_pdl(tc_merge_kernel, dim3((rows + 127) / 128, B), dim3(128), 0, st, part, ksplit, np, rows, B, out, ldo,
                       epi, evec, ld_evec));
    G4_LAUNCHED();
    return G4_OK;
}

// Dynamic shared-memory limits of the tensor-core kernels (once per device,
// outside any stream capture).
int prime_tc_attrs() {
#define G4_PRIME(K, BYTES) G4_CUDA(cudaFuncSetAttribute((const void *)K, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(BYTES)))
    constexpr int s16 = TcSmem<G4_Q5_K, 16>::total, s32 = TcSmem<G4_Q5_K, 32>::total, s64 = TcSmem<G4_Q5_K, 64>::total;
    G4_PRIME((tc_kernel_ptr<G4_Q5_K, 16>()), s16);
    G4_PRIME((tc_kernel_ptr<G4_Q5_K, 32>()), s32);
    G4_PRIME((tc_kernel_ptr<G4_Q5_K, 64>()), s64);
    G4_PRIME(q4tc_kernel_ptr<16>(), Q4Smem<16>::total);
    G4_PRIME(q4tc_kernel_ptr<32>(), Q4Smem<32>::total);
    G4_PRIME(q4tc_kernel_ptr<64>(), Q4Smem<64>::total);
#undef G4_PRIME
    return G4_OK;
}

}  // namespace g4
