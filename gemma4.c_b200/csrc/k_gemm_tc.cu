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
// CTA (one per SM, persistent): warp 0 issues the bulk tensor copies (TMA) of
// 128-row x 1-super-block weight tiles and of the pre-laid-out B operand;
// warp 1 owns TMEM and one lane issues the MMAs; warps 2..9 expand the raw
// weight tile into the A operands (core-matrix layout, no swizzle) and run the
// epilogue of the previous super-block.  Work units are (128-row tile,
// K-slice); slices of one tile are summed in a fixed order by the warp that
// arrives last (per-warp tickets, no spin-waiting).
//
// Every mbarrier wait is bounded (2 s): on expiry the kernel records
// G4_ERR_TIMEOUT in *err, the producer waits for its copies in flight, the
// MMA lane for its MMAs, TMEM is freed and the CTA returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <mutex>

#include "g4_async.cuh"
#include "g4_internal.cuh"
#include "g4_kernels.cuh"
#include "g4_quant.cuh"

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
        for (int i = 0; i < 32; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (S.abort) return false;
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
}

struct TcArgs {
    const uint8_t *bq;  // [nb][320*NP]: q8 quants (core-matrix layout) then the bsum operand
    const float *yd;    // [nb][NP] Q8_K block scales (0 for padding sequences)
    float *out;         // [B][ldo]
    float *part;        // [ksplit][NP][rows] slice partials (ksplit > 1)
    int *tickets;       // [row_tiles][8], zero between launches
    int *err;
    int nb, rows, B, ldo;
    int ksplit, kslice, units;
};

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
        // slices of one 128-row tile: store, or write a partial and let the last warp sum them
        auto finish = [&](int u) {
            const int rt = u / a.ksplit, ks = u % a.ksplit, row = rt * 128 + r;
            if (a.ksplit == 1) {
                if (row < a.rows)
#pragma unroll
                    for (int s = 0; s < HALF; s++) {
                        const int seq = cb * HALF + s;
                        if (seq < a.B) a.out[(size_t)seq * a.ldo + row] = acc[s];
                    }
            } else {
                if (row < a.rows)
#pragma unroll
                    for (int s = 0; s < HALF; s++) {
                        const int seq = cb * HALF + s;
                        if (seq < a.B) a.part[((size_t)ks * NP + seq) * a.rows + row] = acc[s];
                    }
                __threadfence();
                __syncwarp();
                int last = 0;
                if (lane == 0) last = atomicAdd(&a.tickets[rt * kTcMathWarps + mw], 1) == a.ksplit - 1;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
                    if (row < a.rows)
                        for (int s = 0; s < HALF; s++) {
                            const int seq = cb * HALF + s;
                            if (seq >= a.B) break;
                            float v = 0.0f;
                            for (int k = 0; k < a.ksplit; k++) v += __ldcg(a.part + ((size_t)k * NP + seq) * a.rows + row);
                            a.out[(size_t)seq * a.ldo + row] = v;
                        }
                    if (lane == 0) a.tickets[rt * kTcMathWarps + mw] = 0;
                }
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

size_t tc_operand_bytes(int n) { return (size_t)(n / G4_QK) * (320 * 64 + 64 * 4); }

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
        const double cost = waves * (ks + 1.0);  // + per-unit pipeline fill and partial store
        if (cost < best_cost - 1e-9 || (fabs(cost - best_cost) < 1e-9 && ks > best.kslice)) {
            best_cost = cost;
            best = TcPlan{ksplit, ks, units, grid};
        }
    }
    return best;
}

int launch_tc_quant(const float *x, int ldx, int B, int n, int np, uint8_t *bq, float *yd, cudaStream_t st) {
    G4_CUDA(launch_pdl(tc_quant_kernel, dim3(n / G4_QK, np / 8), dim3(256), 0, st, x, ldx, B, np, bq, yd));
    G4_LAUNCHED();
    return G4_OK;
}

int launch_tc_from_q8(const void *q8, int B, int n, int np, uint8_t *bq, float *yd, cudaStream_t st) {
    G4_CUDA(launch_pdl(tc_from_q8_kernel, dim3(n / G4_QK, np / 8), dim3(256), 0, st, (const uint8_t *)q8, n / G4_QK,
                       B, np, bq, yd));
    G4_LAUNCHED();
    return G4_OK;
}

size_t tc_part_bytes(int rows, int n, int nsm) {
    const TcPlan p = tc_plan(rows, n / G4_QK, nsm);
    return p.ksplit > 1 ? (size_t)p.ksplit * 64 * rows * sizeof(float) : 0;
}
int tc_tickets(int rows) { return ((rows + 127) / 128) * kTcMathWarps; }

int launch_gemm_tc(const CUtensorMap *tm, int type, int n, int rows, const uint8_t *bq, const float *yd, int B, int np,
                   float *out, int ldo, float *part, size_t part_bytes, int *tickets, int *err, int nsm,
                   cudaStream_t st) {
    if (type != G4_Q4_K && type != G4_Q5_K) { set_error(G4_ERR_TYPE, "tc gemm: type %d", type); return G4_ERR_TYPE; }
    if (B < 1 || B > np || (np != 16 && np != 32 && np != 64)) { set_error(G4_ERR_ARG, "tc gemm: batch %d / %d", B, np); return G4_ERR_ARG; }
    const int nb = n / G4_QK;
    const TcPlan p = tc_plan(rows, nb, nsm);
    if (p.ksplit > 1 && (size_t)p.ksplit * np * rows * sizeof(float) > part_bytes) {
        set_error(G4_ERR_ARG, "tc gemm: partial buffer too small");
        return G4_ERR_ARG;
    }
    TcArgs a{bq, yd, out, part, tickets, err, nb, rows, B, ldo, p.ksplit, p.kslice, p.units};
    void *k = nullptr;
    size_t smem = 0;
#define G4_TC_CASE(T, N)                                                          \
    if (type == T && np == N) {                                                    \
        k = tc_kernel_ptr<T, N>();                                                 \
        smem = TcSmem<T, N>::total;                                                \
        G4_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
        G4_CUDA(launch_pdl(gemm_tc_kernel<T, N>, dim3(p.grid), dim3(kTcThreads), smem, st, *tm, a)); \
    }
    G4_TC_CASE(G4_Q4_K, 16) else G4_TC_CASE(G4_Q4_K, 32) else G4_TC_CASE(G4_Q4_K, 64)
    else G4_TC_CASE(G4_Q5_K, 16) else G4_TC_CASE(G4_Q5_K, 32) else G4_TC_CASE(G4_Q5_K, 64)
#undef G4_TC_CASE
    (void)k;
    G4_LAUNCHED();
    return G4_OK;
}

}  // namespace g4
