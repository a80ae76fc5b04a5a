// k_gemm_q6tc.cu — batched Q6_K GEMM on the tensor cores (tcgen05.mma
// kind::i8, int32 accumulators and the A operand in tensor memory), for decode
// steps with 2..64 sequences per GPU: the FFN down projection, V, and the tied
// LM head (with the softcap + argmax epilogue).
//
// The reference computes Q6_K rows as an fp32 dequant-dot against the fp32
// activation (mm_quant_rows, gemma4-4b/cpu-blas/main.c:1539-1556; the weight
// of element k of block b is d * sc_j * (q_k - 32), dequant_q6_k, main.c:
// 213-237).  Here every block product is an exact integer:
//   v_k = sc_j * (q_k - 32) = 64*h_k + l_k,   h in [-63, 64], l in [0, 63]
//   X_k = a0_k*2^16 + a1_k*2^8 + a2_k         (the activation on the block's
//                                             fixed-point grid, q6x_block)
//   D_j = sum_k v_k a_jk = 64*sum h a_j + sum l a_j   (int32, exact)
// so two weight planes (h, l) times three activation pieces give the block
// dot sum_k v_k X_k = D_0*2^16 + D_1*2^8 + D_2 exactly, in any order.  The
// epilogue rounds it to float once per block and accumulates
//   P = fma(float(dot), d * 2^(E-22), P)
// block by block in the canonical row order (RowOrder), exactly as the
// streaming GEMV does: batched and single-sequence results are identical.
//
// CTA layout (one per SM, persistent): warp 0 bulk tensor copies (TMA) of
// 128-row x 1-super-block weight tiles and bulk copies of the B operand;
// warp 1 owns TMEM, one lane issues the MMAs; warps 2..9 expand the 6-bit
// quants into the int8 planes of A in TMEM (tcgen05.st), warp group e = half
// e of the block; warps 10..17 run the per-block epilogue for half of the
// sequences of each MMA pass.  The MMA N is 3 pieces x NPP sequences
// (NPP = 32, two passes at 64 sequences), and consecutive passes rotate
// through the TMEM accumulator buffers that fit beside A (two at N = 96,
// four at N = 48).  Every wait is bounded (2 s).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include "g4_async.cuh"
#include "g4_internal.cuh"
#include "g4_kernels.cuh"
#include "g4_quant.cuh"
#include "g4_tc.cuh"

namespace g4 {

namespace {

constexpr int kQ6Threads = 576;
constexpr int kQ6RawStages = 3;
constexpr int kQ6BStagesMax = 4;

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
struct Q6Cfg {
    static constexpr int NPP = tc6_npp(NP);        // sequences per MMA pass
    static constexpr int NPASS = NP / NPP;          // passes per super-block
    static constexpr int N = 3 * NPP;               // MMA N: three activation pieces
    static constexpr int SP = NPP / 2;              // sequences per epilogue warp and pass
    static constexpr int raw = 128 * 208;           // ql, qh, sc of one super-block for 128 rows
    static constexpr int bst = 768 * NP;            // B operand of one super-block
    static constexpr int BS = NP == 64 ? 3 : 4;      // B operand stages (copies in flight)
    static constexpr int b_off = kQ6RawStages * raw;
    static constexpr int total = b_off + BS * bst + 1024;
    // TMEM: NBUF accumulator buffers [D_h | D_l] of N columns each, then A: plane h (64 columns of
    // 4 int8 weights), plane l (64)
    static constexpr uint32_t acc = 2 * N;
    static constexpr int NBUF = (512 - 128) / acc > 4 ? 4 : (512 - 128) / acc;
    static constexpr uint32_t a = NBUF * acc;
    static_assert(NP % NPP == 0, "sequence group");
    static_assert(a + 128 <= 512, "TMEM columns");
};

struct Q6State {
    uint64_t raw_full[kQ6RawStages], raw_empty[kQ6RawStages], b_full[kQ6BStagesMax], b_empty[kQ6BStagesMax];
    uint64_t a_full[4], a_empty[4], acc_full[4], acc_empty[4], mma_done;
    uint32_t tmem_base;
    volatile int abort;
    int mcount;               // row tiles this CTA finished last (merged after its units)
    int mlist[kTcMergeCap];
    alignas(16) float ys[8][2][32];  // per epilogue warp: activation block scales of its sequences (all passes), by block parity
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

// 4 quants q (bytes of qb, 0..63) of one sub-block with scale sc -> the int8 columns of the two
// weight planes: v = sc*(q-32) = 64*h + l.  u = v + 4096 in [32, 8192] is formed in two 16-bit
// lanes per word (exact: each lane's value is non-negative and below 2^16).
__device__ __forceinline__ void q6_planes(uint32_t qb, int sc, uint32_t &h, uint32_t &l) {
    const uint32_t C = (uint32_t)(4096 - 32 * sc) * 0x00010001u;
    const uint32_t u0 = (qb & 0x00FF00FFu) * (uint32_t)sc + C;         // quants 0, 2
    const uint32_t u1 = ((qb >> 8) & 0x00FF00FFu) * (uint32_t)sc + C;  // quants 1, 3
    h = __vsub4(((u0 >> 6) & 0x00FF00FFu) | (((u1 >> 6) & 0x00FF00FFu) << 8), 0x40404040u);
    l = (u0 & 0x003F003Fu) | ((u1 & 0x003F003Fu) << 8);
}

// The K slices of row `row` for this thread's sequences, summed in slice order (0 + P0 + P1 ...).
template <int SP>
__device__ __forceinline__ void q6_merge_rows(const TcArgs &a, int NP, int NPASS, int NPP, int p, int row) {
    if (row >= a.rows) return;
    const size_t rows = (size_t)a.rows;
    for (int ps = 0; ps < NPASS; ps++) {
        const int s0 = ps * NPP + p * SP;
        if (s0 >= a.B) break;
        float v[SP];
        slot_sums<SP>(a.part + (size_t)s0 * rows + row, (size_t)NP * rows, rows, a.ksplit, v);
#pragma unroll
        for (int s = 0; s < SP; s++)
            if (s0 + s < a.B) a.out[(size_t)(s0 + s) * a.ldo + row] = v[s];
    }
}

template <int NP>
__global__ void __launch_bounds__(kQ6Threads, 1) gemm_q6tc_kernel(const __grid_constant__ Q6Maps maps, TcArgs a) {
    using CF = Q6Cfg<NP>;
    constexpr int RAW = CF::raw, BST = CF::bst, BS = CF::BS, RS = kQ6RawStages;
    static_assert(CF::total + sizeof(Q6State) <= 227 * 1024, "shared memory per CTA");
    constexpr int NPP = CF::NPP, NPASS = CF::NPASS, N = CF::N, SP = CF::SP;
    extern __shared__ uint8_t smem_dyn[];
    __shared__ Q6State S;
    uint8_t *smem = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
    uint8_t *raw = smem, *bst = smem + CF::b_off;
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
        for (int i = 0; i < CF::NBUF; i++) {
            mbar_init(&S.acc_full[i], 1);
            mbar_init(&S.acc_empty[i], 8);
        }
        mbar_init(&S.mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.abort = 0;
        S.mcount = 0;
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
            constexpr uint32_t idesc = umma_idesc(2, 1, 1, N);  // s32 += s8 * s8, N = 3 * NPP
            int i = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
                const int b0 = (u % a.ksplit) * a.kslice, b1 = min(a.nb, b0 + a.kslice);
                for (int b = b0; b < b1 && ok; b++, i++) {
                    const int bs = i % BS;
                    if (!q6_wait(S, &S.b_full[bs], (i / BS) & 1)) { ok = false; break; }
                    const uint32_t bsa = smem_u32(bst + bs * BST);
                    for (int ps = 0; ps < NPASS && ok; ps++) {
                        const int it = i * NPASS + ps, buf = it % CF::NBUF;
                        if (!q6_wait(S, &S.acc_empty[buf], ((it / CF::NBUF) & 1) ^ 1)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t dh = tbase + buf * CF::acc, dl = dh + N;
                        for (int qi = 0; qi < 4; qi++) {
                            const int q = ((qi & 1) << 1) | (qi >> 1);  // 0, 2, 1, 3: the order the expand warps finish
                            if (ps == 0) {
                                if (!mbar_try_wait(&S.a_full[q], i & 1) && !q6_wait(S, &S.a_full[q], i & 1)) { ok = false; break; }
                                tc_fence_after();
                            }
#pragma unroll
                            for (int ks = 0; ks < 2; ks++) {
                                const uint64_t bd = umma_desc(bsa + (4 * q + 2 * ks) * (3 * NP * 16) + ps * N * 16,
                                                              3 * NP * 16, 128);
                                const uint32_t acc = (qi | ks) != 0;
                                tc_mma_i8_ts(dh, tbase + CF::a + 16 * q + 8 * ks, bd, idesc, acc);
                                tc_mma_i8_ts(dl, tbase + CF::a + 64 + 16 * q + 8 * ks, bd, idesc, acc);
                            }
                            if (ps == NPASS - 1) tc_commit(&S.a_empty[q]);
                        }
                        if (!ok) break;
                        tc_commit(&S.acc_full[buf]);
                    }
                    if (!ok) break;
                    tc_commit(&S.b_empty[bs]);
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
                    // quarter q = weights 128e + 64qq + [0, 64): column c' = 8t' + w holds weights l = 4w..4w+3 of
                    // group t = 2qq + t' (quant from ql[l + 32t'], low nibble for qq 0 / high for qq 1, bits 2t of
                    // qh[l], scale sc[l/16 + 2t])
                    const int q = 2 * e + qq;
                    if (!q6_wait(S, &S.a_empty[q], (i & 1) ^ 1)) { ok = false; break; }
                    uint32_t ch[16], cl[16];
#pragma unroll
                    for (int cc = 0; cc < 16; cc++) {
                        const int tp = cc >> 3, w = cc & 7, t = 2 * qq + tp;
                        const uint32_t lw = ql[w + 8 * tp];
                        const uint32_t qb = ((qq ? (lw >> 4) : lw) & 0x0F0F0F0Fu) | (((qh[w] >> (2 * t)) & 0x03030303u) << 4);
                        const int sidx = (w >> 2) + 2 * t;
                        const int sc = (int)(int8_t)(((sidx < 4 ? sw0 : sw1) >> (8 * (sidx & 3))) & 0xffu);
                        q6_planes(qb, sc, ch[cc], cl[cc]);
                    }
                    tc_st16(tl + CF::a + 16 * q, ch);
                    tc_st16(tl + CF::a + 64 + 16 * q, cl);
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
        float P[NPASS][SP];
#pragma unroll
        for (int ps = 0; ps < NPASS; ps++)
#pragma unroll
            for (int s = 0; s < SP; s++) P[ps][s] = 0.0f;
        int i = 0;
        bool ok = true;
        // final value v of sequence seq for row `row`
        auto emit = [&](int row, int seq, float v, unsigned long long &key) {
            if (a.epi == EPI_SOFTCAP_ARGMAX) {  // logits softcap (main.c:1780-1796), then argmax over rows
                if (a.cap > 0.0f) v = a.cap * tanhf(v / a.cap);
                key = row < a.rows ? argmax_key(v, row) : 0ull;
                if (!a.out) return;
            }
            if (row < a.rows && seq < a.B) a.out[(size_t)seq * a.ldo + row] = v;
        };
        auto finish = [&](int u) {  // end of this CTA's K slice of a row tile: final values or the slice's partial
            const int ks = u % a.ksplit, row = (u / a.ksplit) * 128 + r;
#pragma unroll
            for (int ps = 0; ps < NPASS; ps++)
#pragma unroll
                for (int s = 0; s < SP; s++) {
                    const int seq = ps * NPP + p * SP + s;
                    if (a.ksplit == 1) {
                        unsigned long long key = 0ull;
                        emit(row, seq, P[ps][s], key);
                        if (a.epi == EPI_SOFTCAP_ARGMAX) {
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) {
                                const unsigned long long t = __shfl_xor_sync(0xffffffffu, key, o);
                                key = t > key ? t : key;
                            }
                            if (lane == 0 && seq < a.B && key) atomicMax(a.keys + seq, key);
                        }
                    } else if (row < a.rows) {  // all NP slots of the partial exist: no per-sequence bound
                        a.part[((size_t)ks * NP + seq) * a.rows + row] = P[ps][s];
                    }
                    P[ps][s] = 0.0f;
                }
            if (a.ksplit > 1 && a.tickets) {
                // Count this slice in; the CTA that completes the row tile merges it after its units.
                __threadfence();
                asm volatile("bar.sync 1, 256;" ::: "memory");  // the 8 epilogue warps
                if (warp == 10 && lane == 0) {
                    const int rt = u / a.ksplit;
                    if (atomicAdd(a.tickets + rt, 1) == a.ksplit - 1) {
                        if (S.mcount < kTcMergeCap) S.mlist[S.mcount++] = rt;
                        else if (a.err) atomicExch(a.err, G4_ERR_STATE);
                    }
                }
            }
        };
        int u = blockIdx.x, b = u < a.units ? (u % a.ksplit) * a.kslice : 0;
        // d of row r for the block (fp16 after the quant planes of the row), loaded one block ahead
        auto fetch_d = [&](int uu, int bb) -> uint16_t {
            const int row = (uu / a.ksplit) * 128 + r;
            return row < a.rows ? __ldg(reinterpret_cast<const uint16_t *>(a.w + (size_t)row * a.row_bytes + (size_t)a.nb * 208) + bb)
                                : (uint16_t)0;
        };
        // activation block scales of this warp's sequences for block bb, both passes (lane < SP: pass 0,
        // lane - SP: pass 1), loaded one block ahead
        auto fetch_ys = [&](int bb) -> float {
            const int ps = lane / SP, l = lane % SP;
            return ps < NPASS ? __ldg(a.yd + (size_t)bb * NP + ps * NPP + p * SP + l) : 0.0f;
        };
        uint16_t nhd = u < a.units ? fetch_d(u, b) : (uint16_t)0;
        float nys = u < a.units ? fetch_ys(b) : 0.0f;
        while (u < a.units && ok) {
            const int b1 = min(a.nb, (u % a.ksplit) * a.kslice + a.kslice);
            const float dw = f16_to_f32(nhd);
            if (lane < NPASS * SP) S.ys[pw][i & 1][lane] = nys;
            __syncwarp();
            int nu = u, nbk = b + 1;
            if (nbk >= b1) { nu = u + gridDim.x; nbk = nu < a.units ? (nu % a.ksplit) * a.kslice : 0; }
            if (nu < a.units) { nhd = fetch_d(nu, nbk); nys = fetch_ys(nbk); }
#pragma unroll
            for (int ps = 0; ps < NPASS; ps++) {
                const int it = i * NPASS + ps, buf = it % CF::NBUF;
                if (!q6_wait(S, &S.acc_full[buf], (it / CF::NBUF) & 1)) { ok = false; break; }
                tc_fence_after();
                const float *yv = S.ys[pw][i & 1] + ps * SP;
                const uint32_t col = tl + buf * CF::acc + p * SP;
#pragma unroll
                for (int c = 0; c < SP / 8; c++) {
                    uint32_t h0[8], h1[8], h2[8], l0[8], l1[8], l2[8];
                    tc_ld8(col + 8 * c, h0);
                    tc_ld8(col + NPP + 8 * c, h1);
                    tc_ld8(col + 2 * NPP + 8 * c, h2);
                    tc_ld8(col + N + 8 * c, l0);
                    tc_ld8(col + N + NPP + 8 * c, l1);
                    tc_ld8(col + N + 2 * NPP + 8 * c, l2);
                    tc_wait_ld();
                    if (c == SP / 8 - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&S.acc_empty[buf]);
                    }
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        const float dot = q6x_dot(64 * (int)h0[k] + (int)l0[k], 64 * (int)h1[k] + (int)l1[k],
                                                  64 * (int)h2[k] + (int)l2[k]);
                        P[ps][8 * c + k] = __fmaf_rn(dot, __fmul_rn(dw, yv[8 * c + k]), P[ps][8 * c + k]);
                    }
                }
            }
            if (!ok) break;
            if (nu != u) finish(u);
            u = nu; b = nbk; i++;
        }
        if (!ok) {
            q6_fail(S, a.err);
        } else if (a.ksplit > 1 && a.tickets) {
            asm volatile("bar.sync 1, 256;" ::: "memory");  // S.mlist complete
            const int nm = S.mcount;
            if (nm) __threadfence();
            for (int m = 0; m < nm; m++) q6_merge_rows<SP>(a, NP, NPASS, NPP, p, S.mlist[m] * 128 + r);
            if (warp == 10 && lane < nm) a.tickets[S.mlist[lane]] = 0;  // ready for the next launch
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tc_dealloc(tbase, 512);
    }
}

// B operand of gemm_q6tc (tc6_store_block layout) from fp32 activations.
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

RowOrder q6_row_order(int rows, int n, int nsm, bool argmax) {
    if (argmax) return RowOrder{0, 0, 0};  // the argmax epilogue keeps whole rows in one CTA
    const TcPlan p = tc_plan(rows, n / G4_QK, nsm);
    return RowOrder{0, 0, p.ksplit > 1 ? p.kslice : 0};
}

size_t tc6_operand_bytes(int n) { return (size_t)(n / G4_QK) * (768 * 64 + 64 * 4); }
size_t tc6_ys_offset(int n) { return (size_t)(n / G4_QK) * 768 * 64; }

int launch_tc6_split(const float *x, int ldx, int B, int n, int np, uint8_t *bq, float *ys, cudaStream_t st) {
    if (n % G4_QK || (ldx % 4) || ((uintptr_t)x & 15u)) { set_error(G4_ERR_ARG, "tc6 split: bad shape/alignment"); return G4_ERR_ARG; }
    G4_CUDA(launch_pdl(tc6_split_kernel, dim3(n / G4_QK, np / 8), dim3(256), 0, st, x, ldx, B, np, bq, ys));
    G4_LAUNCHED();
    return G4_OK;
}

int launch_gemm_q6tc(const void *maps, const void *w, int n, int rows, const uint8_t *bq, const float *ys, int B,
                     int np, float *out, int ldo, float *part, size_t part_bytes, int *err, int nsm,
                     int epi, float cap, unsigned long long *keys, cudaStream_t st, int *tickets) {
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
    // in-kernel merges: a CTA keeps at most kTcMergeCap row tiles to merge (one per unit it runs)
    if (tickets && (p.units + p.grid - 1) / p.grid > kTcMergeCap) tickets = nullptr;
    TcArgs a{(const uint8_t *)w, device_row_bytes(G4_Q6_K, n), bq, ys, out, part, err, nb, rows, B, ldo,
             p.ksplit, p.kslice, p.units, epi, cap, keys};
    a.tickets = tickets;
#define G4_Q6TC_CASE(N)                                                                             \
    if (np == N) {                                                                                   \
        const size_t smem = Q6Cfg<N>::total;                                                         \
        G4_CUDA(launch_pdl(gemm_q6tc_kernel<N>, dim3(p.grid), dim3(kQ6Threads), smem, st, *(const Q6Maps *)maps, a)); \
    }
    G4_Q6TC_CASE(16) else G4_Q6TC_CASE(32) else G4_Q6TC_CASE(64)
#undef G4_Q6TC_CASE
    G4_LAUNCHED();
    if (p.ksplit > 1 && !tickets) return launch_tc_merge(part, p.ksplit, np, rows, B, out, ldo, EPI_STORE, nullptr, 0, st);
    return G4_OK;
}

int prime_tc6_attrs() {
    G4_CUDA(cudaFuncSetAttribute(q6tc_kernel_ptr<16>(), cudaFuncAttributeMaxDynamicSharedMemorySize, Q6Cfg<16>::total));
    G4_CUDA(cudaFuncSetAttribute(q6tc_kernel_ptr<32>(), cudaFuncAttributeMaxDynamicSharedMemorySize, Q6Cfg<32>::total));
    G4_CUDA(cudaFuncSetAttribute(q6tc_kernel_ptr<64>(), cudaFuncAttributeMaxDynamicSharedMemorySize, Q6Cfg<64>::total));
    return G4_OK;
}

}  // namespace g4
