// k_gemm_bf16tc.cu — batched BF16-weight GEMM on the tensor cores for the
// per-layer-embedding projections of the batched decode step (inp_gate,
// proj, ple_proj stored as BF16 in the Q4_K_M mix).
//
// The reference's BF16 rows are an fp32 dot against the fp32 activation,
// v += x[j] * bf16_to_f32(w[j]) (mm_bf16, gemma4-4b/cpu-blas/main.c:
// 1520-1537).  Here x is split into three bf16 parts, x = x1 + x2 + x3 to
// 2^-24 relative (each remainder is exact in fp32), stacked as 3*NP rows of
// the MMA B operand; every bf16 x bf16 product is exact in fp32 and the
// three column blocks of the fp32 accumulator are added in the epilogue.
//
// The weights need no expansion: a three-dimensional tensor map (k within a
// 16-byte chunk, row, chunk) lands a 128-row x 64-weight tile in shared
// memory directly in the K-major core-matrix layout (chunk-major, 16 bytes
// per row), and the MMA reads A and B from shared memory.  Warp 0 issues the
// copies, warp 1 the MMAs, warps 2..5 (one per TMEM lane quadrant) run the
// epilogue; work units are (128-row tile, K-slice) with the slice partials
// summed in slice order by the last warp to finish.  Waits are bounded (2 s).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <math.h>

#include <algorithm>

#include "g4_async.cuh"
#include "g4_internal.cuh"
#include "g4_kernels.cuh"
#include "g4_tc.cuh"

namespace g4 {

namespace {

constexpr int kBfThreads = 192;  // producer, MMA, 4 epilogue warps
constexpr int kBfStages = 4;

template <int NP>
struct BfSmem {
    static constexpr int a = 128 * kBfK * 2;        // 16 KB
    static constexpr int b = 3 * NP * kBfK * 2;     // x1|x2|x3
    static constexpr int stage = a + b;
    static constexpr int total = kBfStages * stage + 1024;
};

struct BfState {
    uint64_t full[kBfStages], empty[kBfStages], acc_full[2], acc_empty[2], mma_done;
    uint32_t tmem_base;
    volatile int abort;
};

__device__ __forceinline__ bool bf_wait(BfState &S, uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
        if (S.abort) return false;
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
}
__device__ __forceinline__ void bf_fail(BfState &S, int *err) {
    S.abort = 1;
    if (err) atomicExch(err, G4_ERR_TIMEOUT);
}

__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)) : "memory");
}

// Epilogue inputs beyond TcArgs (a.nb counts 64-weight K groups here).
struct BfExtra {
    const float *evec;  // EPI_GELU_SCALE: out = gelu(acc) * evec[s*ld_evec + row]
    int ld_evec;
};

template <int NP>
__global__ void __launch_bounds__(kBfThreads, 1) gemm_bf16tc_kernel(const __grid_constant__ CUtensorMap tmw, TcArgs a,
                                                                    BfExtra ex) {
    constexpr int ST = BfSmem<NP>::stage, SA = BfSmem<NP>::a, SB = BfSmem<NP>::b, N3 = 3 * NP;
    constexpr int ACC = N3 <= 128 ? 128 : 256;  // TMEM columns per accumulator buffer (>= 3*NP)
    extern __shared__ uint8_t smem_dyn[];
    __shared__ BfState S;
    uint8_t *smem = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_trigger();
    if (tid == 0) {
        for (int i = 0; i < kBfStages; i++) {
            mbar_init(&S.full[i], 1);
            mbar_init(&S.empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&S.acc_full[i], 1);
            mbar_init(&S.acc_empty[i], 4);
        }
        mbar_init(&S.mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.abort = 0;
    }
    if (warp == 1) tc_alloc(&S.tmem_base, 2 * ACC);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = S.tmem_base;

    if (warp == 0) {
        if (lane == 0) {  // ------------------------------------------------ producer
            int i = 0;
            bool ok = true, dep = false;
            for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
                const int rt = u / a.ksplit, g0 = (u % a.ksplit) * a.kslice, g1 = min(a.nb, g0 + a.kslice);
                for (int g = g0; g < g1; g++, i++) {
                    const int st = i % kBfStages;
                    if (!bf_wait(S, &S.empty[st], ((i / kBfStages) & 1) ^ 1)) { ok = false; break; }
                    uint8_t *dst = smem + st * ST;
                    mbar_expect_tx(&S.full[st], ST);
                    tma_load_3d(dst, &tmw, 0, rt * 128, g * (kBfK / 8), &S.full[st]);
                    if (!dep) { pdl_wait(); dep = true; }
                    bulk_g2s(dst + SA, a.bq + (size_t)g * SB, SB, &S.full[st]);
                }
            }
            if (!dep) pdl_wait();
            if (!ok) {
                bf_fail(S, a.err);
                for (int k = max(0, i - kBfStages); k < i; k++) {
                    const unsigned long long t0 = global_ns();
                    while (!mbar_try_wait(&S.full[k % kBfStages], (k / kBfStages) & 1) && global_ns() - t0 < kWaitLimitNs) {}
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ------------------------------------------------ MMA issuer
            constexpr uint32_t idesc = umma_idesc(1, 1, 1, N3);  // f32 += bf16 * bf16
            int i = 0, t = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x, t++) {
                const int g0 = (u % a.ksplit) * a.kslice, g1 = min(a.nb, g0 + a.kslice);
                const int abuf = t & 1;
                if (!bf_wait(S, &S.acc_empty[abuf], ((t >> 1) & 1) ^ 1)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tbase + abuf * ACC;
                for (int g = g0; g < g1; g++, i++) {
                    const int st = i % kBfStages;
                    if (!bf_wait(S, &S.full[st], (i / kBfStages) & 1)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + st * ST), sb = sa + SA;
#pragma unroll
                    for (int ks = 0; ks < kBfK / 16; ks++)
                        tc_mma_f16(d, umma_desc(sa + 2 * ks * 2048, 2048, 128),
                                   umma_desc(sb + 2 * ks * N3 * 16, N3 * 16, 128), idesc, (g > g0 || ks > 0) ? 1u : 0u);
                    tc_commit(&S.empty[st]);
                }
                if (!ok) break;
                tc_commit(&S.acc_full[abuf]);
            }
            if (!ok) bf_fail(S, a.err);
            tc_commit(&S.mma_done);
            const unsigned long long t0 = global_ns();
            while (!mbar_try_wait(&S.mma_done, 0) && global_ns() - t0 < kWaitLimitNs) {}
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- epilogue: rows 32*quad + lane
        const int quad = warp & 3, r = 32 * quad + lane;
        const uint32_t tl = tbase + ((uint32_t)(32 * quad) << 16);
        pdl_wait();
        int t = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x, t++) {
            const int rt = u / a.ksplit, ks = u % a.ksplit, row = rt * 128 + r;
            const int abuf = t & 1;
            if (!bf_wait(S, &S.acc_full[abuf], (t >> 1) & 1)) { ok = false; break; }
            tc_fence_after();
            float *dst = a.ksplit == 1 ? a.out : a.part + (size_t)ks * NP * a.rows;
            const size_t ld = a.ksplit == 1 ? (size_t)a.ldo : (size_t)a.rows;
            const bool final_now = a.ksplit == 1;
#pragma unroll 1
            for (int c = 0; c < NP / 8; c++) {
                uint32_t v1[8], v2[8], v3[8];
                tc_ld8(tl + abuf * ACC + 8 * c, v1);
                tc_ld8(tl + abuf * ACC + NP + 8 * c, v2);
                tc_ld8(tl + abuf * ACC + 2 * NP + 8 * c, v3);
                tc_wait_ld();
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int seq = 8 * c + k;
                    float v = __uint_as_float(v1[k]) + __uint_as_float(v2[k]) + __uint_as_float(v3[k]);
                    if (seq < a.B && row < a.rows) {
                        if (final_now && a.epi == EPI_GELU_SCALE) {
                            v = gelu_f32(v) * ex.evec[(size_t)seq * ex.ld_evec + row];
                        }
                        dst[(size_t)seq * ld + row] = v;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.acc_empty[abuf]);
            (void)rt;  // split tiles: the partials are summed by tc_merge_kernel
        }
        if (!ok) bf_fail(S, a.err);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tc_dealloc(tbase, 2 * ACC);
    }
}

// B operand for K group g (64 weights) of gemm_bf16tc: rows x1 (0..NP-1),
// x2 (NP..2NP-1), x3 (2NP..3NP-1) of every sequence as bf16, K-major core
// matrices: byte (k/8)*(3*NP*16) + row*16 + (k%8)*2.  grid (n/64, NP/8),
// 256 threads: warp w handles sequence 8*blockIdx.y + w, lane l weights 2l, 2l+1.
__global__ void bf3_split_kernel(const float *__restrict__ x, int ldx, int B, int NP, uint8_t *__restrict__ bq) {
    pdl_trigger();
    pdl_wait();
    const int g = blockIdx.x, lane = threadIdx.x & 31, s = blockIdx.y * 8 + (threadIdx.x >> 5);
    float v0 = 0.0f, v1 = 0.0f;
    if (s < B) {
        const float2 t = *reinterpret_cast<const float2 *>(x + (size_t)s * ldx + (size_t)g * kBfK + 2 * lane);
        v0 = t.x;
        v1 = t.y;
    }
    bf3_store_group(bq, g, NP, s, lane, v0, v1);
}

template <int NP>
void *bf16tc_kernel_ptr() { return (void *)gemm_bf16tc_kernel<NP>; }

PFN_cuTensorMapEncodeTiled_v12000 g_enc_bf = nullptr;

}  // namespace

size_t bf16tc_operand_bytes(int n) { return (size_t)(n / kBfK) * 3 * 64 * kBfK * 2; }

// 3-D view of a [rows][n] bf16 matrix: (k within a 16-byte chunk, row, chunk).
int bf16tc_weight_map(CUtensorMap *m, const void *w, int n, int rows) {
    if (!g_enc_bf) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        G4_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn) { set_error(G4_ERR_CUDA, "cuTensorMapEncodeTiled not available"); return G4_ERR_CUDA; }
        g_enc_bf = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }
    if (n % kBfK || ((uintptr_t)w & 15u)) { set_error(G4_ERR_ARG, "bf16 tc: n %% 64 or alignment"); return G4_ERR_ARG; }
    const cuuint64_t dims[3] = {8, (cuuint64_t)rows, (cuuint64_t)(n / 8)};
    const cuuint64_t strides[2] = {(cuuint64_t)n * 2, 16};
    const cuuint32_t box[3] = {8, 128, kBfK / 8}, es[3] = {1, 1, 1};
    const CUresult rc = g_enc_bf(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void *>(w), dims, strides, box, es,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) { set_error(G4_ERR_CUDA, "cuTensorMapEncodeTiled (bf16) failed (%d)", (int)rc); return G4_ERR_CUDA; }
    return G4_OK;
}

int launch_bf3_split(const float *x, int ldx, int B, int n, int np, uint8_t *bq, cudaStream_t st) {
    if (n % kBfK || (ldx % 2) || ((uintptr_t)x & 7u)) { set_error(G4_ERR_ARG, "bf3 split: bad shape/alignment"); return G4_ERR_ARG; }
    G4_CUDA(launch_pdl(bf3_split_kernel, dim3(n / kBfK, np / 8), dim3(256), 0, st, x, ldx, B, np, bq));
    G4_LAUNCHED();
    return G4_OK;
}

int launch_gemm_bf16tc(const CUtensorMap *tm, int n, int rows, const uint8_t *bq, int B, int np, float *out, int ldo,
                       float *part, size_t part_bytes, int *err, int nsm, int epi, const float *evec,
                       int ld_evec, cudaStream_t st) {
    if (B < 1 || B > np || (np != 16 && np != 32 && np != 64)) { set_error(G4_ERR_ARG, "bf16 tc gemm: batch %d / %d", B, np); return G4_ERR_ARG; }
    if (epi != EPI_STORE && epi != EPI_GELU_SCALE) { set_error(G4_ERR_ARG, "bf16 tc gemm: epilogue %d", epi); return G4_ERR_ARG; }
    const int ng = n / kBfK;
    // K-split so that about one CTA per SM has work; split tiles go through bf16_merge_kernel
    const int tiles = (rows + 127) / 128;
    int ksplit = std::max(1, std::min(ng, nsm / tiles));
    const int kslice = (ng + ksplit - 1) / ksplit;
    ksplit = (ng + kslice - 1) / kslice;
    if (ksplit > 1 && (size_t)ksplit * np * rows * sizeof(float) > part_bytes) ksplit = 1;
    const TcPlan p{ksplit, ksplit > 1 ? kslice : ng, tiles * ksplit, std::min(tiles * ksplit, nsm)};
    TcArgs a{nullptr, 0, bq, nullptr, out, part, err, ng, rows, B, ldo, p.ksplit, p.kslice, p.units, epi, 0.0f,
             nullptr};
    const BfExtra ex{evec, ld_evec};
#define G4_BFTC_CASE(N)                                                                                        \
    if (np == N) G4_CUDA(launch_pdl(gemm_bf16tc_kernel<N>, dim3(p.grid), dim3(kBfThreads), (size_t)BfSmem<N>::total, st, \
                                    *tm, a, ex));
    G4_BFTC_CASE(16) else G4_BFTC_CASE(32) else G4_BFTC_CASE(64)
#undef G4_BFTC_CASE
    G4_LAUNCHED();
    if (p.ksplit > 1) return launch_tc_merge(part, p.ksplit, np, rows, B, out, ldo, epi, evec, ld_evec, st);
    return G4_OK;
}

int prime_bf16tc_attrs() {
    G4_CUDA(cudaFuncSetAttribute(bf16tc_kernel_ptr<16>(), cudaFuncAttributeMaxDynamicSharedMemorySize, BfSmem<16>::total));
    G4_CUDA(cudaFuncSetAttribute(bf16tc_kernel_ptr<32>(), cudaFuncAttributeMaxDynamicSharedMemorySize, BfSmem<32>::total));
    G4_CUDA(cudaFuncSetAttribute(bf16tc_kernel_ptr<64>(), cudaFuncAttributeMaxDynamicSharedMemorySize, BfSmem<64>::total));
    return G4_OK;
}

}  // namespace g4
