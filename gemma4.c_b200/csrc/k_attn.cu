// k_attn.cu — ISWA decode attention with Neox RoPE and shared KV.
//
// Reference: the attention block of forward (gemma4-4b/cpu-blas/main.c:
// 1878-1950): q/k per-head RMSNorm (1458-1466), v RMSNorm without weight
// (1468-1476), Neox RoPE (1725-1745), KV store (1901-1904), the window
// t_start = max(0, pos+1-window) for sliding-window layers (1909-1915), and per
// q head h: scores over the kv head h/(n_heads/n_kv) rows of the source
// layer's cache (scale 1), max-subtracted softmax (1478-1488) and the
// probability-weighted sum of V rows.  Layers >= 24 read layer 22 (sliding)
// or 23 (global) and store nothing (main.c:739-746).
//
// Device layout of a KV layer: K and V each [B][n_kv][slots][hd] fp32, where
// slots = the window (ring buffer, slot = pos % window) for sliding-window
// layers and max_seq (slot = pos) for global ones.  A ring reads the same
// logical rows in the same logical order as the reference's linear cache.
//
// One kernel, attn_fused_kernel: split-K flash-decoding where a CTA owns
// (chunk of 32 positions, kv head, sequence) and all G query heads of that
// kv head, so each K/V row is read from HBM once per step; the q/k norms,
// RoPE and the KV append run in the same CTA, and the chunk partials (max,
// sum, unnormalised output) are merged by the last CTA to finish.
// The position is read from device memory so one CUDA graph serves all
// positions; the grid covers the largest window and idle chunks exit.
#include <algorithm>
#include <math.h>

#include "g4_async.cuh"
#include "g4_internal.cuh"
#include "g4_kernels.cuh"
#include "g4_quant.cuh"
#include "g4_tc.cuh"

namespace g4 {

constexpr int kChunk = 32;  // positions per CTA (8 warps x 4 rows, loads issued together)
constexpr int kMaxWts = 512;  // chunk weights kept in shared memory by the merging CTA
int attn_chunk_size() { return kChunk; }

// Reference-exact RoPE angles (apply_rope_neox, main.c:1725-1745): theta
// starts at pos and is multiplied by theta_scale = powf(base, -2/n_rot) once
// per pair; angle = freq_scale * theta / ff[j].  cosf/sinf/powf are the host
// libm's, as in the reference, so the table matches it bit for bit.
void rope_table_host(float2 *out, int npos, int n_rot, float base, float freq_scale, const float *ff) {
    const float theta_scale = powf(base, -2.0f / (float)n_rot);
    const int half = n_rot / 2;
    for (int p = 0; p < npos; p++) {
        float theta = (float)p;
        for (int j = 0; j < half; j++) {
            const float f = ff ? ff[j] : 1.0f;
            const float angle = freq_scale * theta / f;
            out[(size_t)p * half + j] = make_float2(cosf(angle), sinf(angle));
            theta *= theta_scale;
        }
    }
}

template <int EPL>
__device__ __forceinline__ void load_row(float (&dst)[EPL], const float *src) {
    if constexpr (EPL % 4 == 0) {
#pragma unroll
        for (int e = 0; e < EPL; e += 4) {
            const float4 a = *reinterpret_cast<const float4 *>(src + e);
            dst[e] = a.x; dst[e + 1] = a.y; dst[e + 2] = a.z; dst[e + 3] = a.w;
        }
    } else {
#pragma unroll
        for (int e = 0; e < EPL; e += 2) {
            const float2 a = *reinterpret_cast<const float2 *>(src + e);
            dst[e] = a.x; dst[e + 1] = a.y;
        }
    }
}

// Per-head RMSNorm (+ weight) and Neox RoPE of one head vector by one warp
// (main.c:1458-1476, 1725-1745).  Lane l holds elements l + 32 i, so the RoPE
// partner j + hd/2 of element j sits in the same lane.  Writes dst[hd].
// Element e of a lane's share of a row in the streaming kernel: vectors of V
// floats, lane-interleaved (lane l holds [V*l, V*l+V), [32V + V*l, ...), ...),
// so every vector load of a warp reads one contiguous span of shared memory
// (no bank conflicts).
template <int EPL>
__device__ __forceinline__ int row_elem(int lane, int e) {
    constexpr int V = EPL % 4 == 0 ? 4 : 2;
    return V * lane + 32 * V * (e / V) + e % V;
}
template <int EPL>
__device__ __forceinline__ void load_row_il(float (&dst)[EPL], const float *row, int lane) {
    if constexpr (EPL % 4 == 0) {
#pragma unroll
        for (int e = 0; e < EPL; e += 4) {
            const float4 a = *reinterpret_cast<const float4 *>(row + row_elem<EPL>(lane, e));
            dst[e] = a.x; dst[e + 1] = a.y; dst[e + 2] = a.z; dst[e + 3] = a.w;
        }
    } else {
#pragma unroll
        for (int e = 0; e < EPL; e += 2) {
            const float2 a = *reinterpret_cast<const float2 *>(row + row_elem<EPL>(lane, e));
            dst[e] = a.x; dst[e + 1] = a.y;
        }
    }
}

template <int EPL>
__device__ __forceinline__ void warp_norm_rope(const float *src, const float *w, const float2 *cs, int n_rot, float eps,
                                               float *dst, float *dst2) {
    constexpr int HD = EPL * 32;
    const int lane = threadIdx.x & 31;
    float v[EPL];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < EPL; i++) {
        v[i] = src[lane + 32 * i];
        ss = fmaf(v[i], v[i], ss);
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)HD + eps);
#pragma unroll
    for (int i = 0; i < EPL; i++) v[i] = w ? v[i] * (inv * w[lane + 32 * i]) : v[i] * inv;
    if (cs) {
#pragma unroll
        for (int i = 0; i < EPL / 2; i++) {
            const int j = lane + 32 * i;
            if (j < n_rot / 2) {  // products rounded separately like the reference
                const float2 c = cs[j];
                const float v0 = v[i], v1 = v[i + EPL / 2];
                v[i] = __fsub_rn(__fmul_rn(v0, c.x), __fmul_rn(v1, c.y));
                v[i + EPL / 2] = __fadd_rn(__fmul_rn(v0, c.y), __fmul_rn(v1, c.x));
            }
        }
    }
#pragma unroll
    for (int i = 0; i < EPL; i++) {
        dst[lane + 32 * i] = v[i];
        if (dst2) dst2[lane + 32 * i] = v[i];
    }
}

// Head dims up to 256 stage the chunk's K and V rows in shared memory with
// bulk copies (TMA) issued at CTA start, so the score and P.V phases do not
// each wait for HBM; head dim 512 loads rows into registers.
template <int EPL>
constexpr bool attn_tma() { return EPL <= 8; }

template <int EPL, int G>
constexpr size_t attn_smem_bytes() {
    return sizeof(float) * ((size_t)G * EPL * 32 + (size_t)8 * G * EPL * 32 + (size_t)G * kChunk + 2 * G +
                            2 * (size_t)EPL * 32 + (size_t)G * kMaxWts +
                            (attn_tma<EPL>() ? (size_t)2 * kChunk * EPL * 32 : 0));
}

// One CTA per (chunk of 32 positions, kv head, sequence), all G query heads
// of the kv head: q-norm + RoPE of the G heads; on the chunk holding `pos`
// of a layer that stores KV, k-norm + RoPE and v-norm of the new row, written
// to the cache slot; scores, chunk softmax statistics and the unnormalised
// P.V; then the last CTA of the (kv head, sequence) to finish (atomic ticket,
// no waiting) merges the chunk partials into qo.
template <int EPL, int G>
__global__ void __launch_bounds__(256) attn_fused_kernel(AttnLayer L, const int *__restrict__ pos_dev) {
    constexpr int HD = EPL * 32;
    extern __shared__ __align__(16) float dsm[];
    float(*qs)[HD] = reinterpret_cast<float(*)[HD]>(dsm);                       // [G][HD]
    float(*red)[G][HD] = reinterpret_cast<float(*)[G][HD]>(dsm + G * HD);       // [8][G][HD]
    float(*sc)[kChunk] = reinterpret_cast<float(*)[kChunk]>(dsm + 9 * G * HD);  // [G][kChunk]
    float(*ml)[2] = reinterpret_cast<float(*)[2]>(dsm + 9 * G * HD + G * kChunk);
    float *knew = dsm + 9 * G * HD + G * kChunk + 2 * G;                        // [HD]
    float *vnew = knew + HD;                                                    // [HD]
    float *wts = vnew + HD;                                                     // [G][kMaxWts] combine weights
    float *kbuf = wts + G * kMaxWts;                                            // [kChunk][HD] (TMA staging)
    float *vbuf = kbuf + kChunk * HD;                                           // [kChunk][HD]
    __shared__ int ticket;
    __shared__ __align__(8) uint64_t kvbar;
    pdl_trigger();
    pdl_wait();
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = L.row_pos ? L.row_pos[b] : *pos_dev;
    const int cb = L.row_seq ? L.row_seq[b] : b;  // cache sequence of this query row
    int t0 = 0;
    if (L.window > 0) { t0 = pos + 1 - L.window; if (t0 < 0) t0 = 0; }
    const int nwin = pos + 1 - t0;
    const int nch = (nwin + kChunk - 1) / kChunk;
    if (c >= nch) return;
    const int cbeg = c * kChunk;
    const int cnt = min(kChunk, nwin - cbeg);
    const bool last_chunk = c == nch - 1;
    const bool new_row = L.append && last_chunk;  // this CTA owns row `pos`
    const int qd = L.n_heads * HD, kvd = L.n_kv * HD;
    const size_t head_base = ((size_t)cb * L.n_kv + h) * L.src_ring;
    if constexpr (attn_tma<EPL>()) {
        // 0. the chunk's rows in ring order: slots s_a.. (and 0.. after a wrap) -> kbuf/vbuf rows 0..cnt-1.
        // Row `pos` of a layer that appends is (re)written below; its stale slot is read here and ignored.
        if (threadIdx.x == 0) {
            mbar_init(&kvbar, 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            const int s_a = (t0 + cbeg) % L.src_ring, n1 = min(cnt, L.src_ring - s_a);
            const uint32_t rb = HD * sizeof(float);
            mbar_expect_tx(&kvbar, 2u * (uint32_t)cnt * rb);
            bulk_g2s(kbuf, L.src_kc + (head_base + s_a) * HD, (uint32_t)n1 * rb, &kvbar);
            bulk_g2s(vbuf, L.src_vc + (head_base + s_a) * HD, (uint32_t)n1 * rb, &kvbar);
            if (n1 < cnt) {
                bulk_g2s(kbuf + n1 * HD, L.src_kc + head_base * HD, (uint32_t)(cnt - n1) * rb, &kvbar);
                bulk_g2s(vbuf + n1 * HD, L.src_vc + head_base * HD, (uint32_t)(cnt - n1) * rb, &kvbar);
            }
        }
    }
    const float2 *cs = L.rope ? L.rope + (size_t)pos * (L.n_rot / 2) : nullptr;

    // 1. query heads (and the new K/V row) into shared memory
    if (warp < G) {
        const float *src = L.q + (size_t)b * qd + (size_t)(h * G + warp) * HD;
        if (L.prep) {
            warp_norm_rope<EPL>(src, L.q_norm, cs, L.n_rot, L.eps, qs[warp], nullptr);
        } else {
#pragma unroll
            for (int i = 0; i < EPL; i++) qs[warp][lane + 32 * i] = src[lane + 32 * i];
        }
    } else if (new_row && warp == G) {
        const int slot = pos % L.ring;
        float *kdst = L.kc + (((size_t)cb * L.n_kv + h) * L.ring + slot) * HD;
        warp_norm_rope<EPL>(L.k + (size_t)b * kvd + (size_t)h * HD, L.k_norm, cs, L.n_rot, L.eps, knew, kdst);
    } else if (new_row && warp == G + 1) {
        const int slot = pos % L.ring;
        float *vdst = L.vc + (((size_t)cb * L.n_kv + h) * L.ring + slot) * HD;
        warp_norm_rope<EPL>(L.v + (size_t)b * kvd + (size_t)h * HD, nullptr, nullptr, 0, L.eps, vnew, vdst);
    }
    __syncthreads();
    float qv[G][EPL];
#pragma unroll
    for (int g = 0; g < G; g++) load_row<EPL>(qv[g], qs[g] + lane * EPL);
    if constexpr (attn_tma<EPL>()) {
        // bounded: on expiry record the status and go on (no thread leaves before the barriers below)
        if (!mbar_wait(&kvbar, 0) && L.err) atomicExch(L.err, G4_ERR_TIMEOUT);
    }
    // 2. scores: warp w owns rows w, w+8, ...; all its row loads are issued first
    constexpr int RPW = kChunk / 8;
    {
        float kv[RPW][EPL];
#pragma unroll
        for (int r = 0; r < RPW; r++) {
            const int tl = warp + 8 * r;
            const int t = t0 + cbeg + min(tl, cnt - 1);
            const float *kr = (new_row && t == pos) ? knew + lane * EPL
                              : attn_tma<EPL>() ? kbuf + min(tl, cnt - 1) * HD + lane * EPL
                                                : L.src_kc + (head_base + (size_t)(t % L.src_ring)) * HD + lane * EPL;
            load_row<EPL>(kv[r], kr);
        }
#pragma unroll
        for (int r = 0; r < RPW; r++) {
            const int tl = warp + 8 * r;
#pragma unroll
            for (int g = 0; g < G; g++) {
                float sv = 0.0f;
#pragma unroll
                for (int e = 0; e < EPL; e++) sv = fmaf(kv[r][e], qv[g][e], sv);
                sv = warp_sum(sv);
                if (lane == 0 && tl < cnt) sc[g][tl] = sv;
            }
        }
    }
    __syncthreads();
    // 3. chunk softmax statistics, one warp per query head
    if (warp < G) {
        float m = -INFINITY;
        for (int tl = lane; tl < cnt; tl += 32) m = fmaxf(m, sc[warp][tl]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int tl = lane; tl < cnt; tl += 32) {
            const float pr = expf(sc[warp][tl] - m);
            sc[warp][tl] = pr;
            l += pr;
        }
        l = warp_sum(l);
        if (lane == 0) { ml[warp][0] = m; ml[warp][1] = l; }
    }
    __syncthreads();
    // 4. unnormalised P.V over the chunk
    float acc[G][EPL];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[g][e] = 0.0f;
    {
        float vv[RPW][EPL];
#pragma unroll
        for (int r = 0; r < RPW; r++) {
            const int tl = warp + 8 * r;
            const int t = t0 + cbeg + min(tl, cnt - 1);
            const float *vr = (new_row && t == pos) ? vnew + lane * EPL
                              : attn_tma<EPL>() ? vbuf + min(tl, cnt - 1) * HD + lane * EPL
                                                : L.src_vc + (head_base + (size_t)(t % L.src_ring)) * HD + lane * EPL;
            load_row<EPL>(vv[r], vr);
        }
#pragma unroll
        for (int r = 0; r < RPW; r++) {
            const int tl = warp + 8 * r;
            if (tl >= cnt) break;
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float pr = sc[g][tl];
#pragma unroll
                for (int e = 0; e < EPL; e++) acc[g][e] = fmaf(pr, vv[r][e], acc[g][e]);
            }
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < EPL; e++) red[warp][g][lane * EPL + e] = acc[g][e];
    __syncthreads();
    // 5. chunk partial -> scratch; the last CTA to finish merges
    const size_t ps = (size_t)HD + 2;
    for (int i = threadIdx.x; i < G * HD; i += 256) {
        const int g = i / HD, d = i % HD;
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) o += red[w][g][d];
        float *pr = L.part + (((size_t)b * L.n_heads + (size_t)h * G + g) * L.max_chunks + c) * ps;
        pr[2 + d] = o;
        if (d == 0) { pr[0] = ml[g][0]; pr[1] = ml[g][1]; }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) ticket = atomicAdd(L.counters + (size_t)b * L.n_kv + h, 1);
    __syncthreads();
    if (ticket != nch - 1) return;
    __threadfence();
    // merge: M = max_c m_c; out = sum_c e^(m_c-M) o_c / sum_c e^(m_c-M) l_c
    if (warp < G) {
        const float *base = L.part + ((size_t)b * L.n_heads + (size_t)h * G + warp) * L.max_chunks * ps;
        float M = -INFINITY;
        for (int cc = lane; cc < nch; cc += 32) M = fmaxf(M, __ldcg(base + cc * ps));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float S = 0.0f;
        for (int cc = lane; cc < nch; cc += 32) {
            const float wgt = expf(__ldcg(base + cc * ps) - M);
            if (cc < kMaxWts) wts[warp * kMaxWts + cc] = wgt;
            S = fmaf(wgt, __ldcg(base + cc * ps + 1), S);
        }
        S = warp_sum(S);
        if (lane == 0) { ml[warp][0] = M; ml[warp][1] = 1.0f / S; }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * HD; i += 256) {
        const int g = i / HD, d = i % HD;
        const float *base = L.part + ((size_t)b * L.n_heads + (size_t)h * G + g) * L.max_chunks * ps;
        float o = 0.0f;
#pragma unroll 8
        for (int cc = 0; cc < nch; cc++) {
            const float wgt = cc < kMaxWts ? wts[g * kMaxWts + cc] : expf(__ldcg(base + cc * ps) - ml[g][0]);
            o = fmaf(wgt, __ldcg(base + cc * ps + 2 + d), o);
        }
        L.qo[(size_t)b * qd + (size_t)(h * G + g) * HD + d] = o * ml[g][1];
    }
    if (threadIdx.x == 0) L.counters[(size_t)b * L.n_kv + h] = 0;  // ready for the next launch
}

// ---------------------------------------------------------------- streaming variant (head dim <= 256)
//
// One CTA per (split of `span` positions, kv head, sequence), span a multiple
// of 32 chosen so that the grid is about four waves: the split is streamed in
// sub-chunks of kSub rows through a kStages-deep shared-memory ring filled by
// bulk copies (TMA), so the copies of the next sub-chunks overlap the
// arithmetic of this one.  Two CTAs share an SM, so one CTA's prologue and
// merge tail overlap the other's streaming.  Each warp keeps an online
// softmax state (max, sum, unnormalised P.V) per query head over the rows it
// owns; the warp states are combined once at the end, then the split partials
// are merged by the last CTA of the (kv head, sequence) as in
// attn_fused_kernel.
constexpr int kSub = 16;        // rows per ring stage
constexpr int kStages = 3;      // 96 KB of K/V per CTA at head dim 256
constexpr int kStreamWarps = 8;

template <int EPL, int G>
constexpr size_t attn_stream_smem() {
    return sizeof(float) * ((size_t)G * EPL * 32 + 2 * (size_t)EPL * 32 + 2 * kStages * (size_t)kSub * EPL * 32 +
                            (size_t)kStreamWarps * G * 2 + (size_t)G * kMaxWts);
}

// Sum of NV = 2^H values per lane over the 32 lanes of a warp with 31 - H
// shuffles less than NV separate reductions: each halving step exchanges half
// of the values.  Returns the total of value index (lane >> (5 - H)).
template <int NV>
__device__ __forceinline__ float warp_transpose_sum(float (&v)[NV], int lane) {
    constexpr int H = NV == 1 ? 0 : NV == 2 ? 1 : NV == 4 ? 2 : NV == 8 ? 3 : 4;
#pragma unroll
    for (int step = 0; step < H; step++) {
        const int o = 16 >> step, half = NV >> (step + 1);
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int k = 0; k < half; k++) {
            const float send = up ? v[k] : v[k + half];
            const float keep = up ? v[k + half] : v[k];
            v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    float r = v[0];
#pragma unroll
    for (int o = 16 >> H; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    return r;
}

template <int EPL, int G, bool MULTI>
__global__ void __launch_bounds__(kStreamWarps * 32, 2) attn_stream_kernel(AttnLayer L, const int *__restrict__ pos_dev, int span,
                                                                      int per) {
    constexpr int HD = EPL * 32, NW = kStreamWarps, RPW = kSub / NW, NV = RPW * G;
    static_assert(RPW == 2, "two rows per warp and sub-chunk: rows differ in lane bit 4 after the transpose sum");
    static_assert(NW * G <= 2 * kSub, "a split's warp states fit in one ring stage");
    constexpr int H = NV == 2 ? 1 : NV == 4 ? 2 : 3;  // log2(NV)
    extern __shared__ __align__(16) float dsm[];
    float(*qs)[HD] = reinterpret_cast<float(*)[HD]>(dsm);  // [G][HD]
    float *knew = dsm + G * HD, *vnew = knew + HD;          // [HD] each
    float *ring = vnew + HD;                                // [kStages][K, V][kSub][HD]
    float(*wml)[G][2] = reinterpret_cast<float(*)[G][2]>(ring + 2 * kStages * kSub * HD);  // [NW][G] (max, sum)
    float *wts = reinterpret_cast<float *>(wml + NW);       // [G][kMaxWts] merge weights
    __shared__ __align__(8) uint64_t full[kStages];
    __shared__ int ticket;
    __shared__ float mlf[G][2];
    pdl_trigger();
    if (!L.early) pdl_wait();
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pos = L.row_pos ? L.row_pos[b] : *pos_dev;
    const int cb = L.row_seq ? L.row_seq[b] : b;  // cache sequence of this query row
    int t0 = 0;
    if (L.window > 0) { t0 = pos + 1 - L.window; if (t0 < 0) t0 = 0; }
    const int nwin = pos + 1 - t0;
    const int nsplit = (nwin + span - 1) / span;  // canonical splits of `span` rows
    const int ncta = (nsplit + per - 1) / per;     // this CTA: splits [c*per, c*per + per)
    if (c >= ncta) return;
    const int sp0 = c * per, sp1 = min(nsplit, sp0 + per);
    const int beg = sp0 * span, ctot = min(sp1 * span, nwin) - beg, nsub = (ctot + kSub - 1) / kSub;
    const bool new_row = L.append && c == ncta - 1;  // this CTA owns row `pos`
    const int qd = L.n_heads * HD, kvd = L.n_kv * HD;
    const size_t head_base = ((size_t)cb * L.n_kv + h) * L.src_ring;
    const float2 *cs = L.rope ? L.rope + (size_t)pos * (L.n_rot / 2) : nullptr;

    // rows [beg + kSub*j, +cnt) of the split (ring slots, split at a wrap) -> stage j % kStages.  Row `pos`
    // of a layer that appends is (re)written below; its stale slot may be read here and is ignored.
    auto issue = [&](int j) {
        const int st = j % kStages, cnt = min(kSub, ctot - j * kSub);
        float *kb = ring + (size_t)st * 2 * kSub * HD, *vb = kb + kSub * HD;
        const int s_a = (t0 + beg + j * kSub) % L.src_ring, n1 = min(cnt, L.src_ring - s_a);
        const uint32_t rb = HD * sizeof(float);
        mbar_expect_tx(&full[st], 2u * (uint32_t)cnt * rb);
        bulk_g2s(kb, L.src_kc + (head_base + s_a) * HD, (uint32_t)n1 * rb, &full[st]);
        bulk_g2s(vb, L.src_vc + (head_base + s_a) * HD, (uint32_t)n1 * rb, &full[st]);
        if (n1 < cnt) {
            bulk_g2s(kb + n1 * HD, L.src_kc + head_base * HD, (uint32_t)(cnt - n1) * rb, &full[st]);
            bulk_g2s(vb + n1 * HD, L.src_vc + head_base * HD, (uint32_t)(cnt - n1) * rb, &full[st]);
        }
    };
    // Sub-chunk j may be copied before the dependency wait (L.early) unless it holds row `pos` of a
    // cache that an earlier kernel of this step writes (a layer without its own cache reads row
    // `pos` of layer 22/23).  Row `pos` of a layer that appends comes from knew/vnew instead.
    auto early_ok = [&](int j) { return L.append || c != ncta - 1 || (j + 1) * kSub < ctot; };
    if (tid == 0) {
        for (int k = 0; k < kStages; k++) mbar_init(&full[k], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (L.early)
            for (int k = 0; k < kStages && k < nsub; k++)
                if (early_ok(k)) issue(k);
    }
    if (L.early) pdl_wait();
    if (tid == 0)
        for (int k = 0; k < kStages && k < nsub; k++)
            if (!L.early || !early_ok(k)) issue(k);
    // query heads (and the new K/V row) into shared memory
    if (warp < G) {
        const float *src = L.q + (size_t)b * qd + (size_t)(h * G + warp) * HD;
        if (L.prep) {
            warp_norm_rope<EPL>(src, L.q_norm, cs, L.n_rot, L.eps, qs[warp], nullptr);
        } else {
#pragma unroll
            for (int i = 0; i < EPL; i++) qs[warp][lane + 32 * i] = src[lane + 32 * i];
        }
    } else if (new_row && warp == G) {
        const int slot = pos % L.ring;
        float *kdst = L.kc + (((size_t)cb * L.n_kv + h) * L.ring + slot) * HD;
        warp_norm_rope<EPL>(L.k + (size_t)b * kvd + (size_t)h * HD, L.k_norm, cs, L.n_rot, L.eps, knew, kdst);
    } else if (new_row && warp == G + 1) {
        const int slot = pos % L.ring;
        float *vdst = L.vc + (((size_t)cb * L.n_kv + h) * L.ring + slot) * HD;
        warp_norm_rope<EPL>(L.v + (size_t)b * kvd + (size_t)h * HD, nullptr, nullptr, 0, L.eps, vnew, vdst);
    }
    __syncthreads();
    float qv[G][EPL];
#pragma unroll
    for (int g = 0; g < G; g++) load_row_il<EPL>(qv[g], qs[g], lane);
    float m[G], l[G], acc[G][EPL];
    // the NW warp states of canonical split sp combined (M = max m, S = sum f l, o = sum f acc in
    // warp order, f = e^(m - M)) into its partial (m, l, o); red: [NW][GH][HD] floats, GH heads at a time
    auto combine = [&](int sp, float *red, int GH) {
        if (lane == 0)
#pragma unroll
            for (int g = 0; g < G; g++) { wml[warp][g][0] = m[g]; wml[warp][g][1] = l[g]; }
        __syncthreads();
        if (tid < G) {
            float M = -INFINITY;
            for (int w = 0; w < NW; w++) M = fmaxf(M, wml[w][tid][0]);
            float S = 0.0f;
            for (int w = 0; w < NW; w++) {
                const float f = wml[w][tid][0] == -INFINITY ? 0.0f : expf(wml[w][tid][0] - M);
                wml[w][tid][0] = f;  // combine weight of warp w
                S = fmaf(f, wml[w][tid][1], S);
            }
            mlf[tid][0] = M;
            mlf[tid][1] = S;
        }
        const size_t ps_ = (size_t)HD + 2;
        for (int g0 = 0; g0 < G; g0 += GH) {
#pragma unroll
            for (int g = 0; g < G; g++)
                if (g >= g0 && g < g0 + GH)
#pragma unroll
                    for (int e = 0; e < EPL; e++)
                        red[((size_t)warp * GH + (g - g0)) * HD + row_elem<EPL>(lane, e)] = acc[g][e];
            __syncthreads();
            for (int i = tid; i < GH * HD; i += NW * 32) {
                const int gg = i / HD, d = i % HD, g = g0 + gg;
                float o = 0.0f;
#pragma unroll
                for (int w = 0; w < NW; w++) o = fmaf(wml[w][g][0], red[((size_t)w * GH + gg) * HD + d], o);
                float *pr = L.part + (((size_t)b * L.n_heads + (size_t)h * G + g) * L.max_chunks + sp) * ps_;
                pr[2 + d] = o;
                if (d == 0) { pr[0] = mlf[g][0]; pr[1] = mlf[g][1]; }
            }
            __syncthreads();
        }
    };
    // this lane's score after the transpose sum: row r_l = idx / G, head g_l = idx % G
    const int idx = (lane >> (5 - H)) & (NV - 1), g_l = idx % G, r_l = idx / G;
    const int spl = MULTI ? span / kSub : nsub;  // sub-chunks per canonical split
    int jj = 0;                                     // sub-chunk within the current split
    for (int j = 0; j < nsub; j++) {
        const int st = j % kStages, cnt = min(kSub, ctot - j * kSub);
        if (jj == 0) {  // a new canonical split: fresh softmax state
#pragma unroll
            for (int g = 0; g < G; g++) {
                m[g] = -INFINITY;
                l[g] = 0.0f;
#pragma unroll
                for (int e = 0; e < EPL; e++) acc[g][e] = 0.0f;
            }
        }
        // bounded: on expiry record the status and go on (every thread still reaches the barriers)
        if (!mbar_wait(&full[st], (j / kStages) & 1) && L.err) atomicExch(L.err, G4_ERR_TIMEOUT);
        const float *kb = ring + (size_t)st * 2 * kSub * HD, *vb = kb + kSub * HD;
        float pv[NV];
#pragma unroll
        for (int r = 0; r < RPW; r++) {
            const int tl = warp + NW * r;
            const int t = t0 + beg + j * kSub + tl;
            float kr[EPL];
            load_row_il<EPL>(kr, (new_row && t == pos) ? knew : kb + min(tl, cnt - 1) * HD, lane);
#pragma unroll
            for (int g = 0; g < G; g++) {
                float d = 0.0f;
#pragma unroll
                for (int e = 0; e < EPL; e++) d = fmaf(kr[e], qv[g][e], d);
                pv[r * G + g] = d;
            }
        }
        float sc = warp_transpose_sum<NV>(pv, lane);  // score of (r_l, g_l)
        if (warp + NW * r_l >= cnt) sc = -INFINITY;
        // online softmax: the row max of each head (rows differ in lane bit 4), broadcast per head
        const float mxl = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 16));
        float mn_l = 0.0f;
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float mx = __shfl_sync(0xffffffffu, mxl, g << (5 - H));
            const float mn = fmaxf(m[g], mx);
            if (mn > m[g]) {  // warp-uniform: rescale only when the running max moves
                const float f = expf(m[g] - mn);  // 0 while m is -inf
                l[g] *= f;
#pragma unroll
                for (int e = 0; e < EPL; e++) acc[g][e] *= f;
                m[g] = mn;
            }
            if (g == g_l) mn_l = m[g];
        }
        const float p = sc == -INFINITY ? 0.0f : expf(sc - mn_l);
        const float ps = p + __shfl_xor_sync(0xffffffffu, p, 16);
#pragma unroll
        for (int g = 0; g < G; g++) l[g] += __shfl_sync(0xffffffffu, ps, g << (5 - H));
        // P.V over this warp's rows
#pragma unroll
        for (int r = 0; r < RPW; r++) {
            const int tl = warp + NW * r;
            if (tl >= cnt) break;
            const int t = t0 + beg + j * kSub + tl;
            float vr[EPL];
            load_row_il<EPL>(vr, (new_row && t == pos) ? vnew : vb + tl * HD, lane);
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float pr = __shfl_sync(0xffffffffu, p, (r * G + g) << (5 - H));
#pragma unroll
                for (int e = 0; e < EPL; e++) acc[g][e] = fmaf(pr, vr[e], acc[g][e]);
            }
        }
        __syncthreads();  // stage st consumed by every warp
        ++jj;
        if (MULTI && jj == spl && j != nsub - 1) {
            // a split ends while the ring still streams: its warp states are combined in stage st
            // (NW * G * HD floats <= 2 * kSub * HD for G <= 4), whose next copy waits until then
            combine(sp0 + j / spl, ring + (size_t)st * 2 * kSub * HD, G);
            jj = 0;
            if (tid == 0 && j + kStages < nsub) {
                fence_proxy_async_smem();  // the combine's shared stores before the copy's writes
                issue(j + kStages);
            }
        } else if (tid == 0 && j + kStages < nsub) {
            issue(j + kStages);
        }
    }
    combine(MULTI ? sp0 + (nsub - 1) / spl : sp0, ring, G);  // the CTA's last split: the ring is free, all heads at once
    __threadfence();
    __syncthreads();
    if (tid == 0) ticket = atomicAdd(L.counters + (size_t)b * L.n_kv + h, 1);
    __syncthreads();
    if (ticket != ncta - 1) return;
    __threadfence();
    const size_t ps_ = (size_t)HD + 2;
    // merge: M = max_c m_c; out = sum_c e^(m_c-M) o_c / sum_c e^(m_c-M) l_c
    if (warp < G) {
        const float *base = L.part + ((size_t)b * L.n_heads + (size_t)h * G + warp) * L.max_chunks * ps_;
        float M = -INFINITY;
        for (int cc = lane; cc < nsplit; cc += 32) M = fmaxf(M, __ldcg(base + cc * ps_));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float S = 0.0f;
        for (int cc = lane; cc < nsplit; cc += 32) {
            const float wgt = expf(__ldcg(base + cc * ps_) - M);
            if (cc < kMaxWts) wts[warp * kMaxWts + cc] = wgt;
            S = fmaf(wgt, __ldcg(base + cc * ps_ + 1), S);
        }
        S = warp_sum(S);
        if (lane == 0) { mlf[warp][0] = M; mlf[warp][1] = 1.0f / S; }
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += NW * 32) {
        const int g = i / HD, d = i % HD;
        const float *base = L.part + ((size_t)b * L.n_heads + (size_t)h * G + g) * L.max_chunks * ps_;
        float o = 0.0f;
#pragma unroll 8
        for (int cc = 0; cc < nsplit; cc++) {
            const float wgt = cc < kMaxWts ? wts[g * kMaxWts + cc] : expf(__ldcg(base + cc * ps_) - mlf[g][0]);
            o = fmaf(wgt, __ldcg(base + cc * ps_ + 2 + d), o);
        }
        const float y = o * mlf[g][1];
        L.qo[(size_t)b * qd + (size_t)(h * G + g) * HD + d] = y;
        if (L.op_bq) ring[i] = y;
    }
    if (tid == 0) L.counters[(size_t)b * L.n_kv + h] = 0;  // ready for the next launch
    if (L.op_bq) {  // the Q8_K blocks of these G heads for the output projection (as tc4_quant_kernel)
        __syncthreads();
        for (int w = warp; w < G * HD / G4_QK; w += NW) {
            const int kb = (h * G * HD) / G4_QK + w;
            uint32_t q[2];
            float d;
            int ls;
            warp_quant_block(ring + w * G4_QK, lane, q, d, ls);
            tc4_store_q8(L.op_bq + (size_t)kb * 544 * L.op_np, L.op_yd + (size_t)kb * L.op_np, L.op_np, b, lane, q, d, ls);
        }
    }
}

template <int EPL, int G>
static int launch_stream_eg(dim3 grid, const AttnLayer &L, const int *pos_dev, int span, int per, cudaStream_t st) {
    if (per > 1)
        G4_CUDA(launch_pdl(attn_stream_kernel<EPL, G, true>, grid, dim3(kStreamWarps * 32), attn_stream_smem<EPL, G>(), st,
                           L, pos_dev, span, per));
    else
        G4_CUDA(launch_pdl(attn_stream_kernel<EPL, G, false>, grid, dim3(kStreamWarps * 32), attn_stream_smem<EPL, G>(), st,
                           L, pos_dev, span, per));
    return G4_OK;
}

template <int EPL>
static int launch_stream_g(const AttnLayer &L, int G, dim3 grid, const int *pos_dev, int span, int per, cudaStream_t st) {
    switch (G) {
    case 1: return launch_stream_eg<EPL, 1>(grid, L, pos_dev, span, per, st);
    case 2: return launch_stream_eg<EPL, 2>(grid, L, pos_dev, span, per, st);
    case 4: return launch_stream_eg<EPL, 4>(grid, L, pos_dev, span, per, st);
    default: set_error(G4_ERR_ARG, "attention: GQA group %d unsupported", G); return G4_ERR_ARG;
    }
}

template <int EPL, int G>
static int launch_fused_eg(dim3 grid, const AttnLayer &L, const int *pos_dev, cudaStream_t st) {
    G4_CUDA(launch_pdl(attn_fused_kernel<EPL, G>, grid, dim3(256), attn_smem_bytes<EPL, G>(), st, L, pos_dev));
    return G4_OK;
}

template <int EPL>
static int launch_fused_g(const AttnLayer &L, int G, dim3 grid, const int *pos_dev, cudaStream_t st) {
    switch (G) {
    case 1: return launch_fused_eg<EPL, 1>(grid, L, pos_dev, st);
    case 2: return launch_fused_eg<EPL, 2>(grid, L, pos_dev, st);
    case 4: return launch_fused_eg<EPL, 4>(grid, L, pos_dev, st);
    default: set_error(G4_ERR_ARG, "attention: GQA group %d unsupported", G); return G4_ERR_ARG;
    }
}

// K/V rows of prefill row blockIdx.x, kv head blockIdx.y: warp 0 normalises and rotates K, warp 1
// normalises V, with the same device function and expressions as the attention kernels' new row.
template <int EPL>
__global__ void kv_append_kernel(AttnLayer L) {
    constexpr int HD = EPL * 32;
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x, h = blockIdx.y, warp = threadIdx.x >> 5;
    const int pos = L.row_pos[r], cb = L.row_seq[r];
    const int kvd = L.n_kv * HD, slot = pos % L.ring;
    const float2 *cs = L.rope ? L.rope + (size_t)pos * (L.n_rot / 2) : nullptr;
    const size_t dst = (((size_t)cb * L.n_kv + h) * L.ring + slot) * HD;
    if (warp == 0)
        warp_norm_rope<EPL>(L.k + (size_t)r * kvd + (size_t)h * HD, L.k_norm, cs, L.n_rot, L.eps, L.kc + dst, nullptr);
    else
        warp_norm_rope<EPL>(L.v + (size_t)r * kvd + (size_t)h * HD, nullptr, nullptr, 0, L.eps, L.vc + dst, nullptr);
}

int launch_kv_append(const AttnLayer &L, int rows, cudaStream_t st) {
    if (!L.row_pos || !L.row_seq || rows <= 0) { set_error(G4_ERR_ARG, "kv_append: rows missing"); return G4_ERR_ARG; }
    const dim3 grid(rows, L.n_kv);
    switch (L.hd) {
    case 64: G4_CUDA(launch_pdl(kv_append_kernel<2>, grid, dim3(64), 0, st, L)); break;
    case 128: G4_CUDA(launch_pdl(kv_append_kernel<4>, grid, dim3(64), 0, st, L)); break;
    case 256: G4_CUDA(launch_pdl(kv_append_kernel<8>, grid, dim3(64), 0, st, L)); break;
    case 512: G4_CUDA(launch_pdl(kv_append_kernel<16>, grid, dim3(64), 0, st, L)); break;
    default: set_error(G4_ERR_ARG, "kv_append: head_dim %d unsupported", L.hd); return G4_ERR_ARG;
    }
    G4_LAUNCHED();
    return G4_OK;
}

int launch_attention(const AttnLayer &L, int B, const int *pos_dev, int max_seq, cudaStream_t st) {
    const int G = L.n_heads / L.n_kv;
    if (L.n_kv <= 0 || L.n_heads % L.n_kv) { set_error(G4_ERR_ARG, "attention: n_heads %% n_kv != 0"); return G4_ERR_ARG; }
    const int span = L.window > 0 ? (L.window < max_seq ? L.window : max_seq) : max_seq;
    const int nch = (span + kChunk - 1) / kChunk;
    if (nch > L.max_chunks) { set_error(G4_ERR_ARG, "attention: %d chunks > scratch %d", nch, L.max_chunks); return G4_ERR_ARG; }
    if (L.append && G + 2 > 8) { set_error(G4_ERR_ARG, "attention: GQA group %d too large", G); return G4_ERR_ARG; }
    dim3 grid(nch, L.n_kv, B);
    int rc;
    if (L.hd <= 256) {
        // Split length: a fixed number of rows per canonical split for each layer kind (by default
        // 64 for a sliding window, 256 for the global context), never derived from the batch or the
        // cache length.  The float sums of a sequence then follow the same split boundaries whether
        // it is decoded alone or in a batch, so batched and single-sequence decoding give identical
        // results.  (Both are multiples of kChunk, which keeps the partials within max_chunks.)
        // A CTA takes `per` consecutive splits when there are more than two CTAs per SM of them
        // (sliding layers of a large batch): one wave of longer CTAs, the same per-split arithmetic.
        const int sp = L.split > 0 ? L.split : (L.window > 0 ? 64 : 256);
        if (sp % kChunk) { set_error(G4_ERR_ARG, "attention: split %d not a multiple of %d", sp, kChunk); return G4_ERR_ARG; }
        static int nsm = 0;
        if (!nsm) {
            int dev = 0;
            G4_CUDA(cudaGetDevice(&dev));
            G4_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
        }
        const int nsp = (span + sp - 1) / sp;
        int per = 1;
        const long ctas1 = (long)nsp * L.n_kv * B, target = 2L * nsm;
        if (L.window > 0 && ctas1 > target)
            per = (int)std::min<long>(nsp, (ctas1 + target - 1) / target);
        const dim3 g2((nsp + per - 1) / per, L.n_kv, B);
        switch (L.hd) {
        case 64: rc = launch_stream_g<2>(L, G, g2, pos_dev, sp, per, st); break;
        case 128: rc = launch_stream_g<4>(L, G, g2, pos_dev, sp, per, st); break;
        default: rc = launch_stream_g<8>(L, G, g2, pos_dev, sp, per, st); break;
        }
        if (rc) return rc;
        G4_LAUNCHED();
        G4_CUDA(cudaGetLastError());
        return G4_OK;
    }
    switch (L.hd) {
    case 64: rc = launch_fused_g<2>(L, G, grid, pos_dev, st); break;
    case 128: rc = launch_fused_g<4>(L, G, grid, pos_dev, st); break;
    case 256: rc = launch_fused_g<8>(L, G, grid, pos_dev, st); break;
    case 512: rc = launch_fused_g<16>(L, G, grid, pos_dev, st); break;
    default: set_error(G4_ERR_ARG, "attention: head_dim %d unsupported", L.hd); return G4_ERR_ARG;
    }
    if (rc) return rc;
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}

template <int EPL, int G>
static int prime_one() {
    G4_CUDA(cudaFuncSetAttribute(attn_fused_kernel<EPL, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)attn_smem_bytes<EPL, G>()));
    return G4_OK;
}
template <int EPL, int G>
static int prime_stream() {
    G4_CUDA(cudaFuncSetAttribute(attn_stream_kernel<EPL, G, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)attn_stream_smem<EPL, G>()));
    G4_CUDA(cudaFuncSetAttribute(attn_stream_kernel<EPL, G, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)attn_stream_smem<EPL, G>()));
    return G4_OK;
}
int prime_attn_attrs() {
    int rc = 0;
    rc |= prime_stream<2, 1>(); rc |= prime_stream<2, 2>(); rc |= prime_stream<2, 4>();
    rc |= prime_stream<4, 1>(); rc |= prime_stream<4, 2>(); rc |= prime_stream<4, 4>();
    rc |= prime_stream<8, 1>(); rc |= prime_stream<8, 2>(); rc |= prime_stream<8, 4>();
    rc |= prime_one<2, 1>(); rc |= prime_one<2, 2>(); rc |= prime_one<2, 4>();
    rc |= prime_one<4, 1>(); rc |= prime_one<4, 2>(); rc |= prime_one<4, 4>();
    rc |= prime_one<8, 1>(); rc |= prime_one<8, 2>(); rc |= prime_one<8, 4>();
    rc |= prime_one<16, 1>(); rc |= prime_one<16, 2>(); rc |= prime_one<16, 4>();
    return rc ? G4_ERR_CUDA : G4_OK;
}

}  // namespace g4
