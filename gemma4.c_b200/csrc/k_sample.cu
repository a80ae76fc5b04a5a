// k_sample.cu — the sampler of generate (sample_token and
// apply_repetition_penalty, gemma4-4b/cpu-blas/main.c:2035-2126) split
// between the GPU and the host.
//
// The vocabulary-wide work runs on the device, next to the logits the LM head
// just wrote: the repetition penalty on the recent tokens, then the top-k
// candidates of each sequence.  The reference builds its top-k list by
// insertion sort over the whole vocabulary with strict comparisons, so the
// list is the first k logits in the total order (value descending, index
// ascending); topk_kernel selects exactly that list with a radix select on
// order-preserving keys (-0 and +0 compare equal, as in float) and an
// index-ordered scan for ties at the k-th value.  Only the k (value, index)
// pairs cross PCIe.  The rest of sample_token — the temperature softmax over k
// values, top-p, and the xorshift64* draws — is k-long sequential float work,
// so the host replays it with the reference's own expressions (expf from the
// C library, the same summation order): the sampled token is the reference's
// token for the same logits and rng state, bit for bit.
#include <math.h>

#include "g4_internal.cuh"
#include "g4_kernels.cuh"

namespace g4 {

namespace {

constexpr int kTopkThreads = 1024;

// Order-preserving 32-bit key of a float with both zeros equal (the
// reference compares floats with < and >).
__device__ __forceinline__ uint32_t f_key(float v) {
    uint32_t b = __float_as_uint(v);
    if ((b & 0x7fffffffu) == 0u) b = 0u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// apply_repetition_penalty (main.c:2114-2126) for sequence blockIdx.x: the
// recent tokens of the sequence in order, repeats applied again each time.
__global__ void rep_penalty_kernel(float *logits, int ld, const int *recent, int rec_ld, const int *nrec, int vocab,
                                   float penalty) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0) return;
    const int b = blockIdx.x, n = nrec[b];
    float *lg = logits + (size_t)b * ld;
    const int *t = recent + (size_t)b * rec_ld;
    for (int i = 0; i < n; i++) {
        const int id = t[i];
        if (id < 0 || id >= vocab) continue;
        const float v = lg[id];
        lg[id] = v >= 0.0f ? v / penalty : v * penalty;
    }
}

// Top-k candidates of row blockIdx.x (k <= 64): out_v/out_i[b][0..k) sorted by
// (value descending, index ascending).  One CTA per row; each thread owns a
// contiguous index range (the tie scan needs index order).
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(const float *logits, int ld, int n, int k, float *out_v,
                                                            int *out_i) {
    __shared__ int whist[kTopkThreads / 32][256];
    __shared__ int hist[256];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_remaining, s_count;
    __shared__ int scan[kTopkThreads];
    __shared__ uint32_t ck[64];
    __shared__ int ci[64];
    __shared__ float cv[64];
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float *lg = logits + (size_t)b * ld;
    const int per = (n + kTopkThreads - 1) / kTopkThreads;
    const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
    if (tid == 0) { s_prefix = 0u; s_mask = 0u; s_remaining = k; s_count = 0; }
    // radix select of the k-th largest key, 8 bits at a time from the top
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int j = lane; j < 256; j += 32) whist[warp][j] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int i = i0; i < i1; i++) {
            const uint32_t key = f_key(lg[i]);
            if ((key & mask) == prefix) atomicAdd(&whist[warp][(key >> shift) & 255u], 1);
        }
        __syncthreads();
        if (tid < 256) {
            int s = 0;
            for (int w = 0; w < kTopkThreads / 32; w++) s += whist[w][tid];
            hist[tid] = s;
        }
        __syncthreads();
        if (tid == 0) {
            int rem = s_remaining, bin = 255;
            for (; bin > 0; bin--) {
                if (hist[bin] >= rem) break;
                rem -= hist[bin];
            }
            s_remaining = rem;  // how many of the k still come from this bin (and below in later digits)
            s_prefix = prefix | ((uint32_t)bin << shift);
            s_mask = mask | (255u << shift);
        }
        __syncthreads();
    }
    const uint32_t T = s_prefix;  // key of the k-th largest logit
    const int need_eq = s_remaining;  // candidates with key == T, lowest indices first
    // keys above T (fewer than k of them), in any order
    int my_eq = 0;
    for (int i = i0; i < i1; i++) {
        const uint32_t key = f_key(lg[i]);
        if (key > T) {
            const int slot = atomicAdd(&s_count, 1);
            ck[slot] = key; ci[slot] = i; cv[slot] = lg[i];
        } else if (key == T) {
            my_eq++;
        }
    }
    // ties at T: exclusive scan of the per-thread counts in index order
    scan[tid] = my_eq;
    __syncthreads();
    for (int off = 1; off < kTopkThreads; off <<= 1) {
        const int v = tid >= off ? scan[tid - off] : 0;
        __syncthreads();
        scan[tid] += v;
        __syncthreads();
    }
    const int base = k - need_eq;  // slots after the keys above T
    int rank = scan[tid] - my_eq;
    for (int i = i0; i < i1 && rank < need_eq; i++) {
        if (f_key(lg[i]) == T) {
            ck[base + rank] = T; ci[base + rank] = i; cv[base + rank] = lg[i];
            rank++;
        }
    }
    __syncthreads();
    // order the k candidates: (key descending, index ascending)
    if (warp == 0) {
        for (int c = lane; c < k; c += 32) {
            int r = 0;
            for (int j = 0; j < k; j++) r += (ck[j] > ck[c]) || (ck[j] == ck[c] && ci[j] < ci[c]);
            out_v[(size_t)b * k + r] = cv[c];
            out_i[(size_t)b * k + r] = ci[c];
        }
    }
}

}  // namespace

int launch_rep_penalty(float *logits, int ld, const int *recent, int rec_ld, const int *nrec, int vocab, float penalty,
                       int B, cudaStream_t st) {
    G4_CUDA(launch_pdl(rep_penalty_kernel, dim3(B), dim3(32), 0, st, logits, ld, recent, rec_ld, nrec, vocab, penalty));
    G4_LAUNCHED();
    return G4_OK;
}

int launch_topk(const float *logits, int ld, int n, int k, float *out_v, int *out_i, int B, cudaStream_t st) {
    if (k < 1 || k > 64 || k > n) { set_error(G4_ERR_ARG, "top-k: k=%d must be in [1, min(64, n=%d)]", k, n); return G4_ERR_ARG; }
    G4_CUDA(launch_pdl(topk_kernel, dim3(B), dim3(kTopkThreads), 0, st, logits, ld, n, k, out_v, out_i));
    G4_LAUNCHED();
    return G4_OK;
}

// rng_f32 (main.c:2035-2040): xorshift64*, top 24 bits as a float in [0, 1).
static float rng_f32_host(uint64_t *state) {
    *state ^= *state >> 12;
    *state ^= *state << 25;
    *state ^= *state >> 27;
    return (float)((*state * 0x2545F4914F6CDD1DULL) >> 40) / (float)(1 << 24);
}

// The tail of sample_token (main.c:2071-2111) over the k candidates sorted by
// (value descending, index ascending), with the reference's float expressions
// and order: softmax at temperature temp, then a plain draw or a top-p draw.
// p is scratch of k floats.  Returns the sampled token id.
int sample_tail_host(const float *vals, const int *idx, int k, float temp, float topp, uint64_t *rng, float *p) {
    const float maxv = vals[0];
    float sum = 0.0f;
    for (int i = 0; i < k; i++) {
        p[i] = expf((vals[i] - maxv) / temp);
        sum += p[i];
    }
    for (int i = 0; i < k; i++) p[i] /= sum;
    const float coin = rng_f32_host(rng);
    if (topp <= 0.0f || topp >= 1.0f) {
        float cdf = 0.0f;
        int result = idx[k - 1];
        for (int i = 0; i < k; i++) {
            cdf += p[i];
            if (coin < cdf) { result = idx[i]; break; }
        }
        return result;
    }
    float cum = 0.0f;
    int last = k - 1;
    for (int i = 0; i < k; i++) {
        cum += p[i];
        if (cum > topp) { last = i; break; }
    }
    const float r = rng_f32_host(rng) * cum;
    float cdf = 0.0f;
    int result = idx[last];
    for (int i = 0; i <= last; i++) {
        cdf += p[i];
        if (r < cdf) { result = idx[i]; break; }
    }
    return result;
}

}  // namespace g4
