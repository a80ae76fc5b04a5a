// noalloc.cu — decode attention for callers that cannot allocate device memory.
//
// Some hosts of this library own every byte of device memory themselves: an
// inference server that carves HBM into its own pools at start-up, a plugin
// that runs inside someone else's process and memory budget, or a loop that
// must not pay the device-wide synchronisation a cudaMalloc/cudaFree can
// imply.  Such callers can hand us device pointers for inputs and outputs but
// cannot let us allocate the attention kernel's scratch (the per-chunk
// partial results of the split-K softmax and the tickets that pick the CTA
// merging them).  g4d_attn_decode_noalloc therefore takes its scratch from a
// fixed array compiled into the library instead of from cudaMalloc.
//
// The array lives in every GPU's memory that loads the library, for the life
// of the process.  Its host-side name is only a stand-in for the symbol, so
// the device address is looked up (cudaGetSymbolAddress) once per device, on
// the first call made on that device; that first call should therefore come
// before any stream capture.  Every call shares the one array: calls whose
// work can overlap on the GPU (different streams, or different host threads)
// race on it and must be ordered by the caller.
//
// The call is asynchronous, so it cannot return the status of the kernel's
// bounded device-side waits.  A wait that gave up (2 s without progress; not
// expected on a healthy GPU) is recorded in a status word inside the array and
// a follow-up kernel then fills `out` with NaN, so the failure is visible in
// the result instead of silently returning partial sums.
#include <mutex>

#include "g4_internal.cuh"
#include "g4_kernels.cuh"

namespace g4 {
int prime_attn_attrs();
}

using namespace g4;

// Maximum scratch: partials n_heads * ceil(nwin/32) * (head_dim + 2) floats,
// then one int per kv head (tickets) followed by the wait-status word, then
// the position, each group 256-byte aligned.
// 4 MiB covers 8 heads of head_dim 256 over an 8192-position window
// (about 2.1 MiB).
static constexpr size_t kNoAllocScratchBytes = (size_t)4 << 20;
static __device__ __align__(256) unsigned char g4_noalloc_scratch[kNoAllocScratchBytes];

// Writes the query position into the scratch array (a kernel argument, so no
// host buffer has to outlive the asynchronous call).
static __global__ void noalloc_set_pos(int *dst, int value) { *dst = value; }

// After the attention: if a bounded wait gave up, the output is not the
// attention result; make that visible as NaN.
static __global__ void noalloc_poison(const int *status, float *out, int n) {
    if (*status == 0) return;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = __int_as_float(0x7fc00000);
}

static std::mutex g_na_mu;
static void *g_na_addr[64];   // device address of the array, per device ordinal
static bool g_na_primed[64];

extern "C" int g4d_attn_decode_noalloc(float *out, const float *q, const float *k, const float *v, int nwin,
                                       int n_heads, int n_kv_heads, int hd, void *stream) {
    if (!out || !q || nwin < 0 || n_kv_heads <= 0 || n_heads <= 0 || n_heads % n_kv_heads ||
        (hd != 64 && hd != 128 && hd != 256 && hd != 512) || (nwin > 0 && (!k || !v))) {
        set_error(G4_ERR_ARG, "attn_decode_noalloc: bad arguments");
        return G4_ERR_ARG;
    }
    const int G = n_heads / n_kv_heads;
    if (G != 1 && G != 2 && G != 4) {
        set_error(G4_ERR_ARG, "attn_decode_noalloc: GQA group %d unsupported", G);
        return G4_ERR_ARG;
    }
    cudaStream_t st = (cudaStream_t)stream;
    if (nwin == 0) {  // the reference zeroes the head outputs (main.c:1947-1949)
        G4_CUDA(cudaMemsetAsync(out, 0, sizeof(float) * (size_t)n_heads * hd, st));
        return G4_OK;
    }
    const int chunk = attn_chunk_size();
    const int nch = (nwin + chunk - 1) / chunk;
    const size_t part_bytes = sizeof(float) * (size_t)n_heads * nch * (hd + 2);
    const size_t ctr_off = (part_bytes + 255) & ~(size_t)255;
    const size_t pos_off = (ctr_off + sizeof(int) * ((size_t)n_kv_heads + 1) + 255) & ~(size_t)255;
    const size_t need = pos_off + sizeof(int);
    if (need > kNoAllocScratchBytes) {
        set_error(G4_ERR_ARG, "attn_decode_noalloc: needs %zu scratch bytes, the static limit is %zu", need,
                  kNoAllocScratchBytes);
        return G4_ERR_ARG;
    }
    int dev = 0;
    G4_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) { set_error(G4_ERR_NO_DEVICE, "device ordinal %d out of range", dev); return G4_ERR_NO_DEVICE; }
    void *base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_na_mu);
        if (!g_na_addr[dev]) {  // once per device, with that device current
            void *p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g4_noalloc_scratch);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g4_noalloc_scratch)", __FILE__, __LINE__);
            g_na_addr[dev] = p;
        }
        if (!g_na_primed[dev]) {  // shared-memory limits of the attention kernels on this device
            const int rc = prime_attn_attrs();
            if (rc) return rc;
            g_na_primed[dev] = true;
        }
        base = g_na_addr[dev];
    }
    int *counters = (int *)((unsigned char *)base + ctr_off);
    int *status = counters + n_kv_heads;
    int *pos_dev = (int *)((unsigned char *)base + pos_off);
    // the tickets and the status word must start at zero; the array keeps whatever the last call left
    G4_CUDA(cudaMemsetAsync(counters, 0, sizeof(int) * ((size_t)n_kv_heads + 1), st));
    noalloc_set_pos<<<1, 1, 0, st>>>(pos_dev, nwin - 1);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    AttnLayer L{};
    L.hd = hd; L.n_rot = 0; L.n_heads = n_heads; L.n_kv = n_kv_heads;
    L.q = q; L.prep = 0; L.append = 0;
    L.src_kc = k; L.src_vc = v; L.src_ring = nwin;   // [n_kv][nwin][hd]: slot t = t
    L.window = 0; L.eps = 0.0f; L.err = status;
    L.qo = out; L.part = (float *)base; L.counters = counters; L.max_chunks = nch;
    const int rc = launch_attention(L, 1, pos_dev, nwin, st);
    if (rc) return rc;
    noalloc_poison<<<4, 256, 0, st>>>(status, out, n_heads * hd);
    G4_LAUNCHED();
    G4_CUDA(cudaGetLastError());
    return G4_OK;
}
