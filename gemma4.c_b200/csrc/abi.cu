// abi.cu — error state, weight upload, and the per-call C ABI: drop-ins for
// the static functions of gemma4-4b/cpu-blas/main.c that take host buffers.
//
// Each call copies its activation to the device, runs the sm_100a kernel on
// the library's stream and copies the result back before returning.  Weight
// tensors are uploaded once per host pointer (the reference's weights are
// read-only views of the GGUF mmap) and found again by pointer, type and
// shape.  All entry points are serialised by one mutex.
#include <math.h>
#include <stdarg.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <vector>

#include "g4_internal.cuh"
#include "g4_kernels.cuh"

namespace g4 {

static thread_local int t_err = 0;
static thread_local char t_msg[512] = {0};
static std::atomic<uint64_t> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(int code, const char *fmt, ...) {
    t_err = code;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof t_msg, fmt, ap);
    va_end(ap);
}

int cuda_fail(cudaError_t e, const char *what, const char *file, int line) {
    set_error(e == cudaErrorMemoryAllocation ? G4_ERR_OOM : G4_ERR_CUDA, "%s failed: %s (%s:%d)", what,
              cudaGetErrorString(e), file, line);
    return t_err;
}

int upload_tensor(void *dst, const void *src, int type, int n, int rows, cudaStream_t st) {
    if (type != G4_Q6_K) {
        G4_CUDA(cudaMemcpyAsync(dst, src, row_bytes(type, n) * (size_t)rows, cudaMemcpyHostToDevice, st));
        G4_CUDA(cudaStreamSynchronize(st));
        return G4_OK;
    }
    // Q6_K: raw blocks through a bounded staging buffer, then split into per-row planes.
    const size_t total = (size_t)rows * (n / G4_QK);
    const size_t chunk = total < (size_t)(1 << 20) ? total : (size_t)(1 << 20);  // 1M blocks = 210 MB
    void *tmp = nullptr;
    G4_CUDA(cudaMalloc(&tmp, chunk * 210));
    int rc = G4_OK;
    for (size_t off = 0; off < total && rc == G4_OK; off += chunk) {
        const size_t nb = total - off < chunk ? total - off : chunk;
        cudaError_t e = cudaMemcpyAsync(tmp, (const uint8_t *)src + off * 210, nb * 210, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) { rc = cuda_fail(e, "cudaMemcpyAsync", __FILE__, __LINE__); break; }
        rc = launch_repack_q6(tmp, nb, off, dst, n / G4_QK, st);
        if (rc == G4_OK) {
            e = cudaStreamSynchronize(st);
            if (e != cudaSuccess) rc = cuda_fail(e, "cudaStreamSynchronize", __FILE__, __LINE__);
        }
    }
    cudaFree(tmp);
    return rc;
}

// Device (cos, sin) of the reference RoPE angles for one position.
void rope_row_host(float2 *out, int pos, int n_rot, float base, float freq_scale, const float *ff) {
    const float theta_scale = powf(base, -2.0f / (float)n_rot);
    float theta = (float)pos;
    for (int j = 0; j < n_rot / 2; j++) {
        const float angle = freq_scale * theta / (ff ? ff[j] : 1.0f);
        out[j] = make_float2(cosf(angle), sinf(angle));
        theta *= theta_scale;
    }
}

int launch_rope(float *vec, int n_heads, int hd, int n_rot, const float2 *cs, cudaStream_t st);
int prime_kernel_attrs();
int launch_gemv_deq(const void *w, int type, int n, int rows, const float *x, float *out, cudaStream_t st);

// ---------------------------------------------------------------- per-call context

struct RegEntry {
    void *dev;
    size_t bytes;
    int type, n, rows;
};

struct Ctx {
    int device = -1;
    cudaStream_t st = nullptr;
    std::map<const void *, RegEntry> reg;
    size_t reg_bytes = 0;
    uint8_t *scratch = nullptr;
    size_t scratch_bytes = 0;
    int *err = nullptr;  // device status word of bounded waits
};

static std::mutex g_mu;
static Ctx g_ctx;
static int g_req_device = -1;

static void reg_release(Ctx &c) {
    for (auto &kv : c.reg) cudaFree(kv.second.dev);
    c.reg.clear();
    c.reg_bytes = 0;
}

static int ctx_ready() {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        set_error(G4_ERR_NO_DEVICE, "no CUDA device (%s)", cudaGetErrorString(e));
        return G4_ERR_NO_DEVICE;
    }
    int dev = g_req_device;
    if (dev < 0) G4_CUDA(cudaGetDevice(&dev));
    if (g_ctx.device == dev && g_ctx.st) {
        G4_CUDA(cudaSetDevice(dev));
        return G4_OK;
    }
    if (g_ctx.st) {  // switching devices: drop everything held on the old one
        cudaSetDevice(g_ctx.device);
        reg_release(g_ctx);
        cudaFree(g_ctx.scratch);
        cudaFree(g_ctx.err);
        cudaStreamDestroy(g_ctx.st);
        g_ctx = Ctx();
    }
    G4_CUDA(cudaSetDevice(dev));
    cudaDeviceProp p;
    G4_CUDA(cudaGetDeviceProperties(&p, dev));
    if (p.major != 10) {
        set_error(G4_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", dev, p.major, p.minor);
        return G4_ERR_NO_DEVICE;
    }
    {
        const int rc = prime_kernel_attrs();  // dynamic shared memory limits, once per device
        if (rc) return rc;
    }
    G4_CUDA(cudaStreamCreateWithFlags(&g_ctx.st, cudaStreamNonBlocking));
    G4_CUDA(cudaMalloc(&g_ctx.err, sizeof(int)));
    G4_CUDA(cudaMemset(g_ctx.err, 0, sizeof(int)));
    g_ctx.device = dev;
    return G4_OK;
}

// Scratch carving: sizes are rounded up to 256 bytes.
struct Carve {
    size_t off = 0;
    size_t take(size_t b) { size_t o = off; off += (b + 255) & ~(size_t)255; return o; }
};

static int scratch_reserve(size_t bytes) {
    if (bytes <= g_ctx.scratch_bytes) return G4_OK;
    if (g_ctx.scratch) cudaFree(g_ctx.scratch);
    g_ctx.scratch = nullptr;
    g_ctx.scratch_bytes = 0;
    G4_CUDA(cudaMalloc(&g_ctx.scratch, bytes));
    g_ctx.scratch_bytes = bytes;
    return G4_OK;
}

static int weight_dev(const void *host, int type, int n, int rows, const void **out) {
    const size_t bytes = row_bytes(type, n) * (size_t)rows;
    auto it = g_ctx.reg.find(host);
    if (it != g_ctx.reg.end()) {
        const RegEntry &r = it->second;
        const bool ok = r.type == type && r.n == n && (type == G4_Q6_K ? r.rows == rows : r.rows >= rows);
        if (ok) { *out = r.dev; return G4_OK; }
        cudaFree(r.dev);
        g_ctx.reg_bytes -= r.bytes;
        g_ctx.reg.erase(it);
    }
    void *d = nullptr;
    const size_t dbytes = device_tensor_bytes(type, n, rows);
    G4_CUDA(cudaMalloc(&d, dbytes));
    int rc = upload_tensor(d, host, type, n, rows, g_ctx.st);
    if (rc) { cudaFree(d); return rc; }
    g_ctx.reg[host] = RegEntry{d, dbytes, type, n, rows};
    g_ctx.reg_bytes += dbytes;
    (void)bytes;
    *out = d;
    return G4_OK;
}

static int check_mm_args(const void *o, const void *w, int n, int d, int type) {
    if (!o || !w || n <= 0 || d <= 0) { set_error(G4_ERR_ARG, "mm: bad pointer or size (n=%d d=%d)", n, d); return G4_ERR_ARG; }
    if (!type_known(type)) { set_error(G4_ERR_TYPE, "Unsupported tensor type %d in matmul", type); return G4_ERR_TYPE; }
    if ((type == G4_Q4_K || type == G4_Q5_K || type == G4_Q6_K) && n % G4_QK) {
        set_error(G4_ERR_ARG, "mm: n=%d not multiple of QK_K", n);
        return G4_ERR_ARG;
    }
    return G4_OK;
}

#define G4_TRY(x) do { int rc_ = (x); if (rc_) return rc_; } while (0)

// o_dev = W x for any supported type.  Q4_K/Q5_K use q8_dev (already filled).
static int gemv_any(float *o_dev, const float *x_dev, const void *wd, int n, int d, int type, const void *q8_dev,
                    int epi, unsigned long long *keys, float cap) {
    if (type == G4_Q4_K || type == G4_Q5_K || type == G4_Q6_K) {
        GemvJobs jobs{};
        jobs.njobs = 1;
        GemvJob &J = jobs.j[0];
        J.w = wd; J.type = type; J.n = n; J.rows = d;
        J.act = (type == G4_Q6_K) ? (const void *)x_dev : q8_dev;
        J.act_stride = n; J.out = o_dev; J.out_stride = d; J.epi = epi; J.amax = keys; J.cap = cap;
        jobs.err = g_ctx.err;
        return launch_gemv_kquant(jobs, 1, g_ctx.st);
    }
    G4_TRY(launch_gemv_dense(wd, type, n, d, x_dev, n, o_dev, d, 1, EPI_STORE, nullptr, 0, g_ctx.st));
    if (epi == EPI_SOFTCAP_ARGMAX) return launch_softcap_argmax(o_dev, d, d, cap, keys, 1, g_ctx.st);
    return G4_OK;
}

static int sync_ctx() {
    int h = 0;
    G4_CUDA(cudaMemcpyAsync(&h, g_ctx.err, sizeof(int), cudaMemcpyDeviceToHost, g_ctx.st));
    G4_CUDA(cudaStreamSynchronize(g_ctx.st));
    if (h) {
        G4_CUDA(cudaMemset(g_ctx.err, 0, sizeof(int)));
        set_error(h, "a device-side wait gave up (bounded wait timeout); results are invalid");
        return h;
    }
    return G4_OK;
}

}  // namespace g4

using namespace g4;

extern "C" {

int g4_last_error(void) { return t_err; }
const char *g4_last_error_string(void) { return t_msg; }
void g4_clear_error(void) { t_err = 0; t_msg[0] = 0; }
uint64_t g4_kernel_launch_count(void) { return g_launches.load(); }

int g4_set_device(int device) {
    std::lock_guard<std::mutex> lk(g_mu);
    g_req_device = device;
    return ctx_ready();
}

int g4_registry_clear(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_ctx.st) {
        cudaSetDevice(g_ctx.device);
        cudaStreamSynchronize(g_ctx.st);
        reg_release(g_ctx);
    }
    return G4_OK;
}

int g4_registry_stats(int *n_tensors, size_t *bytes) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (n_tensors) *n_tensors = (int)g_ctx.reg.size();
    if (bytes) *bytes = g_ctx.reg_bytes;
    return G4_OK;
}

int g4_quantize_row_q8_K_ex(const float *x, g4_block_q8_K *y, int k) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!x || !y || k < 0 || k % G4_QK) { set_error(G4_ERR_ARG, "quantize_row_q8_K: k=%d must be a non-negative multiple of 256", k); return G4_ERR_ARG; }
    if (k == 0) return G4_OK;
    G4_TRY(ctx_ready());
    Carve cv;
    const size_t ox = cv.take((size_t)k * 4), oy = cv.take((size_t)(k / G4_QK) * G4_Q8_BYTES);
    G4_TRY(scratch_reserve(cv.off));
    float *xd = (float *)(g_ctx.scratch + ox);
    uint8_t *yd = g_ctx.scratch + oy;
    G4_CUDA(cudaMemcpyAsync(xd, x, (size_t)k * 4, cudaMemcpyHostToDevice, g_ctx.st));
    G4_TRY(launch_quantize_q8k(xd, k, yd, k, 1, g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(y, yd, (size_t)(k / G4_QK) * G4_Q8_BYTES, cudaMemcpyDeviceToHost, g_ctx.st));
    return sync_ctx();
}
void g4_quantize_row_q8_K(const float *x, g4_block_q8_K *y, int k) { (void)g4_quantize_row_q8_K_ex(x, y, k); }

static int vec_dot_ex(int type, int n, const void *x, const g4_block_q8_K *y, float *out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!x || !y || !out || n <= 0 || n % G4_QK) { set_error(G4_ERR_ARG, "vec_dot: bad arguments (n=%d)", n); return G4_ERR_ARG; }
    G4_TRY(ctx_ready());
    const int nb = n / G4_QK;
    Carve cv;
    const size_t ow = cv.take(row_bytes(type, n)), oq = cv.take((size_t)nb * G4_Q8_BYTES), oo = cv.take(4);
    G4_TRY(scratch_reserve(cv.off));
    G4_CUDA(cudaMemcpyAsync(g_ctx.scratch + ow, x, row_bytes(type, n), cudaMemcpyHostToDevice, g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(g_ctx.scratch + oq, y, (size_t)nb * G4_Q8_BYTES, cudaMemcpyHostToDevice, g_ctx.st));
    G4_TRY(gemv_any((float *)(g_ctx.scratch + oo), nullptr, g_ctx.scratch + ow, n, 1, type, g_ctx.scratch + oq,
                    EPI_STORE, nullptr, 0.0f));
    G4_CUDA(cudaMemcpyAsync(out, g_ctx.scratch + oo, 4, cudaMemcpyDeviceToHost, g_ctx.st));
    return sync_ctx();
}
int g4_vec_dot_q4_K_q8_K_ex(int n, const void *x, const g4_block_q8_K *y, float *out) { return vec_dot_ex(G4_Q4_K, n, x, y, out); }
int g4_vec_dot_q5_K_q8_K_ex(int n, const void *x, const g4_block_q8_K *y, float *out) { return vec_dot_ex(G4_Q5_K, n, x, y, out); }
void g4_vec_dot_q4_K_q8_K(int n, const void *x, const g4_block_q8_K *y, float *out) { (void)vec_dot_ex(G4_Q4_K, n, x, y, out); }
void g4_vec_dot_q5_K_q8_K(int n, const void *x, const g4_block_q8_K *y, float *out) { (void)vec_dot_ex(G4_Q5_K, n, x, y, out); }

int g4_quant_dot_block_sums(const void *w, int n, int d, int type, const g4_block_q8_K *q8, int32_t *sumi_s,
                            int32_t *sumi_m) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (type != G4_Q4_K && type != G4_Q5_K) { set_error(G4_ERR_TYPE, "block sums: type %d is not Q4_K/Q5_K", type); return G4_ERR_TYPE; }
    if (!w || !q8 || !sumi_s || !sumi_m || n <= 0 || d <= 0 || n % G4_QK) { set_error(G4_ERR_ARG, "block sums: bad arguments"); return G4_ERR_ARG; }
    G4_TRY(ctx_ready());
    const int nb = n / G4_QK;
    const size_t wb = row_bytes(type, n) * (size_t)d, ob = (size_t)d * nb * 4;
    Carve cv;
    const size_t ow = cv.take(wb), oq = cv.take((size_t)nb * G4_Q8_BYTES), os = cv.take(ob), om = cv.take(ob);
    G4_TRY(scratch_reserve(cv.off));
    uint8_t *s = g_ctx.scratch;
    G4_CUDA(cudaMemcpyAsync(s + ow, w, wb, cudaMemcpyHostToDevice, g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(s + oq, q8, (size_t)nb * G4_Q8_BYTES, cudaMemcpyHostToDevice, g_ctx.st));
    G4_TRY(launch_qk_block_sums(s + ow, type, n, d, s + oq, (int *)(s + os), (int *)(s + om), g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(sumi_s, s + os, ob, cudaMemcpyDeviceToHost, g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(sumi_m, s + om, ob, cudaMemcpyDeviceToHost, g_ctx.st));
    return sync_ctx();
}

// mm (main.c:1669-1694)
static int mm_impl(float *o, const float *x, const void *w, int n, int d, int type, g4_block_q8_K *q8, int q8_ready,
                   int f32_path) {
    G4_TRY(check_mm_args(o, w, n, d, type));
    const bool q8t = is_q8_type(type) && !f32_path;
    if (q8t && !q8) { set_error(G4_ERR_ARG, "mm: Q8_K buffer required for type %d", type); return G4_ERR_ARG; }
    if (!x && !(q8t && q8_ready)) { set_error(G4_ERR_ARG, "mm: x is NULL"); return G4_ERR_ARG; }
    G4_TRY(ctx_ready());
    const void *wd;
    G4_TRY(weight_dev(w, type, n, d, &wd));
    const int nb = (n + G4_QK - 1) / G4_QK;
    Carve cv;
    const size_t ox = cv.take((size_t)n * 4), oq = cv.take((size_t)nb * G4_Q8_BYTES), oo = cv.take((size_t)d * 4);
    G4_TRY(scratch_reserve(cv.off));
    uint8_t *s = g_ctx.scratch;
    float *xd = (float *)(s + ox), *od = (float *)(s + oo);
    if (x) G4_CUDA(cudaMemcpyAsync(xd, x, (size_t)n * 4, cudaMemcpyHostToDevice, g_ctx.st));
    if (q8t) {
        if (q8_ready) {
            G4_CUDA(cudaMemcpyAsync(s + oq, q8, (size_t)nb * G4_Q8_BYTES, cudaMemcpyHostToDevice, g_ctx.st));
        } else {  // the reference leaves the quantized activation in q8 (main.c:1686)
            G4_TRY(launch_quantize_q8k(xd, n, s + oq, n, 1, g_ctx.st));
            G4_CUDA(cudaMemcpyAsync(q8, s + oq, (size_t)nb * G4_Q8_BYTES, cudaMemcpyDeviceToHost, g_ctx.st));
        }
        G4_TRY(gemv_any(od, xd, wd, n, d, type, s + oq, EPI_STORE, nullptr, 0.0f));
    } else if (is_q8_type(type)) {  // fp32 dequant-dot of Q4_K/Q5_K rows (mm_quant_rows)
        G4_TRY(launch_gemv_deq(wd, type, n, d, xd, od, g_ctx.st));
    } else {
        G4_TRY(gemv_any(od, xd, wd, n, d, type, nullptr, EPI_STORE, nullptr, 0.0f));
    }
    G4_CUDA(cudaMemcpyAsync(o, od, (size_t)d * 4, cudaMemcpyDeviceToHost, g_ctx.st));
    return sync_ctx();
}

int g4_mm_ex(float *o, const float *x, const void *w, int n, int d, int type, g4_block_q8_K *q8, int q8_ready) {
    std::lock_guard<std::mutex> lk(g_mu);
    return mm_impl(o, x, w, n, d, type, q8, q8_ready, 0);
}
void g4_mm(float *o, const float *x, const void *w, int n, int d, int type, g4_block_q8_K *q8, int q8_ready) {
    (void)g4_mm_ex(o, x, w, n, d, type, q8, q8_ready);
}

int g4_mm_quant_dot_rows_ex(float *o, const void *w, int n, int d, int type, const g4_block_q8_K *q8) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!is_q8_type(type)) { set_error(G4_ERR_TYPE, "vec_dot_row_q8_K: unsupported type %d", type); return G4_ERR_TYPE; }
    return mm_impl(o, nullptr, w, n, d, type, const_cast<g4_block_q8_K *>(q8), 1, 0);
}
void g4_mm_quant_dot_rows(float *o, const void *w, int n, int d, int type, const g4_block_q8_K *q8) {
    (void)g4_mm_quant_dot_rows_ex(o, w, n, d, type, q8);
}

int g4_mm_quant_rows_ex(float *o, const float *x, const void *w, int n, int d, int type) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (type != G4_Q4_K && type != G4_Q5_K && type != G4_Q6_K) {
        set_error(G4_ERR_TYPE, "dequant_one_block_to: bad type %d", type);
        return G4_ERR_TYPE;
    }
    return mm_impl(o, x, w, n, d, type, nullptr, 0, 1);
}
void g4_mm_quant_rows(float *o, const float *x, const void *w, int n, int d, int type) {
    (void)g4_mm_quant_rows_ex(o, x, w, n, d, type);
}

// mm_argmax_row (main.c:1570-1667): no softcap; F16 is not supported there.
int g4_mm_argmax_row(const float *x, const void *w, int n, int d, int type, g4_block_q8_K *q8) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (type == G4_F16 || !type_known(type)) { set_error(G4_ERR_TYPE, "mm_argmax_row: unsupported type %d", type); return -1; }
    if (!x) { set_error(G4_ERR_ARG, "mm_argmax_row: x is NULL"); return -1; }
    float dummy;
    if (check_mm_args(&dummy, w, n, d, type)) return -1;
    if (is_q8_type(type) && !q8) { set_error(G4_ERR_ARG, "mm_argmax_row: Q8_K buffer required"); return -1; }
    if (ctx_ready()) return -1;
    const void *wd;
    if (weight_dev(w, type, n, d, &wd)) return -1;
    const int nb = (n + G4_QK - 1) / G4_QK;
    Carve cv;
    const size_t ox = cv.take((size_t)n * 4), oq = cv.take((size_t)nb * G4_Q8_BYTES), oo = cv.take((size_t)d * 4),
                 ok = cv.take(8);
    if (scratch_reserve(cv.off)) return -1;
    uint8_t *s = g_ctx.scratch;
    float *xd = (float *)(s + ox), *od = (float *)(s + oo);
    unsigned long long *kd = (unsigned long long *)(s + ok), key = 0;
    if (cudaMemcpyAsync(xd, x, (size_t)n * 4, cudaMemcpyHostToDevice, g_ctx.st) != cudaSuccess ||
        cudaMemsetAsync(kd, 0, 8, g_ctx.st) != cudaSuccess) {
        set_error(G4_ERR_CUDA, "mm_argmax_row: copy failed");
        return -1;
    }
    if (is_q8_type(type)) {
        if (launch_quantize_q8k(xd, n, s + oq, n, 1, g_ctx.st)) return -1;
        cudaMemcpyAsync(q8, s + oq, (size_t)nb * G4_Q8_BYTES, cudaMemcpyDeviceToHost, g_ctx.st);
    }
    if (gemv_any(od, xd, wd, n, d, type, s + oq, EPI_SOFTCAP_ARGMAX, kd, 0.0f)) return -1;
    if (cudaMemcpyAsync(&key, kd, 8, cudaMemcpyDeviceToHost, g_ctx.st) != cudaSuccess || sync_ctx()) {
        set_error(G4_ERR_CUDA, "mm_argmax_row: readback failed");
        return -1;
    }
    return argmax_key_index(key);
}

int g4_apply_rope_neox_ex(float *vec, int n_heads, int head_dim, int n_rot, int pos, float freq_base, float freq_scale,
                          const float *freq_factors) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!vec || n_heads <= 0 || head_dim <= 0 || head_dim % 2 || n_rot < 0 || n_rot > head_dim || n_rot % 2 || pos < 0) {
        set_error(G4_ERR_ARG, "apply_rope_neox: bad arguments");
        return G4_ERR_ARG;
    }
    G4_TRY(ctx_ready());
    std::vector<float2> cs((size_t)(n_rot / 2 > 0 ? n_rot / 2 : 1));
    rope_row_host(cs.data(), pos, n_rot, freq_base, freq_scale, freq_factors);
    const size_t nv = (size_t)n_heads * head_dim;
    Carve cv;
    const size_t ov = cv.take(nv * 4), oc = cv.take(cs.size() * sizeof(float2));
    G4_TRY(scratch_reserve(cv.off));
    float *vd = (float *)(g_ctx.scratch + ov);
    float2 *cd = (float2 *)(g_ctx.scratch + oc);
    G4_CUDA(cudaMemcpyAsync(vd, vec, nv * 4, cudaMemcpyHostToDevice, g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(cd, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice, g_ctx.st));
    G4_TRY(launch_rope(vd, n_heads, head_dim, n_rot, cd, g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(vec, vd, nv * 4, cudaMemcpyDeviceToHost, g_ctx.st));
    return sync_ctx();
}
void g4_apply_rope_neox(float *vec, int n_heads, int head_dim, int n_rot, int pos, float freq_base, float freq_scale,
                        const float *freq_factors) {
    (void)g4_apply_rope_neox_ex(vec, n_heads, head_dim, n_rot, pos, freq_base, freq_scale, freq_factors);
}

// logits_tied (main.c:1780-1796) with the greedy pick of sample_token.
int g4_logits_tied(float *logits, int *argmax, const float *x, const void *embd, int embd_type, int dim, int vocab,
                   float softcap) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!x || (!logits && !argmax)) { set_error(G4_ERR_ARG, "logits_tied: bad arguments"); return G4_ERR_ARG; }
    float dummy;
    G4_TRY(check_mm_args(&dummy, embd, dim, vocab, embd_type));
    G4_TRY(ctx_ready());
    const void *wd;
    G4_TRY(weight_dev(embd, embd_type, dim, vocab, &wd));
    const int nb = (dim + G4_QK - 1) / G4_QK;
    Carve cv;
    const size_t ox = cv.take((size_t)dim * 4), oq = cv.take((size_t)nb * G4_Q8_BYTES), oo = cv.take((size_t)vocab * 4),
                 ok = cv.take(8);
    G4_TRY(scratch_reserve(cv.off));
    uint8_t *s = g_ctx.scratch;
    float *xd = (float *)(s + ox), *od = (float *)(s + oo);
    unsigned long long *kd = (unsigned long long *)(s + ok), key = 0;
    G4_CUDA(cudaMemcpyAsync(xd, x, (size_t)dim * 4, cudaMemcpyHostToDevice, g_ctx.st));
    G4_CUDA(cudaMemsetAsync(kd, 0, 8, g_ctx.st));
    if (is_q8_type(embd_type)) G4_TRY(launch_quantize_q8k(xd, dim, s + oq, dim, 1, g_ctx.st));
    G4_TRY(gemv_any(od, xd, wd, dim, vocab, embd_type, s + oq, EPI_SOFTCAP_ARGMAX, kd, softcap));
    if (logits) G4_CUDA(cudaMemcpyAsync(logits, od, (size_t)vocab * 4, cudaMemcpyDeviceToHost, g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(&key, kd, 8, cudaMemcpyDeviceToHost, g_ctx.st));
    G4_TRY(sync_ctx());
    if (argmax) *argmax = argmax_key_index(key);
    return G4_OK;
}

// The per-head attention block of forward (main.c:1924-1950) on a caller
// window whose rows are laid out like the reference cache (row stride kv_stride).
int g4_attn_decode(float *out, const float *q, const float *k, const float *v, int nwin, int kv_stride, int n_heads,
                   int n_kv_heads, int hd) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!out || !q || nwin < 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || kv_stride < n_kv_heads * hd ||
        (hd != 64 && hd != 128 && hd != 256 && hd != 512) || (nwin > 0 && (!k || !v))) {
        set_error(G4_ERR_ARG, "attn_decode: bad arguments");
        return G4_ERR_ARG;
    }
    if (nwin == 0) {  // the reference zeroes the head output (main.c:1947-1949)
        memset(out, 0, sizeof(float) * (size_t)n_heads * hd);
        return G4_OK;
    }
    G4_TRY(ctx_ready());
    // repack rows [t][kvh*hd + i] into the device cache layout [kvh][t][hd]
    std::vector<float> kk((size_t)n_kv_heads * nwin * hd), vv(kk.size());
    for (int h = 0; h < n_kv_heads; h++)
        for (int t = 0; t < nwin; t++) {
            memcpy(&kk[((size_t)h * nwin + t) * hd], k + (size_t)t * kv_stride + (size_t)h * hd, sizeof(float) * hd);
            memcpy(&vv[((size_t)h * nwin + t) * hd], v + (size_t)t * kv_stride + (size_t)h * hd, sizeof(float) * hd);
        }
    const int ch = attn_chunk_size(), max_chunks = (nwin + ch - 1) / ch;
    const size_t qn = (size_t)n_heads * hd;
    Carve cv;
    const size_t oqd = cv.take(qn * 4), ok = cv.take(kk.size() * 4), ov = cv.take(vv.size() * 4),
                 op = cv.take((size_t)n_heads * max_chunks * (hd + 2) * 4), oo = cv.take(qn * 4), opos = cv.take(4),
                 octr = cv.take((size_t)n_kv_heads * 4);
    G4_TRY(scratch_reserve(cv.off));
    uint8_t *s = g_ctx.scratch;
    const int pos = nwin - 1;
    G4_CUDA(cudaMemcpyAsync(s + oqd, q, qn * 4, cudaMemcpyHostToDevice, g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(s + ok, kk.data(), kk.size() * 4, cudaMemcpyHostToDevice, g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(s + ov, vv.data(), vv.size() * 4, cudaMemcpyHostToDevice, g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(s + opos, &pos, 4, cudaMemcpyHostToDevice, g_ctx.st));
    G4_CUDA(cudaMemsetAsync(s + octr, 0, (size_t)n_kv_heads * 4, g_ctx.st));
    AttnLayer L{};
    L.hd = hd; L.n_rot = 0; L.n_heads = n_heads; L.n_kv = n_kv_heads;
    L.q = (const float *)(s + oqd); L.prep = 0;
    L.append = 0; L.ring = nwin; L.src_kc = (const float *)(s + ok); L.src_vc = (const float *)(s + ov);
    L.src_ring = nwin; L.window = 0; L.eps = 0.0f;
    L.qo = (float *)(s + oo); L.part = (float *)(s + op); L.counters = (int *)(s + octr); L.max_chunks = max_chunks;
    G4_TRY(launch_attention(L, 1, (const int *)(s + opos), nwin, g_ctx.st));
    G4_CUDA(cudaMemcpyAsync(out, s + oo, qn * 4, cudaMemcpyDeviceToHost, g_ctx.st));
    return sync_ctx();
}

}  // extern "C"

extern "C" {

int g4d_weight_upload(const void *host, int type, int n, int rows, void **dev) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!host || !dev || n <= 0 || rows <= 0) { set_error(G4_ERR_ARG, "weight_upload: bad arguments"); return G4_ERR_ARG; }
    float dummy;
    G4_TRY(check_mm_args(&dummy, host, n, rows, type));
    G4_TRY(ctx_ready());
    void *d = nullptr;
    G4_CUDA(cudaMalloc(&d, device_tensor_bytes(type, n, rows)));
    const int rc = upload_tensor(d, host, type, n, rows, g_ctx.st);
    if (rc) { cudaFree(d); return rc; }
    *dev = d;
    return G4_OK;
}

int g4d_free(void *dev) {
    G4_CUDA(cudaFree(dev));
    return G4_OK;
}

int g4d_quantize_row_q8_K(const float *x, g4_block_q8_K *y, int k, int batch, void *stream) {
    if (!x || !y || k < 0 || k % G4_QK || batch < 0) { set_error(G4_ERR_ARG, "quantize: k=%d must be a multiple of 256", k); return G4_ERR_ARG; }
    return launch_quantize_q8k(x, k, y, k, batch, (cudaStream_t)stream);
}

}  // extern "C"

// ---------------------------------------------------------------- tensor-core batch path of g4d_mm

static std::atomic<int> g_tc_min_batch{16};

struct TcScratchDev {  // per device; calls that use it must be ordered on the GPU
    uint8_t *bq = nullptr;
    size_t bq_bytes = 0;
    float *part = nullptr;
    size_t part_bytes = 0;
    int nsm = 0;
};
static TcScratchDev g_tcs[64];
static std::mutex g_tcs_mu;

static int tc_scratch(int n, int d, TcScratchDev **out) {
    int dev = 0;
    G4_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) { set_error(G4_ERR_NO_DEVICE, "device ordinal %d out of range", dev); return G4_ERR_NO_DEVICE; }
    std::lock_guard<std::mutex> lk(g_tcs_mu);
    TcScratchDev &S = g_tcs[dev];
    if (!S.nsm) {  // first use on this device
        G4_CUDA(cudaDeviceGetAttribute(&S.nsm, cudaDevAttrMultiProcessorCount, dev));
        G4_TRY(prime_tc_attrs());
        G4_TRY(prime_tc6_attrs());
        G4_TRY(prime_bf16tc_attrs());
    }
    const int tiles = (d + 127) / 128;
    const size_t bq = std::max(std::max(tc_operand_bytes(n), tc6_operand_bytes(n)), bf16tc_operand_bytes((n + 63) / 64 * 64)),
                 part = std::max(tc_part_bytes(d, n, S.nsm),
                                 (size_t)std::max(1, std::min(n / 64, S.nsm / tiles)) * 64 * d * sizeof(float));
    if (bq > S.bq_bytes || part > S.part_bytes) {
        G4_CUDA(cudaDeviceSynchronize());  // earlier calls may still use the old buffers
        if (bq > S.bq_bytes) {
            cudaFree(S.bq);
            S.bq = nullptr; S.bq_bytes = 0;
            G4_CUDA(cudaMalloc(&S.bq, bq));
            S.bq_bytes = bq;
        }
        if (part > S.part_bytes) {
            cudaFree(S.part);
            S.part = nullptr; S.part_bytes = 0;
            G4_CUDA(cudaMalloc(&S.part, part));
            S.part_bytes = part;
        }
    }
    *out = &S;
    return G4_OK;
}

// Q4_K/Q5_K rows against `batch` Q8_K activations (already in q8) on the
// tensor cores, in groups of up to 64 sequences.
static int mm_tc(float *o, const void *w, int n, int d, int type, const g4_block_q8_K *q8, int batch, cudaStream_t st) {
    TcScratchDev *S = nullptr;
    G4_TRY(tc_scratch(n, d, &S));
    CUtensorMap tm;
    G4_TRY(tc_weight_map(&tm, w, type, n, d));
    const int nb = n / G4_QK;
    float *yd = (float *)(S->bq + tc_yd_offset(n));
    for (int g0 = 0; g0 < batch; g0 += 64) {
        const int gb = batch - g0 < 64 ? batch - g0 : 64, np = tc_np(gb);
        G4_TRY(launch_tc_from_q8(type, (const uint8_t *)q8 + (size_t)g0 * nb * G4_Q8_BYTES, gb, n, np, S->bq, yd, st));
        G4_TRY(launch_gemm_tc(&tm, w, type, n, d, S->bq, yd, gb, np, o + (size_t)g0 * d, d, S->part, S->part_bytes,
                              nullptr, S->nsm, st, nullptr));
    }
    return G4_OK;
}

// Q6_K rows against `batch` fp32 activations on the tensor cores.
static int mm_tc6(float *o, const float *x, const void *w, int n, int d, int batch, cudaStream_t st) {
    TcScratchDev *S = nullptr;
    G4_TRY(tc_scratch(n, d, &S));
    alignas(64) unsigned char maps[512];
    if (tc6_maps_bytes() > sizeof(maps)) { set_error(G4_ERR_STATE, "tensor-map bundle size"); return G4_ERR_STATE; }
    G4_TRY(tc6_weight_maps(maps, w, n, d));
    float *ys = (float *)(S->bq + tc6_ys_offset(n));
    for (int g0 = 0; g0 < batch; g0 += 64) {
        const int gb = batch - g0 < 64 ? batch - g0 : 64, np = tc_np(gb);
        G4_TRY(launch_tc6_split(x + (size_t)g0 * n, n, gb, n, np, S->bq, ys, st));
        G4_TRY(launch_gemm_q6tc(maps, w, n, d, S->bq, ys, gb, np, o + (size_t)g0 * d, d, S->part, S->part_bytes,
                                nullptr, S->nsm, EPI_STORE, 0.0f, nullptr, st, nullptr));
    }
    return G4_OK;
}

// BF16 rows against `batch` fp32 activations on the tensor cores.
static int mm_tcbf(float *o, const float *x, const void *w, int n, int d, int batch, cudaStream_t st) {
    TcScratchDev *S = nullptr;
    G4_TRY(tc_scratch(n, d, &S));
    CUtensorMap tm;
    G4_TRY(bf16tc_weight_map(&tm, w, n, d));
    for (int g0 = 0; g0 < batch; g0 += 64) {
        const int gb = batch - g0 < 64 ? batch - g0 : 64, np = tc_np(gb);
        G4_TRY(launch_bf3_split(x + (size_t)g0 * n, n, gb, n, np, S->bq, st));
        G4_TRY(launch_gemm_bf16tc(&tm, n, d, S->bq, gb, np, o + (size_t)g0 * d, d, S->part, S->part_bytes,
                                  nullptr, S->nsm, EPI_STORE, nullptr, 0, st));
    }
    return G4_OK;
}

extern "C" {

// sample_token (main.c:2044-2112) on host logits: the top-k candidates are selected on the GPU,
// the temperature / top-p tail runs on the host with the reference's expressions.
int g4_sample_token(const float *logits, int n, float temp, float topp, int topk, uint64_t *rng) {
    if (!logits || n <= 0 || !rng) { set_error(G4_ERR_ARG, "sample_token: bad arguments"); return -1; }
    const int k = temp <= 0.0f ? 1 : (topk <= 0 || topk > n ? n : topk);
    if (k > 64) { set_error(G4_ERR_ARG, "sample_token: top-k %d above 64 is not supported", k); return -1; }
    std::lock_guard<std::mutex> lk(g_mu);
    if (ctx_ready()) return -1;
    Carve cv;
    const size_t o_l = cv.take((size_t)n * 4), o_v = cv.take(64 * 4), o_i = cv.take(64 * 4);
    if (scratch_reserve(cv.off)) return -1;
    float *dl = (float *)(g_ctx.scratch + o_l), *dv = (float *)(g_ctx.scratch + o_v);
    int *di = (int *)(g_ctx.scratch + o_i);
    float hv[64], p[64];
    int hi[64];
    cudaError_t ce = cudaMemcpyAsync(dl, logits, (size_t)n * 4, cudaMemcpyHostToDevice, g_ctx.st);
    if (ce != cudaSuccess) { cuda_fail(ce, "sample_token upload", __FILE__, __LINE__); return -1; }
    if (launch_topk(dl, n, n, k, dv, di, 1, g_ctx.st) != G4_OK) return -1;
    ce = cudaMemcpyAsync(hv, dv, (size_t)k * 4, cudaMemcpyDeviceToHost, g_ctx.st);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(hi, di, (size_t)k * 4, cudaMemcpyDeviceToHost, g_ctx.st);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(g_ctx.st);
    if (ce != cudaSuccess) { cuda_fail(ce, "sample_token", __FILE__, __LINE__); return -1; }
    if (temp <= 0.0f) return hi[0];  // first index of the largest logit (main.c:2045-2050)
    return sample_tail_host(hv, hi, k, temp, topp, rng, p);
}

int g4_set_gemv_rows(int on) { return g4::set_gemv_rows(on ? 1 : 0); }

int g4_set_tc_min_batch(int b) {
    if (b < 1) { set_error(G4_ERR_ARG, "tc min batch %d", b); return -1; }
    return g_tc_min_batch.exchange(b);
}

int g4d_mm(float *o, const float *x, const void *w, int n, int d, int type, g4_block_q8_K *q8, int q8_ready,
           int batch, void *stream) {
    G4_TRY(check_mm_args(o, w, n, d, type));
    if (batch <= 0) { set_error(G4_ERR_ARG, "mm: batch %d", batch); return G4_ERR_ARG; }
    cudaStream_t st = (cudaStream_t)stream;
    if (is_q8_type(type)) {
        if (!q8 || (!q8_ready && !x)) { set_error(G4_ERR_ARG, "mm: Q8_K buffer / x required"); return G4_ERR_ARG; }
        if (!q8_ready) G4_TRY(launch_quantize_q8k(x, n, q8, n, batch, st));
    } else if (!x) {
        set_error(G4_ERR_ARG, "mm: x is NULL");
        return G4_ERR_ARG;
    }
    if (type == G4_BF16 && batch >= g_tc_min_batch.load() && n % 64 == 0) return mm_tcbf(o, x, w, n, d, batch, st);
    if (type == G4_F32 || type == G4_F16 || type == G4_BF16)
        return launch_gemv_dense(w, type, n, d, x, n, o, d, batch, EPI_STORE, nullptr, 0, st);
    if (is_q8_type(type) && batch >= g_tc_min_batch.load()) return mm_tc(o, w, n, d, type, q8, batch, st);
    if (type == G4_Q6_K && batch >= g_tc_min_batch.load()) return mm_tc6(o, x, w, n, d, batch, st);
    GemvJobs jobs{};
    jobs.njobs = 1;
    GemvJob &J = jobs.j[0];
    J.w = w; J.type = type; J.n = n; J.rows = d;
    J.act = type == G4_Q6_K ? (const void *)x : (const void *)q8;
    J.act_stride = n; J.out = o; J.out_stride = d; J.epi = EPI_STORE;
    return launch_gemv_kquant(jobs, batch, st);
}

}  // extern "C"
