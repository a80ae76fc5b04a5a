// engine.cu — the device-resident decode step: forward of
// gemma4-4b/cpu-blas/main.c:1838-2029 for B sequences in lockstep, with the
// weights, KV cache and activations resident in HBM.
//
// One step (token ids -> next-token argmax) is a fixed launch sequence that
// reads the position and the token ids from device memory, so it is captured
// once per (batch, lm_mode, token source) into a CUDA graph and replayed for
// every position.  Greedy generation feeds each step's argmax keys straight
// into the next step's embedding lookup: no host round trip per token.
//
// Per layer l (main.c:1865-2010):
//   resnorm   x = (x + rms(p_raw)*post_norm[l-1]) * out_scale[l-1];
//             xn = rms(x)*attn_norm[l]; q8 = Q8_K(xn)
//   gemv      q = Wq.xn; k = Wk.xn; v = Wv.xn (l < 24), one grouped launch
//   attn      q/k norms, RoPE, KV append, split-K decode attention -> qo
//   gemv      o_raw = Wo.qo
//   resnorm   x += rms(o_raw)*post_attn_norm; xn = rms(x)*ffn_norm; q8
//   gemv      hb = gelu(Wgate.xn) * (Wup.xn)           (fused epilogue)
//   gemv      d_raw = Wdown.hb
//   resnorm   x += rms(d_raw)*post_ffw_norm
//   gemv      g = gelu(Winp_gate.x) * ple[l]           (fused epilogue)
//   gemv      p_raw = Wproj.g
// then the final residual, output norm, tied LM head + softcap + argmax.
#include <dlfcn.h>
#include <math.h>
#include <nccl.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <vector>

#include "g4_internal.cuh"
#include "g4_kernels.cuh"

namespace g4 {

struct LayerDev {
    int swa, hd, n_rot, qd, kvd, src;
    const void *wq, *wk, *wv, *wo, *gate, *up, *down, *inp_gate, *proj;
    int wq_t, wk_t, wv_t, wo_t, gate_t, up_t, down_t, inp_gate_t, proj_t;
    const float *attn_norm, *post_attn_norm, *ffn_norm, *post_ffw_norm, *q_norm, *k_norm, *post_norm, *out_scale;
    float *kc, *vc;
    int ring;
};

int prime_kernel_attrs();

}  // namespace g4

using namespace g4;

struct g4_engine {
    int device = 0;
    cudaStream_t st = nullptr;
    int dim = 0, hidden = 0, L = 0, nh = 0, nkv = 0, vocab = 0, pd = 0, window = 0, max_seq = 0, max_batch = 0;
    int qd_max = 0, kvd_max = 0, hd_max = 0;
    float eps = 0, softcap = 0, emb_scale = 0, ple_scale = 0, ctx_scale = 0, mix_scale = 0;
    std::vector<LayerDev> layers;
    const void *embd = nullptr, *ple_tok = nullptr, *ple_proj = nullptr;
    int embd_t = 0, ple_tok_t = 0, ple_proj_t = 0;
    const float *ple_proj_norm = nullptr, *norm_out = nullptr;
    float *hidden_src = nullptr;  // buffer holding the State.x view after the last step
    float2 *rope_swa = nullptr, *rope_full = nullptr;
    // state
    float *x = nullptr, *x2 = nullptr, *xn = nullptr, *xf = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *qn = nullptr,
          *qo = nullptr, *o_raw = nullptr, *hb = nullptr, *hb2 = nullptr, *d_raw = nullptr, *g = nullptr,
          *p_raw = nullptr, *ple_tokb = nullptr, *ple_ctx = nullptr, *ple = nullptr, *logits = nullptr,
          *attn_part = nullptr;
    uint8_t *q8 = nullptr;
    int q8_blocks = 0, max_chunks = 0;
    unsigned long long *keys = nullptr;
    int *d_tokens = nullptr, *d_next = nullptr, *d_pos = nullptr, *d_hist = nullptr, *attn_ctr = nullptr;
    int *h_pos = nullptr, *h_tok = nullptr, *h_err = nullptr;
    int *d_err = nullptr;  // bounded-wait status word written by the kernels
    // prefill: rows per g4_prefill call, the (sequence, position) of each row (device, pinned host)
    int prefill_cap = 0;
    // row-split LM head over `split_world` ranks (g4_engine_lm_split): this rank's rows [lm_r0, lm_r1)
    ncclComm_t comm = nullptr;
    int split_rank = 0, split_world = 1, lm_r0 = 0, lm_r1 = 0, lm_chunk = 0;
    float *xf_all = nullptr;
    unsigned long long *keys_loc = nullptr, *keys_all = nullptr;
    int *d_rowpos = nullptr, *d_rowseq = nullptr, *h_rows = nullptr;
    // sampler: top-k candidates per sequence (device and pinned host), recent tokens for the penalty
    float *cand_v = nullptr, *h_cand_v = nullptr;
    int *cand_i = nullptr, *h_cand_i = nullptr, *d_recent = nullptr, *d_nrec = nullptr;
    std::vector<void *> allocs;
    size_t dev_bytes = 0;
    std::map<long, cudaGraphExec_t> graphs;
    std::map<long, int> graph_kernels;  // kernel nodes per captured step
    std::map<long, float *> graph_hidden;  // where each step leaves State.x
    int last_lm_mode = 0, last_step_kernels = 0;
    // tensor-core path for the batched step (B >= tc_min_batch)
    struct alignas(64) MapBuf { unsigned char b[512]; };
    std::map<const void *, MapBuf> tmaps;  // tensor maps per weight matrix
    uint8_t *tcq = nullptr, *tc6 = nullptr, *tcb = nullptr;  // B operands (Q4_K/Q5_K, Q6_K, BF16)
    float *tc_part = nullptr;
    size_t tc_part_bytes = 0;
    int *tc_tickets = nullptr;  // per row tile, zero between launches (in-kernel merge of split tiles)
    // side lane: the V projection's tensor-core GEMM runs on its own stream, beside the Q+K launch
    // (both read the same normed input), with its own split partials and tickets
    cudaStream_t st2 = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    float *tc_part2 = nullptr;
    size_t tc_part2_bytes = 0;
    int *tc_tickets2 = nullptr;
    int attn_split_swa = 0, attn_split_full = 0;  // attention rows per CTA (0: the kernel's default)
    int nsm = 0, tc_min_batch = 2;  // measured: the tensor-core step wins from 2 sequences (5.2 vs 9.2 ms)
    std::mutex mu;
};

namespace {

// NCCL is loaded at run time (the copy a host process already loaded, e.g. torch's, when there
// is one), so the library has no link-time dependency on it.
struct NcclApi {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};
NcclApi g_nccl;
std::mutex g_nccl_mu;

int nccl_load() {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.ok) return G4_OK;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) { set_error(G4_ERR_STATE, "NCCL (libnccl.so.2) not found: %s", dlerror()); return G4_ERR_STATE; }
    g_nccl.get_unique_id = (ncclResult_t(*)(ncclUniqueId *))dlsym(h, "ncclGetUniqueId");
    g_nccl.comm_init_rank = (ncclResult_t(*)(ncclComm_t *, int, ncclUniqueId, int))dlsym(h, "ncclCommInitRank");
    g_nccl.all_gather = (ncclResult_t(*)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t))dlsym(h, "ncclAllGather");
    g_nccl.comm_destroy = (ncclResult_t(*)(ncclComm_t))dlsym(h, "ncclCommDestroy");
    g_nccl.error_string = (const char *(*)(ncclResult_t))dlsym(h, "ncclGetErrorString");
    if (!g_nccl.get_unique_id || !g_nccl.comm_init_rank || !g_nccl.all_gather || !g_nccl.comm_destroy || !g_nccl.error_string) {
        set_error(G4_ERR_STATE, "NCCL symbols missing");
        return G4_ERR_STATE;
    }
    g_nccl.ok = true;
    return G4_OK;
}
#define G4_NCCL(call)                                                                          \
    do {                                                                                       \
        const ncclResult_t r_ = (call);                                                        \
        if (r_ != ncclSuccess) {                                                               \
            set_error(G4_ERR_CUDA, "%s failed: %s", #call, g_nccl.error_string(r_));           \
            return G4_ERR_CUDA;                                                                \
        }                                                                                      \
    } while (0)

__global__ void lm_split_merge_kernel(const unsigned long long *keys_all, int world, int rank, int B, int chunk,
                                      unsigned long long *keys) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) keys[b] = lm_split_merge_one(keys_all, world, rank, B, chunk, b);
}

int dalloc(g4_engine *e, void **p, size_t bytes) {
    *p = nullptr;
    if (bytes == 0) bytes = 16;
    G4_CUDA(cudaMalloc(p, bytes));
    e->allocs.push_back(*p);
    e->dev_bytes += bytes;
    G4_CUDA(cudaMemsetAsync(*p, 0, bytes, e->st));
    return G4_OK;
}

template <class T>
int dalloc_t(g4_engine *e, T **p, size_t count) {
    void *v = nullptr;
    int rc = dalloc(e, &v, count * sizeof(T));
    *p = (T *)v;
    return rc;
}

int upload_w(g4_engine *e, const void *host, int type, int n, int rows, const void **out, const char *name) {
    *out = nullptr;
    if (!host) { set_error(G4_ERR_ARG, "engine: tensor %s missing", name); return G4_ERR_ARG; }
    if (!type_known(type)) { set_error(G4_ERR_TYPE, "engine: tensor %s has unsupported type %d", name, type); return G4_ERR_TYPE; }
    if ((type == G4_Q4_K || type == G4_Q5_K || type == G4_Q6_K) && n % G4_QK) {
        set_error(G4_ERR_ARG, "engine: tensor %s row length %d not a multiple of 256", name, n);
        return G4_ERR_ARG;
    }
    void *d = nullptr;
    int rc = dalloc(e, &d, device_tensor_bytes(type, n, rows));
    if (rc) return rc;
    rc = upload_tensor(d, host, type, n, rows, e->st);
    *out = d;
    return rc;
}

int upload_f(g4_engine *e, const float *host, int n, const float **out, const char *name, bool optional = false) {
    *out = nullptr;
    if (!host) {
        if (optional) return G4_OK;
        set_error(G4_ERR_ARG, "engine: vector %s missing", name);
        return G4_ERR_ARG;
    }
    void *d = nullptr;
    int rc = dalloc(e, &d, (size_t)n * 4);
    if (rc) return rc;
    G4_CUDA(cudaMemcpyAsync(d, host, (size_t)n * 4, cudaMemcpyHostToDevice, e->st));
    *out = (const float *)d;
    return G4_OK;
}

bool is_swa(const g4_model_desc *m, int l) {  // main.c:716-721
    if (m->swa_layers) return m->swa_layers[l] != 0;
    if (m->swa_pattern <= 0) return false;
    return (l % m->swa_pattern) < (m->swa_pattern - 1);
}

void destroy(g4_engine *e) {
    if (!e) return;
    cudaSetDevice(e->device);
    if (e->st) cudaStreamSynchronize(e->st);
    for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);
    if (e->comm) g_nccl.comm_destroy(e->comm);  // after the graphs that hold its collectives
    for (void *p : e->allocs) cudaFree(p);
    if (e->h_pos) cudaFreeHost(e->h_pos);
    if (e->h_tok) cudaFreeHost(e->h_tok);
    if (e->h_err) cudaFreeHost(e->h_err);
    if (e->h_cand_v) cudaFreeHost(e->h_cand_v);
    if (e->h_rows) cudaFreeHost(e->h_rows);
    if (e->h_cand_i) cudaFreeHost(e->h_cand_i);
    if (e->st2) cudaStreamSynchronize(e->st2);
    if (e->ev_fork) cudaEventDestroy(e->ev_fork);
    if (e->ev_join) cudaEventDestroy(e->ev_join);
    if (e->st2) cudaStreamDestroy(e->st2);
    if (e->st) cudaStreamDestroy(e->st);
    delete e;
}

#define TRY(x) do { int rc_ = (x); if (rc_) return rc_; } while (0)

// y[B][rows] = W . act for any weight type; act is fp32 [B][ld].  For
// Q4_K/Q5_K the activation is quantized into e->q8 unless q8_ready.
int gemv(g4_engine *e, const void *w, int type, int n, int rows, const float *act, int ld, bool q8_ready,
         float *out, int ldo, int B, int epi = EPI_STORE, const float *evec = nullptr, int ld_evec = 0,
         unsigned long long *keys = nullptr, float cap = 0.0f) {
    if (type == G4_F32 || type == G4_F16 || type == G4_BF16) {
        TRY(launch_gemv_dense(w, type, n, rows, act, ld, out, ldo, B, epi == EPI_SOFTCAP_ARGMAX ? EPI_STORE : epi,
                              evec, ld_evec, e->st));
        if (epi == EPI_SOFTCAP_ARGMAX) TRY(launch_softcap_argmax(out, rows, ldo, cap, keys, B, e->st));
        return G4_OK;
    }
    if (is_q8_type(type) && !q8_ready) TRY(launch_quantize_q8k(act, ld, e->q8, n, B, e->st));
    GemvJobs jobs{};
    jobs.njobs = 1;
    GemvJob &J = jobs.j[0];
    J.w = w; J.type = type; J.n = n; J.rows = rows;
    J.act = is_q8_type(type) ? (const void *)e->q8 : (const void *)act;
    J.act_stride = ld; J.out = out; J.out_stride = ldo; J.epi = epi; J.evec = evec; J.ld_evec = ld_evec;
    J.amax = keys; J.cap = cap;
    jobs.err = e->d_err;
    return launch_gemv_kquant(jobs, B, e->st);
}

bool is_kq(int t) { return t == G4_Q4_K || t == G4_Q5_K || t == G4_Q6_K; }

// Q and K of a layer share one tensor-core launch when both are Q4_K (tc_gemm_q4_pair); a GEMV of
// either matrix then follows the row order of that shared launch, so that the projections of a
// sequence are bit-identical at every batch size.
void qk_pair_orders(const g4_engine *e, const LayerDev &ly, GemvJob &J, int which) {
    J.ord = q4_row_order(ly.qd, ly.kvd, e->dim, e->nsm, which);
    J.ord2 = J.ord;
    J.explicit_order = 1;
}
bool qk_paired(const LayerDev &ly, bool has_kv) { return has_kv && ly.wq_t == G4_Q4_K && ly.wk_t == G4_Q4_K; }

// Whether a GEMM of this step runs on the tensor cores.  Dense (F32/F16/BF16) matrices always
// take the multi-sequence dense GEMV, whose per-row summation order does not depend on the batch
// (the per-layer-embedding matrices are small: 55 MB once per step, 1.3 MB per layer).
bool use_tc(const g4_engine *e, int B, int type, int epi) {
    if (!e->tcq || B < e->tc_min_batch) return false;
    if (!is_kq(type)) return false;
    return epi == EPI_STORE || (epi == EPI_SOFTCAP_ARGMAX && type == G4_Q6_K);
}

// Tensor maps of a weight matrix, encoded once per engine.
int tc_maps(g4_engine *e, const void *w, int type, int n, int rows, const void **out) {
    auto it = e->tmaps.find(w);
    if (it == e->tmaps.end()) {
        g4_engine::MapBuf mb{};
        if (type == G4_Q6_K) {
            if (tc6_maps_bytes() > sizeof(mb.b)) { set_error(G4_ERR_STATE, "tensor-map bundle size"); return G4_ERR_STATE; }
            TRY(tc6_weight_maps(mb.b, w, n, rows));
        } else if (type == G4_BF16) {
            TRY(bf16tc_weight_map(reinterpret_cast<CUtensorMap *>(mb.b), w, n, rows));
        } else {
            TRY(tc_weight_map(reinterpret_cast<CUtensorMap *>(mb.b), w, type, n, rows));
        }
        it = e->tmaps.emplace(w, mb).first;
    }
    *out = it->second.b;
    return G4_OK;
}

// y[B][rows] = W . act (fp32 [B][ld]) on the tensor cores, in groups of up
// to 64 sequences.  act_ready: the B operand of this activation is already
// in place (same activation as the previous call of the same type class).
struct TcLane {  // where a tensor-core GEMM runs: stream, split partials, tickets
    cudaStream_t st;
    float *part;
    size_t part_bytes;
    int *tickets;
};
int tc_gemm(g4_engine *e, const void *w, int type, int n, int rows, const float *act, int ld, bool act_ready,
            float *out, int ldo, int B, int epi = EPI_STORE, unsigned long long *keys = nullptr, float cap = 0.0f,
            const float *evec = nullptr, int ld_evec = 0, const TcLane *lane = nullptr) {
    const void *maps = nullptr;
    TRY(tc_maps(e, w, type, n, rows, &maps));
    const TcLane ln = lane ? *lane : TcLane{e->st, e->tc_part, e->tc_part_bytes, e->tc_tickets};
    if (B > 64) act_ready = false;
    for (int g0 = 0; g0 < B; g0 += 64) {
        const int gb = B - g0 < 64 ? B - g0 : 64, np = tc_np(gb);
        float *o = out ? out + (size_t)g0 * ldo : nullptr;
        if (type == G4_BF16) {
            if (!act_ready) TRY(launch_bf3_split(act + (size_t)g0 * ld, ld, gb, n, np, e->tcb, ln.st));
            TRY(launch_gemm_bf16tc((const CUtensorMap *)maps, n, rows, e->tcb, gb, np, o, ldo, ln.part,
                                   ln.part_bytes, e->d_err, e->nsm, epi,
                                   evec ? evec + (size_t)g0 * ld_evec : nullptr, ld_evec, ln.st));
        } else if (type == G4_Q6_K) {
            float *ys = (float *)(e->tc6 + tc6_ys_offset(n));
            if (!act_ready) TRY(launch_tc6_split(act + (size_t)g0 * ld, ld, gb, n, np, e->tc6, ys, ln.st));
            TRY(launch_gemm_q6tc(maps, w, n, rows, e->tc6, ys, gb, np, o, ldo, ln.part, ln.part_bytes,
                                 e->d_err, e->nsm, epi, cap, keys ? keys + g0 : nullptr, ln.st, ln.tickets));
        } else {
            float *yd = (float *)(e->tcq + tc_yd_offset(n));
            if (!act_ready) TRY(launch_tc_quant(type, act + (size_t)g0 * ld, ld, gb, n, np, e->tcq, yd, ln.st));
            TRY(launch_gemm_tc((const CUtensorMap *)maps, w, type, n, rows, e->tcq, yd, gb, np, o, ldo, ln.part,
                               ln.part_bytes, e->d_err, e->nsm, ln.st, ln.tickets));
        }
    }
    return G4_OK;
}

// Attention of layer l at the engine's current position: q/k/v raw projections in, the new K/V row
// normed, rotated and appended (layers that own a cache), qo out (main.c:1886-1950).
static AttnLayer attn_args(const g4_engine *e, int l) {
    const LayerDev &ly = e->layers[l];
    AttnLayer A{};
    A.hd = ly.hd; A.n_rot = ly.n_rot; A.n_heads = e->nh; A.n_kv = e->nkv;
    A.q = e->q; A.k = e->k; A.v = e->v; A.prep = 1;
    A.q_norm = ly.q_norm; A.k_norm = ly.k_norm;
    A.rope = ly.swa ? e->rope_swa : e->rope_full;
    A.append = l < G4_N_LAYER_KV; A.kc = ly.kc; A.vc = ly.vc; A.ring = ly.ring;
    const LayerDev &src = e->layers[ly.src];
    A.src_kc = src.kc; A.src_vc = src.vc; A.src_ring = src.ring;
    A.window = ly.swa ? e->window : 0;
    A.eps = e->eps; A.err = e->d_err;
    A.qo = e->qo; A.part = e->attn_part; A.counters = e->attn_ctr; A.max_chunks = e->max_chunks;
    A.split = ly.swa ? e->attn_split_swa : e->attn_split_full;
    // Steps run as whole CUDA graphs in stream order, so every cache row but `pos` was written by an
    // earlier graph launch (or fill_kv) that has completed; row `pos` of a shared-KV source is
    // written by an earlier kernel of this step and is only read after the dependency wait.
    A.early = 1;
    return A;
}

// Two Q4_K matrices that read the same activation (Q and K, or gate and up) in one tensor-core
// launch.  epi EPI_GELU_MUL: out = GELU(W act) * (W2 act) (out2 unused).
int tc_gemm_q4_pair(g4_engine *e, const void *w, int rows, float *out, int ldo, const void *w2, int rows2, float *out2,
                    int ldo2, int n, const float *act, int ld, bool act_ready, int B, int epi) {
    const void *m1 = nullptr, *m2 = nullptr;
    TRY(tc_maps(e, w, G4_Q4_K, n, rows, &m1));
    TRY(tc_maps(e, w2, G4_Q4_K, n, rows2, &m2));
    if (B > 64) act_ready = false;
    float *yd = (float *)(e->tcq + tc_yd_offset(n));
    for (int g0 = 0; g0 < B; g0 += 64) {
        const int gb = B - g0 < 64 ? B - g0 : 64, np = tc_np(gb);
        if (!act_ready) TRY(launch_tc_quant(G4_Q4_K, act + (size_t)g0 * ld, ld, gb, n, np, e->tcq, yd, e->st));
        TRY(launch_gemm_q4tc2((const CUtensorMap *)m1, w, rows, out + (size_t)g0 * ldo, ldo, (const CUtensorMap *)m2, w2,
                              rows2, out2 ? out2 + (size_t)g0 * ldo2 : nullptr, ldo2, n, e->tcq, yd, gb, np, e->tc_part,
                              e->tc_part_bytes, e->d_err, e->nsm, e->st, epi, e->tc_tickets));
    }
    return G4_OK;
}

// Let a residual/norm launch of a batched step also write the tensor-core B operand of its output
// for the GEMM that reads it next (one group of <= 64 sequences): saves that GEMM's own operand
// launch.  Returns whether the operand was attached.
bool attach_operand(g4_engine *e, ResNorm &r, int B, int type, int n) {
    if (!e->tcq || B > 64 || n != r.dim) return false;
    r.tc_np = tc_np(B);
    if (type == G4_Q4_K) {
        r.tc4_bq = e->tcq;
        r.tc4_yd = (float *)(e->tcq + tc_yd_offset(n));
    } else if (type == G4_Q6_K) {
        r.tc6_bq = e->tc6;
        r.tc6_ys = (float *)(e->tc6 + tc6_ys_offset(n));
    } else if (type == G4_BF16 && n % 64 == 0) {
        r.bf3_bq = e->tcb;
    } else {
        return false;
    }
    return true;
}

// Row-split tied LM head (after the output norm wrote xf[B][dim]): gather every rank's final hidden
// states, compute this rank's vocabulary rows for all of them (softcap + first-max key per
// sequence), gather the slice keys and merge them into this rank's sequences' keys: the argmax
// over the whole vocabulary with the reference's first-max rule (main.c:2045-2050).
int enqueue_lm_split(g4_engine *e, int B) {
    const int W = e->split_world, BT = W * B, rows = e->lm_r1 - e->lm_r0;
    G4_NCCL(g_nccl.all_gather(e->xf, e->xf_all, (size_t)B * e->dim, ncclFloat32, e->comm, e->st));
    G4_CUDA(cudaMemsetAsync(e->keys_loc, 0, sizeof(unsigned long long) * BT, e->st));
    const uint8_t *w = (const uint8_t *)e->embd + (size_t)e->lm_r0 * device_row_bytes(e->embd_t, e->dim);
    if (rows > 0) {
        if (use_tc(e, BT, e->embd_t, EPI_SOFTCAP_ARGMAX))
            TRY(tc_gemm(e, w, e->embd_t, e->dim, rows, e->xf_all, e->dim, false, nullptr, rows, BT, EPI_SOFTCAP_ARGMAX,
                        e->keys_loc, e->softcap));
        else
            TRY(gemv(e, w, e->embd_t, e->dim, rows, e->xf_all, e->dim, false, nullptr, rows, BT, EPI_SOFTCAP_ARGMAX,
                     nullptr, 0, e->keys_loc, e->softcap));
    }
    G4_NCCL(g_nccl.all_gather(e->keys_loc, e->keys_all, (size_t)BT, ncclUint64, e->comm, e->st));
    G4_CUDA(launch_pdl(lm_split_merge_kernel, dim3((B + 127) / 128), dim3(128), 0, e->st,
                       (const unsigned long long *)e->keys_all, W, e->split_rank, B, e->lm_chunk, e->keys));
    G4_LAUNCHED();
    return launch_keys_to_tokens(e->keys, e->d_next, B, e->st);
}

// One step for B rows.  Decode: row b is sequence b at the engine position.  Prefill (prefill =
// true, lm_mode 0): row b is sequence d_rowseq[b] at position d_rowpos[b]; every layer that owns a
// cache stores the K/V rows of all rows first, then each row attends with exactly the decode
// step's arithmetic, so a prefilled sequence is bit-identical to one decoded position by position.
int enqueue_step_unfused(g4_engine *e, int B, int lm_mode, bool from_keys, bool want_logits, bool prefill = false) {
    const int dim = e->dim, L = e->L, pd = e->pd;
    TRY(launch_embed_v(e->embd, e->embd_t, dim, (size_t)e->vocab, e->emb_scale, e->ple_tok, e->ple_tok_t, pd * L,
                       e->ple_scale, from_keys ? nullptr : e->d_tokens, e->keys, e->x, e->ple_tokb, B, e->st));
    if (use_tc(e, B, e->ple_proj_t, EPI_STORE) && (e->ple_proj_t != G4_BF16 || dim % 64 == 0))
        TRY(tc_gemm(e, e->ple_proj, e->ple_proj_t, dim, pd * L, e->x, dim, false, e->ple_ctx, pd * L, B));
    else
        TRY(gemv(e, e->ple_proj, e->ple_proj_t, dim, pd * L, e->x, dim, false, e->ple_ctx, pd * L, B));
    TRY(launch_ple_mix(e->ple_tokb, e->ple_ctx, e->ple_proj_norm, pd, L, e->ctx_scale, e->mix_scale, e->eps, e->ple,
                       B, e->st));
    // The residual stream lives in e->x, except between a per-layer-embedding gate GEMV that folded
    // the post-FFN residual into its prologue (it writes e->x2) and the next residual/norm launch.
    const float *xres = e->x;
    for (int l = 0; l < L; l++) {
        const LayerDev &ly = e->layers[l];
        const LayerDev *prev = l > 0 ? &e->layers[l - 1] : nullptr;
        const bool has_kv = l < G4_N_LAYER_KV;
        const bool tcq_l = use_tc(e, B, ly.wq_t, EPI_STORE);  // projections of this layer on the tensor cores
        const bool q8_in = !tcq_l && (is_q8_type(ly.wq_t) || (has_kv && (is_q8_type(ly.wk_t) || is_q8_type(ly.wv_t))));
        ResNorm r{};
        r.x_in = xres; r.delta = prev ? e->p_raw : nullptr; r.post_w = prev ? prev->post_norm : nullptr;
        r.scale = prev ? prev->out_scale : nullptr; r.x_out = e->x; r.pre_w = ly.attn_norm; r.xn_out = e->xn;
        r.q8_out = q8_in ? e->q8 : nullptr; r.dim = dim; r.eps = e->eps;
        // operands of xn for the Q (Q4_K) and V (Q6_K) tensor-core GEMMs, written by this launch
        bool ready8 = false, ready6 = false;  // operand of xn already laid out (Q4/Q5 class, Q6 class)
        if (tcq_l) {
            ready8 = ly.wq_t == G4_Q4_K && attach_operand(e, r, B, G4_Q4_K, dim);
            ready6 = has_kv && ly.wv_t == G4_Q6_K && use_tc(e, B, G4_Q6_K, EPI_STORE) &&
                     attach_operand(e, r, B, G4_Q6_K, dim);
        }
        TRY(launch_resnorm(r, B, e->st));
        xres = e->x;

        // Q / K / V projections (main.c:1884-1891): one launch per tensor type
        struct Proj { const void *w; int t; int rows; float *out; };
        Proj pr[3] = {{ly.wq, ly.wq_t, ly.qd, e->q}, {ly.wk, ly.wk_t, ly.kvd, e->k}, {ly.wv, ly.wv_t, ly.kvd, e->v}};
        const int np = has_kv ? 3 : 1;
        const int ktypes[3] = {G4_Q4_K, G4_Q5_K, G4_Q6_K};
        // V on the side stream, concurrently with the Q+K launch: both read xn; attention joins it
        const bool v_side = tcq_l && np == 3 && pr[2].t == G4_Q6_K && ready6 && e->st2 && e->tc_part2 &&
                            pr[0].t == G4_Q4_K && pr[1].t == G4_Q4_K;
        if (v_side) {
            G4_CUDA(cudaEventRecord(e->ev_fork, e->st));
            G4_CUDA(cudaStreamWaitEvent(e->st2, e->ev_fork, 0));
            const TcLane side{e->st2, e->tc_part2, e->tc_part2_bytes, e->tc_tickets2};
            TRY(tc_gemm(e, pr[2].w, pr[2].t, dim, pr[2].rows, e->xn, dim, true, pr[2].out, pr[2].rows, B, EPI_STORE,
                        nullptr, 0.0f, nullptr, 0, &side));
            G4_CUDA(cudaEventRecord(e->ev_join, e->st2));
        }
        if (tcq_l) {
            int i0 = 0;
            if (np > 1 && pr[0].t == G4_Q4_K && pr[1].t == G4_Q4_K) {  // Q and K in one launch
                TRY(tc_gemm_q4_pair(e, pr[0].w, pr[0].rows, pr[0].out, pr[0].rows, pr[1].w, pr[1].rows, pr[1].out,
                                    pr[1].rows, dim, e->xn, dim, ready8, B, EPI_STORE));
                ready8 = true;
                i0 = 2;
            }
            for (int i = i0; i < (v_side ? 2 : np); i++) {
                if (use_tc(e, B, pr[i].t, EPI_STORE)) {
                    bool &rdy = pr[i].t == G4_Q6_K ? ready6 : ready8;
                    // Q4_K and Q5_K operands differ in layout: reuse only within one type
                    const bool same = rdy && (pr[i].t == G4_Q6_K || i == 0 || pr[i].t == pr[i - 1].t);
                    TRY(tc_gemm(e, pr[i].w, pr[i].t, dim, pr[i].rows, e->xn, dim, same, pr[i].out, pr[i].rows, B));
                    rdy = true;
                } else {
                    TRY(gemv(e, pr[i].w, pr[i].t, dim, pr[i].rows, e->xn, dim, false, pr[i].out, pr[i].rows, B));
                }
            }
        }
        if (!tcq_l)
        for (int kt : ktypes) {
            GemvJobs jobs{};
            for (int i = 0; i < np; i++) {
                if (pr[i].t != kt) continue;
                GemvJob &J = jobs.j[jobs.njobs++];
                J.w = pr[i].w; J.type = pr[i].t; J.n = dim; J.rows = pr[i].rows;
                J.act = is_q8_type(pr[i].t) ? (const void *)e->q8 : (const void *)e->xn;
                J.act_stride = dim; J.out = pr[i].out; J.out_stride = pr[i].rows; J.epi = EPI_STORE;
                if (i < 2 && qk_paired(ly, has_kv)) qk_pair_orders(e, ly, J, i);
            }
            jobs.err = e->d_err;
            if (jobs.njobs) TRY(launch_gemv_kquant(jobs, B, e->st));
        }
        for (int i = 0; i < np && !tcq_l; i++)
            if (pr[i].t == G4_F32 || pr[i].t == G4_F16 || pr[i].t == G4_BF16)
                TRY(gemv(e, pr[i].w, pr[i].t, dim, pr[i].rows, e->xn, dim, false, pr[i].out, pr[i].rows, B));

        if (v_side) G4_CUDA(cudaStreamWaitEvent(e->st, e->ev_join, 0));
        // attention (main.c:1886-1950)
        if (prefill) {
            AttnLayer A = attn_args(e, l);
            A.row_pos = e->d_rowpos; A.row_seq = e->d_rowseq; A.early = 0;
            if (A.append) TRY(launch_kv_append(A, B, e->st));
            A.append = 0;
            TRY(launch_attention(A, B, e->d_pos, e->max_seq, e->st));
        }
        // the merging attention CTAs quantize qo into the Q4_K output projection's operand
        const bool o_fused = !prefill && use_tc(e, B, ly.wo_t, EPI_STORE) && ly.wo_t == G4_Q4_K && B <= 64 &&
                             ly.hd <= 256 && ((e->nh / e->nkv) * ly.hd) % G4_QK == 0;
        if (!prefill) {
            AttnLayer A = attn_args(e, l);
            if (o_fused) {
                A.op_bq = e->tcq;
                A.op_yd = (float *)(e->tcq + tc_yd_offset(ly.qd));
                A.op_np = tc_np(B);
            }
            TRY(launch_attention(A, B, e->d_pos, e->max_seq, e->st));
        }

        // output projection + post-attention norm + residual, FFN pre-norm (1959-1975)
        if (use_tc(e, B, ly.wo_t, EPI_STORE))
            TRY(tc_gemm(e, ly.wo, ly.wo_t, ly.qd, dim, e->qo, ly.qd, o_fused, e->o_raw, dim, B));
        else
            TRY(gemv(e, ly.wo, ly.wo_t, ly.qd, dim, e->qo, ly.qd, false, e->o_raw, dim, B));
        const bool tc_ffn = use_tc(e, B, ly.gate_t, EPI_STORE) && use_tc(e, B, ly.up_t, EPI_STORE);
        const bool q8_ffn = !tc_ffn && (is_q8_type(ly.gate_t) || is_q8_type(ly.up_t));
        ResNorm r2{};
        r2.x_in = e->x; r2.delta = e->o_raw; r2.post_w = ly.post_attn_norm; r2.x_out = e->x; r2.pre_w = ly.ffn_norm;
        r2.xn_out = e->xn; r2.q8_out = q8_ffn ? e->q8 : nullptr; r2.dim = dim; r2.eps = e->eps;
        const bool pair_ffn = tc_ffn && ly.gate_t == G4_Q4_K && ly.up_t == G4_Q4_K;
        const bool ffn_ready = pair_ffn && attach_operand(e, r2, B, G4_Q4_K, dim);
        TRY(launch_resnorm(r2, B, e->st));

        // gate / up with the GELU product fused (1976-1978)
        const bool kq = !(ly.gate_t == G4_F32 || ly.gate_t == G4_F16 || ly.gate_t == G4_BF16);
        if (pair_ffn) {  // one launch, GELU product in its merge
            TRY(tc_gemm_q4_pair(e, ly.gate, e->hidden, e->hb, e->hidden, ly.up, e->hidden, nullptr, e->hidden, dim, e->xn,
                                dim, ffn_ready, B, EPI_GELU_MUL));
        } else if (tc_ffn) {  // gate and up share the activation operand; GELU product as its own pass
            TRY(tc_gemm(e, ly.gate, ly.gate_t, dim, e->hidden, e->xn, dim, false, e->hb, e->hidden, B));
            TRY(tc_gemm(e, ly.up, ly.up_t, dim, e->hidden, e->xn, dim, ly.up_t == ly.gate_t, e->hb2, e->hidden, B));
            TRY(launch_gelu_mul(e->hb, e->hb2, (size_t)B * e->hidden, e->st));
        } else if (kq && ly.gate_t == ly.up_t) {
            GemvJobs fj{};
            fj.njobs = 1;
            GemvJob &J = fj.j[0];
            J.w = ly.gate; J.w2 = ly.up; J.type = ly.gate_t; J.n = dim; J.rows = e->hidden;
            J.act = is_q8_type(ly.gate_t) ? (const void *)e->q8 : (const void *)e->xn;
            J.act_stride = dim; J.out = e->hb; J.out_stride = e->hidden; J.epi = EPI_GELU_MUL;
            fj.err = e->d_err;
            TRY(launch_gemv_kquant(fj, B, e->st));
        } else {
            TRY(gemv(e, ly.gate, ly.gate_t, dim, e->hidden, e->xn, dim, is_q8_type(ly.gate_t), e->hb, e->hidden, B));
            TRY(gemv(e, ly.up, ly.up_t, dim, e->hidden, e->xn, dim, is_q8_type(ly.up_t), e->hb2, e->hidden, B));
            TRY(launch_gelu_mul(e->hb, e->hb2, (size_t)B * e->hidden, e->st));
        }
        // down projection, post-FFN norm + residual (1979-1984)
        if (use_tc(e, B, ly.down_t, EPI_STORE))
            TRY(tc_gemm(e, ly.down, ly.down_t, e->hidden, dim, e->hb, e->hidden, false, e->d_raw, dim, B));
        else
            TRY(gemv(e, ly.down, ly.down_t, e->hidden, dim, e->hb, e->hidden, false, e->d_raw, dim, B));
        ResNorm r3{};
        r3.x_in = e->x; r3.delta = e->d_raw; r3.post_w = ly.post_ffw_norm; r3.x_out = e->x; r3.dim = dim;
        r3.eps = e->eps;
        const bool tc_gate = use_tc(e, B, ly.inp_gate_t, EPI_GELU_SCALE) && (ly.inp_gate_t != G4_BF16 || dim % 64 == 0);
        const bool dense_gate = ly.inp_gate_t == G4_F32 || ly.inp_gate_t == G4_F16 || ly.inp_gate_t == G4_BF16;
        // per-layer embedding injection (1986-1997)
        if (!tc_gate && dense_gate) {
            // the dense gate GEMV computes x + rmsnorm(down)*w itself (each CTA for its sequences, one
            // CTA per group writes it to e->x2): no separate residual launch
            Prologue P{};
            P.x_in = e->x; P.delta = e->d_raw; P.post_w = ly.post_ffw_norm; P.x_out = e->x2; P.dim = dim; P.eps = e->eps;
            TRY(launch_gemv_dense(ly.inp_gate, ly.inp_gate_t, dim, pd, e->x2, dim, e->g, pd, B, EPI_GELU_SCALE,
                                  e->ple + (size_t)l * pd, pd * L, e->st, &P, 1));
            xres = e->x2;
        } else {
            const bool gate_ready = tc_gate && attach_operand(e, r3, B, ly.inp_gate_t, dim);
            TRY(launch_resnorm(r3, B, e->st));
            if (tc_gate)
                TRY(tc_gemm(e, ly.inp_gate, ly.inp_gate_t, dim, pd, e->x, dim, gate_ready, e->g, pd, B, EPI_GELU_SCALE,
                            nullptr, 0.0f, e->ple + (size_t)l * pd, pd * L));
            else
                TRY(gemv(e, ly.inp_gate, ly.inp_gate_t, dim, pd, e->x, dim, false, e->g, pd, B, EPI_GELU_SCALE,
                         e->ple + (size_t)l * pd, pd * L));
        }
        if (use_tc(e, B, ly.proj_t, EPI_STORE) && (ly.proj_t != G4_BF16 || pd % 64 == 0))
            TRY(tc_gemm(e, ly.proj, ly.proj_t, pd, dim, e->g, pd, false, e->p_raw, dim, B));
        else
            TRY(gemv(e, ly.proj, ly.proj_t, pd, dim, e->g, pd, false, e->p_raw, dim, B));
    }
    // last residual + out_scale (1995-2003), output norm (2021)
    const LayerDev &last = e->layers[L - 1];
    ResNorm rf{};
    rf.x_in = xres; rf.delta = e->p_raw; rf.post_w = last.post_norm; rf.scale = last.out_scale; rf.x_out = e->x;
    rf.pre_w = lm_mode ? e->norm_out : nullptr; rf.xn_out = e->xf; rf.dim = dim; rf.eps = e->eps;
    const bool tc_head = lm_mode && !e->comm && use_tc(e, B, e->embd_t, EPI_SOFTCAP_ARGMAX);
    const bool head_ready = tc_head && attach_operand(e, rf, B, e->embd_t, dim);
    TRY(launch_resnorm(rf, B, e->st));
    if (!lm_mode) return G4_OK;
    if (e->comm) return enqueue_lm_split(e, B);
    // tied LM head + softcap + first-max argmax (1780-1796, 2045-2050)
    const bool dense = e->embd_t == G4_F32 || e->embd_t == G4_F16 || e->embd_t == G4_BF16;
    if (tc_head)
        TRY(tc_gemm(e, e->embd, e->embd_t, dim, e->vocab, e->xf, dim, head_ready, want_logits ? e->logits : nullptr,
                    e->vocab, B, EPI_SOFTCAP_ARGMAX, e->keys, e->softcap));
    else
        TRY(gemv(e, e->embd, e->embd_t, dim, e->vocab, e->xf, dim, false, (want_logits || dense) ? e->logits : nullptr,
                 e->vocab, B, EPI_SOFTCAP_ARGMAX, nullptr, 0, e->keys, e->softcap));
    TRY(launch_keys_to_tokens(e->keys, e->d_next, B, e->st));
    return G4_OK;
}

bool is_dense(int t) { return t == G4_F32 || t == G4_F16 || t == G4_BF16; }

// One GEMV whose activation is either computed by a fused prologue (pro != null)
// or read from act (fp32 [B][ld]; quantized to Q8_K first for Q4_K/Q5_K).
int gemv_p(g4_engine *e, const void *w, int type, int n, int rows, const Prologue *pro, int writer, const float *act,
           int ld, float *out, int ldo, int B, int epi = EPI_STORE, const float *evec = nullptr, int ld_evec = 0,
           unsigned long long *keys = nullptr, float cap = 0.0f) {
    if (is_dense(type)) {
        TRY(launch_gemv_dense(w, type, n, rows, act, ld, out, ldo, B, epi == EPI_SOFTCAP_ARGMAX ? EPI_STORE : epi,
                              evec, ld_evec, e->st, pro, writer));
        if (epi == EPI_SOFTCAP_ARGMAX) TRY(launch_softcap_argmax(out, rows, ldo, cap, keys, B, e->st));
        return G4_OK;
    }
    GemvJobs jobs{};
    jobs.njobs = 1;
    GemvJob &J = jobs.j[0];
    J.w = w; J.type = type; J.n = n; J.rows = rows;
    J.out = out; J.out_stride = ldo; J.epi = epi; J.evec = evec; J.ld_evec = ld_evec; J.amax = keys; J.cap = cap;
    if (pro) {
        jobs.has_pro = 1;
        jobs.pro = *pro;
        jobs.pro_writer = writer;
    } else if (is_q8_type(type)) {
        TRY(launch_quantize_q8k(act, ld, e->q8, n, B, e->st));
        J.act = e->q8;
    } else {
        J.act = act;
        J.act_stride = ld;
    }
    jobs.err = e->d_err;
    return launch_gemv_kquant(jobs, B, e->st);
}

// The decode step for B <= 8: every residual/norm/quantize step runs as the
// prologue of the GEMV that consumes it (8 launches per layer).
int enqueue_step_fused(g4_engine *e, int B, int lm_mode, bool from_keys, bool want_logits) {
    const int dim = e->dim, L = e->L, pd = e->pd;
    TRY(launch_embed_v(e->embd, e->embd_t, dim, (size_t)e->vocab, e->emb_scale, e->ple_tok, e->ple_tok_t, pd * L,
                       e->ple_scale, from_keys ? nullptr : e->d_tokens, e->keys, e->x, e->ple_tokb, B, e->st));
    TRY(gemv_p(e, e->ple_proj, e->ple_proj_t, dim, pd * L, nullptr, 0, e->x, dim, e->ple_ctx, pd * L, B));
    TRY(launch_ple_mix(e->ple_tokb, e->ple_ctx, e->ple_proj_norm, pd, L, e->ctx_scale, e->mix_scale, e->eps, e->ple,
                       B, e->st));
    float *cur = e->x, *nxt = e->x2;
    auto flip = [&]() { float *t = cur; cur = nxt; nxt = t; };
    for (int l = 0; l < L; l++) {
        const LayerDev &ly = e->layers[l];
        const LayerDev *prev = l > 0 ? &e->layers[l - 1] : nullptr;
        const bool has_kv = l < G4_N_LAYER_KV;
        // x = (x + rms(p_raw)*post_norm[l-1]) * out_scale[l-1]; act = rms(x)*attn_norm[l]
        Prologue pa{};
        pa.x_in = cur; pa.delta = prev ? e->p_raw : nullptr; pa.post_w = prev ? prev->post_norm : nullptr;
        pa.scale = prev ? prev->out_scale : nullptr; pa.x_out = nxt; pa.pre_w = ly.attn_norm; pa.dim = dim;
        pa.eps = e->eps;
        struct Proj { const void *w; int t; int rows; float *out; };
        Proj pr[3] = {{ly.wq, ly.wq_t, ly.qd, e->q}, {ly.wk, ly.wk_t, ly.kvd, e->k}, {ly.wv, ly.wv_t, ly.kvd, e->v}};
        const int np = has_kv ? 3 : 1;
        int writer = 1;
        const int ktypes[3] = {G4_Q4_K, G4_Q5_K, G4_Q6_K};
        for (int kt : ktypes) {
            GemvJobs jobs{};
            for (int i = 0; i < np; i++) {
                if (pr[i].t != kt) continue;
                GemvJob &J = jobs.j[jobs.njobs++];
                J.w = pr[i].w; J.type = kt; J.n = dim; J.rows = pr[i].rows; J.out = pr[i].out;
                J.out_stride = pr[i].rows; J.epi = EPI_STORE;
                if (i < 2 && qk_paired(ly, has_kv)) qk_pair_orders(e, ly, J, i);
            }
            if (!jobs.njobs) continue;
            jobs.has_pro = 1; jobs.pro = pa; jobs.pro_writer = writer; jobs.err = e->d_err;
            writer = 0;
            TRY(launch_gemv_kquant(jobs, B, e->st));
        }
        for (int i = 0; i < np; i++)
            if (is_dense(pr[i].t)) {
                TRY(gemv_p(e, pr[i].w, pr[i].t, dim, pr[i].rows, &pa, writer, nullptr, dim, pr[i].out, pr[i].rows, B));
                writer = 0;
            }
        flip();  // cur = x after the PLE residual of layer l-1

        TRY(launch_attention(attn_args(e, l), B, e->d_pos, e->max_seq, e->st));

        // O projection: the Q8_K quantization of qo is its prologue
        Prologue po{};
        po.x_in = e->qo; po.dim = ly.qd; po.eps = e->eps;
        TRY(gemv_p(e, ly.wo, ly.wo_t, ly.qd, dim, is_q8_type(ly.wo_t) ? &po : nullptr, 0, e->qo, ly.qd, e->o_raw, dim, B));

        // x += rms(o_raw)*post_attn_norm; act = rms(x)*ffn_norm; gelu(gate)*up
        Prologue pf{};
        pf.x_in = cur; pf.delta = e->o_raw; pf.post_w = ly.post_attn_norm; pf.x_out = nxt; pf.pre_w = ly.ffn_norm;
        pf.dim = dim; pf.eps = e->eps;
        if (!is_dense(ly.gate_t) && ly.gate_t == ly.up_t) {
            GemvJobs fj{};
            fj.njobs = 1;
            GemvJob &J = fj.j[0];
            J.w = ly.gate; J.w2 = ly.up; J.type = ly.gate_t; J.n = dim; J.rows = e->hidden;
            J.out = e->hb; J.out_stride = e->hidden; J.epi = EPI_GELU_MUL;
            fj.has_pro = 1; fj.pro = pf; fj.pro_writer = 1; fj.err = e->d_err;
            TRY(launch_gemv_kquant(fj, B, e->st));
        } else {
            TRY(gemv_p(e, ly.gate, ly.gate_t, dim, e->hidden, &pf, 1, nullptr, dim, e->hb, e->hidden, B));
            TRY(gemv_p(e, ly.up, ly.up_t, dim, e->hidden, &pf, 0, nullptr, dim, e->hb2, e->hidden, B));
            TRY(launch_gelu_mul(e->hb, e->hb2, (size_t)B * e->hidden, e->st));
        }
        flip();

        // down projection (Q8_K quantization of hb as the prologue when needed)
        Prologue pd_{};
        pd_.x_in = e->hb; pd_.dim = e->hidden; pd_.eps = e->eps;
        TRY(gemv_p(e, ly.down, ly.down_t, e->hidden, dim, is_q8_type(ly.down_t) ? &pd_ : nullptr, 0, e->hb,
                   e->hidden, e->d_raw, dim, B));

        // x += rms(d_raw)*post_ffw_norm; g = gelu(inp_gate.x) * ple[l]; p_raw = proj.g
        Prologue pg{};
        pg.x_in = cur; pg.delta = e->d_raw; pg.post_w = ly.post_ffw_norm; pg.x_out = nxt; pg.dim = dim; pg.eps = e->eps;
        TRY(gemv_p(e, ly.inp_gate, ly.inp_gate_t, dim, pd, &pg, 1, nullptr, dim, e->g, pd, B, EPI_GELU_SCALE,
                   e->ple + (size_t)l * pd, pd * L));
        flip();
        Prologue pp{};
        pp.x_in = e->g; pp.dim = pd; pp.eps = e->eps;
        TRY(gemv_p(e, ly.proj, ly.proj_t, pd, dim, is_q8_type(ly.proj_t) ? &pp : nullptr, 0, e->g, pd, e->p_raw, dim, B));
    }
    const LayerDev &last = e->layers[L - 1];
    Prologue pl{};
    pl.x_in = cur; pl.delta = e->p_raw; pl.post_w = last.post_norm; pl.scale = last.out_scale; pl.x_out = nxt;
    pl.pre_w = e->norm_out; pl.xn_out = e->xf; pl.dim = dim; pl.eps = e->eps;
    if (!lm_mode) {  // residual only (State.x after a prefill forward)
        ResNorm rf{};
        rf.x_in = cur; rf.delta = e->p_raw; rf.post_w = last.post_norm; rf.scale = last.out_scale; rf.x_out = nxt;
        rf.dim = dim; rf.eps = e->eps;
        TRY(launch_resnorm(rf, B, e->st));
        e->hidden_src = nxt;
        return G4_OK;
    }
    e->hidden_src = e->xf;
    if (e->comm) {  // the output norm on its own, then the row-split head
        ResNorm rf{};
        rf.x_in = cur; rf.delta = e->p_raw; rf.post_w = last.post_norm; rf.scale = last.out_scale; rf.x_out = nxt;
        rf.pre_w = e->norm_out; rf.xn_out = e->xf; rf.dim = dim; rf.eps = e->eps;
        TRY(launch_resnorm(rf, B, e->st));
        return enqueue_lm_split(e, B);
    }
    const bool dense = is_dense(e->embd_t);
    TRY(gemv_p(e, e->embd, e->embd_t, dim, e->vocab, &pl, 1, nullptr, dim, (want_logits || dense) ? e->logits : nullptr,
               e->vocab, B, EPI_SOFTCAP_ARGMAX, nullptr, 0, e->keys, e->softcap));
    TRY(launch_keys_to_tokens(e->keys, e->d_next, B, e->st));
    return G4_OK;
}

int enqueue_step(g4_engine *e, int B, int lm_mode, bool from_keys, bool want_logits) {
    // below the tensor-core threshold every residual/norm/quantize step runs inside the GEMV that consumes it
    if (B <= kFusedMaxBatch && (B < e->tc_min_batch || !e->tcq) && e->dim % G4_QK == 0)
        return enqueue_step_fused(e, B, lm_mode, from_keys, want_logits);
    e->hidden_src = lm_mode ? e->xf : e->x;
    return enqueue_step_unfused(e, B, lm_mode, from_keys, want_logits);
}

int run_step(g4_engine *e, int B, int lm_mode, bool from_keys, bool want_logits) {
    const long key = ((long)B << 8) | ((long)lm_mode << 2) | ((long)from_keys << 1) | (long)want_logits;
    auto it = e->graphs.find(key);
    if (it == e->graphs.end()) {
        cudaGraph_t g = nullptr;
        G4_CUDA(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_step(e, B, lm_mode, from_keys, want_logits);
        cudaError_t ce = cudaStreamEndCapture(e->st, &g);
        if (rc) { if (g) cudaGraphDestroy(g); return rc; }
        if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture", __FILE__, __LINE__);
        size_t nn = 0;
        int nk = 0;
        if (cudaGraphGetNodes(g, nullptr, &nn) == cudaSuccess && nn) {
            std::vector<cudaGraphNode_t> nodes(nn);
            if (cudaGraphGetNodes(g, nodes.data(), &nn) == cudaSuccess)
                for (auto nd : nodes) {
                    cudaGraphNodeType ty;
                    if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) nk++;
                }
        }
        e->graph_kernels[key] = nk;
        e->graph_hidden[key] = e->hidden_src;
        cudaGraphExec_t ge = nullptr;
        ce = cudaGraphInstantiate(&ge, g, 0);
        cudaGraphDestroy(g);
        if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate", __FILE__, __LINE__);
        it = e->graphs.emplace(key, ge).first;
    }
    G4_CUDA(cudaGraphLaunch(it->second, e->st));
    e->last_lm_mode = lm_mode;
    e->last_step_kernels = e->graph_kernels[key];
    e->hidden_src = e->graph_hidden[key];
    return G4_OK;
}

// Read back the kernels' status word (enqueue before the stream sync).
int enqueue_err_check(g4_engine *e) {
    G4_CUDA(cudaMemcpyAsync(e->h_err, e->d_err, sizeof(int), cudaMemcpyDeviceToHost, e->st));
    return G4_OK;
}
int err_after_sync(g4_engine *e) {
    if (*e->h_err) {
        const int code = *e->h_err;
        *e->h_err = 0;
        cudaMemsetAsync(e->d_err, 0, sizeof(int), e->st);
        set_error(code, "a device-side wait gave up (bounded wait timeout); results are invalid");
        return code;
    }
    return G4_OK;
}

int set_pos(g4_engine *e, int pos) {
    if (pos < 0 || pos >= e->max_seq) {
        set_error(G4_ERR_STATE, "position %d outside [0, max_seq=%d)", pos, e->max_seq);
        return G4_ERR_STATE;
    }
    G4_CUDA(cudaMemcpyAsync(e->d_pos, e->h_pos + pos, 4, cudaMemcpyHostToDevice, e->st));
    return G4_OK;
}

int stage_tokens(g4_engine *e, const int *tokens, int B, int pos) {
    int *h = e->h_tok + (size_t)pos * e->max_batch;
    for (int b = 0; b < B; b++) {
        if (tokens[b] < 0 || tokens[b] >= e->vocab) {
            set_error(G4_ERR_ARG, "token %d outside the vocabulary (%d)", tokens[b], e->vocab);
            return G4_ERR_ARG;
        }
        h[b] = tokens[b];
    }
    G4_CUDA(cudaMemcpyAsync(e->d_tokens, h, sizeof(int) * B, cudaMemcpyHostToDevice, e->st));
    return G4_OK;
}

// After a step that wrote the softcapped logits of B sequences: the repetition penalty over each
// sequence's recent tokens (recent[b][0..n_recent[b]) in order, host arrays; penalty <= 1: none),
// the top-k candidates on the device, then the sampling tail per sequence on the host
// (main.c:2044-2126).  k = 1 for temp <= 0 (the first largest logit).
int sample_after_step(g4_engine *e, int B, float temp, float topp, int topk, float penalty, const int *recent,
                      int recent_ld, const int *n_recent, uint64_t *rng, int *next) {
    const int k = temp <= 0.0f ? 1 : (topk <= 0 || topk > e->vocab ? e->vocab : topk);
    if (k > 64) { set_error(G4_ERR_ARG, "sampling: top-k %d above 64 is not supported", k); return G4_ERR_ARG; }
    if (penalty > 1.0f && recent && n_recent) {
        for (int b = 0; b < B; b++)
            if (n_recent[b] < 0 || n_recent[b] > e->max_seq || n_recent[b] > recent_ld) {
                set_error(G4_ERR_ARG, "sampling: %d recent tokens for sequence %d", n_recent[b], b);
                return G4_ERR_ARG;
            }
        G4_CUDA(cudaMemcpy2DAsync(e->d_recent, sizeof(int) * e->max_seq, recent, sizeof(int) * recent_ld,
                                  sizeof(int) * std::min(recent_ld, e->max_seq), B, cudaMemcpyHostToDevice, e->st));
        G4_CUDA(cudaMemcpyAsync(e->d_nrec, n_recent, sizeof(int) * B, cudaMemcpyHostToDevice, e->st));
        TRY(launch_rep_penalty(e->logits, e->vocab, e->d_recent, e->max_seq, e->d_nrec, e->vocab, penalty, B, e->st));
    }
    TRY(launch_topk(e->logits, e->vocab, e->vocab, k, e->cand_v, e->cand_i, B, e->st));
    G4_CUDA(cudaMemcpyAsync(e->h_cand_v, e->cand_v, sizeof(float) * B * k, cudaMemcpyDeviceToHost, e->st));
    G4_CUDA(cudaMemcpyAsync(e->h_cand_i, e->cand_i, sizeof(int) * B * k, cudaMemcpyDeviceToHost, e->st));
    TRY(enqueue_err_check(e));
    G4_CUDA(cudaStreamSynchronize(e->st));
    TRY(err_after_sync(e));
    float p[64];
    for (int b = 0; b < B; b++)
        next[b] = temp <= 0.0f ? e->h_cand_i[b * k]
                               : sample_tail_host(e->h_cand_v + b * k, e->h_cand_i + b * k, k, temp, topp, rng + b, p);
    return G4_OK;
}

int create(g4_engine *e, const g4_model_desc *m, int max_seq, int max_batch, int prefill_rows) {
    if (!m || max_seq <= 0 || max_batch <= 0 || prefill_rows < 0) { set_error(G4_ERR_ARG, "engine: bad arguments"); return G4_ERR_ARG; }
    e->prefill_cap = prefill_rows;
    if (m->dim <= 0 || m->dim % G4_QK || m->hidden_dim <= 0 || m->n_layers <= 0 || m->n_heads <= 0 ||
        m->n_kv_heads <= 0 || m->n_heads % m->n_kv_heads || m->vocab_size <= 0 || m->ple_dim <= 0 || m->ple_dim > 1024 ||
        m->dim > 12288) {
        set_error(G4_ERR_ARG, "engine: unsupported model shape");
        return G4_ERR_ARG;
    }
    e->dim = m->dim; e->hidden = m->hidden_dim; e->L = m->n_layers; e->nh = m->n_heads; e->nkv = m->n_kv_heads;
    e->vocab = m->vocab_size; e->pd = m->ple_dim; e->window = m->sliding_window; e->max_seq = max_seq;
    e->max_batch = max_batch; e->eps = m->norm_eps; e->softcap = m->logit_softcapping;
    // scale constants exactly as the reference computes them (main.c:1851, 1757, 1762, 1769)
    e->emb_scale = sqrtf((float)m->dim);
    e->ple_scale = sqrtf((float)m->ple_dim);
    e->ctx_scale = 1.0f / sqrtf((float)m->dim);
    e->mix_scale = 1.0f / sqrtf(2.0f);

    G4_CUDA(cudaSetDevice(e->device));
    cudaDeviceProp p;
    G4_CUDA(cudaGetDeviceProperties(&p, e->device));
    if (p.major != 10) { set_error(G4_ERR_NO_DEVICE, "device %d is not sm_100", e->device); return G4_ERR_NO_DEVICE; }
    G4_CUDA(cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking));
    TRY(prime_kernel_attrs());

    const int L = e->L, dim = e->dim, pd = e->pd;
    TRY(upload_w(e, m->embd, m->embd_t, dim, e->vocab, &e->embd, "token_embd"));
    e->embd_t = m->embd_t;
    TRY(upload_w(e, m->ple_tok, m->ple_tok_t, pd * L, e->vocab, &e->ple_tok, "per_layer_token_embd"));
    e->ple_tok_t = m->ple_tok_t;
    TRY(upload_w(e, m->ple_proj, m->ple_proj_t, dim, pd * L, &e->ple_proj, "per_layer_model_proj"));
    e->ple_proj_t = m->ple_proj_t;
    TRY(upload_f(e, m->ple_proj_norm, pd, &e->ple_proj_norm, "per_layer_proj_norm"));
    TRY(upload_f(e, m->norm_out, dim, &e->norm_out, "output_norm"));

    e->layers.resize(L);
    char nm[64];
    for (int l = 0; l < L; l++) {
        LayerDev &ly = e->layers[l];
        memset(&ly, 0, sizeof ly);
        ly.swa = is_swa(m, l);
        ly.hd = ly.swa ? m->head_dim_swa : m->head_dim_full;
        ly.n_rot = ly.swa ? m->n_rot_swa : m->n_rot_full;
        if (ly.hd != 64 && ly.hd != 128 && ly.hd != 256 && ly.hd != 512) {
            set_error(G4_ERR_ARG, "engine: layer %d head_dim %d unsupported", l, ly.hd);
            return G4_ERR_ARG;
        }
        if (ly.n_rot < 0 || ly.n_rot > ly.hd || ly.n_rot % 2) { set_error(G4_ERR_ARG, "engine: layer %d n_rot %d", l, ly.n_rot); return G4_ERR_ARG; }
        ly.qd = e->nh * ly.hd;
        ly.kvd = e->nkv * ly.hd;
        e->qd_max = ly.qd > e->qd_max ? ly.qd : e->qd_max;
        e->kvd_max = ly.kvd > e->kvd_max ? ly.kvd : e->kvd_max;
        e->hd_max = ly.hd > e->hd_max ? ly.hd : e->hd_max;
#define W(field, n_in, rows)                                                                     \
    do {                                                                                         \
        snprintf(nm, sizeof nm, "blk.%d." #field, l);                                            \
        ly.field##_t = m->field##_t[l];                                                          \
        TRY(upload_w(e, m->field[l], ly.field##_t, n_in, rows, &ly.field, nm));                  \
    } while (0)
#define V(field, n, opt)                                                                         \
    do {                                                                                         \
        snprintf(nm, sizeof nm, "blk.%d." #field, l);                                            \
        TRY(upload_f(e, m->field ? m->field[l] : nullptr, n, &ly.field, nm, opt));               \
    } while (0)
        W(wq, dim, ly.qd);
        if (l < G4_N_LAYER_KV) { W(wk, dim, ly.kvd); W(wv, dim, ly.kvd); }
        W(wo, ly.qd, dim);
        W(gate, dim, e->hidden);
        W(up, dim, e->hidden);
        W(down, e->hidden, dim);
        W(inp_gate, dim, pd);
        W(proj, pd, dim);
        V(attn_norm, dim, false); V(post_attn_norm, dim, false); V(ffn_norm, dim, false); V(post_ffw_norm, dim, false);
        V(q_norm, ly.hd, false); V(k_norm, ly.hd, false); V(post_norm, dim, false); V(out_scale, 1, true);
#undef W
#undef V
        if (is_q8_type(ly.wo_t) && ly.qd % G4_QK) { set_error(G4_ERR_ARG, "engine: q_dim %d not a multiple of 256", ly.qd); return G4_ERR_ARG; }
        if (is_q8_type(ly.proj_t) && pd % G4_QK) { set_error(G4_ERR_ARG, "engine: ple_dim %d with a K-quant proj", pd); return G4_ERR_ARG; }
    }
    // KV caches and shared-KV sources (main.c:739-746, 1402-1404)
    for (int l = 0; l < L; l++) {
        LayerDev &ly = e->layers[l];
        if (l < G4_N_LAYER_KV) {
            ly.src = l;
            // a sliding-window ring holds the window plus one prefill call's rows, so the rows a call
            // stores never overwrite window rows that its earlier rows still read
            ly.ring = (ly.swa && e->window > 0 && e->window + prefill_rows < max_seq) ? e->window + prefill_rows : max_seq;
            const size_t n = (size_t)max_batch * e->nkv * ly.ring * ly.hd;
            TRY(dalloc_t(e, &ly.kc, n));
            TRY(dalloc_t(e, &ly.vc, n));
        } else {
            ly.src = ly.swa ? 22 : 23;
            const LayerDev &s = e->layers[ly.src];
            if (s.hd != ly.hd || (!ly.swa && s.ring < max_seq)) {
                set_error(G4_ERR_ARG, "engine: layer %d cannot read the KV of layer %d", l, ly.src);
                return G4_ERR_ARG;
            }
        }
    }
    // RoPE tables (host libm, reference-exact angles)
    {
        std::vector<float2> t;
        const int hs = m->n_rot_swa / 2 > 0 ? m->n_rot_swa / 2 : 1, hf = m->n_rot_full / 2 > 0 ? m->n_rot_full / 2 : 1;
        t.resize((size_t)max_seq * hs);
        rope_table_host(t.data(), max_seq, m->n_rot_swa, m->rope_theta_swa, 1.0f, nullptr);
        TRY(dalloc_t(e, &e->rope_swa, t.size()));
        G4_CUDA(cudaMemcpyAsync(e->rope_swa, t.data(), t.size() * sizeof(float2), cudaMemcpyHostToDevice, e->st));
        G4_CUDA(cudaStreamSynchronize(e->st));
        t.assign((size_t)max_seq * hf, make_float2(0, 0));
        rope_table_host(t.data(), max_seq, m->n_rot_full, m->rope_theta, 1.0f, m->rope_freqs);
        TRY(dalloc_t(e, &e->rope_full, t.size()));
        G4_CUDA(cudaMemcpyAsync(e->rope_full, t.data(), t.size() * sizeof(float2), cudaMemcpyHostToDevice, e->st));
        G4_CUDA(cudaStreamSynchronize(e->st));
    }
    // activations: decode rows (max_batch sequences) or prefill rows, whichever is more
    const size_t B = std::max(max_batch, prefill_rows), BS = max_batch;
    TRY(dalloc_t(e, &e->x, B * dim)); TRY(dalloc_t(e, &e->x2, B * dim)); TRY(dalloc_t(e, &e->xn, B * dim)); TRY(dalloc_t(e, &e->xf, B * dim));
    TRY(dalloc_t(e, &e->q, B * e->qd_max)); TRY(dalloc_t(e, &e->qn, B * e->qd_max)); TRY(dalloc_t(e, &e->qo, B * e->qd_max));
    TRY(dalloc_t(e, &e->k, B * e->kvd_max)); TRY(dalloc_t(e, &e->v, B * e->kvd_max));
    TRY(dalloc_t(e, &e->o_raw, B * dim)); TRY(dalloc_t(e, &e->d_raw, B * dim)); TRY(dalloc_t(e, &e->p_raw, B * dim));
    TRY(dalloc_t(e, &e->hb, B * e->hidden)); TRY(dalloc_t(e, &e->hb2, B * e->hidden));
    TRY(dalloc_t(e, &e->g, B * pd));
    TRY(dalloc_t(e, &e->ple_tokb, B * pd * L)); TRY(dalloc_t(e, &e->ple_ctx, B * pd * L)); TRY(dalloc_t(e, &e->ple, B * pd * L));
    TRY(dalloc_t(e, &e->logits, BS * e->vocab));
    int nmax = dim > e->qd_max ? dim : e->qd_max;
    nmax = nmax > e->hidden ? nmax : e->hidden;
    nmax = nmax > pd ? nmax : pd;
    e->q8_blocks = (nmax + G4_QK - 1) / G4_QK;
    TRY(dalloc_t(e, &e->q8, B * e->q8_blocks * G4_Q8_BYTES));
    e->max_chunks = (max_seq + attn_chunk_size() - 1) / attn_chunk_size();
    TRY(dalloc_t(e, &e->attn_part, B * e->nh * e->max_chunks * (size_t)(e->hd_max + 2)));
    TRY(dalloc_t(e, &e->keys, B));
    G4_CUDA(cudaDeviceGetAttribute(&e->nsm, cudaDevAttrMultiProcessorCount, e->device));
    if (B > 1) {  // tensor-core path of the batched step (and of prefill rows)
        int nmax = std::max(std::max(dim, e->hidden), std::max(e->qd_max, pd));
        size_t part = 0;
        const int shapes[][2] = {{e->qd_max, dim}, {e->kvd_max, dim}, {dim, e->qd_max}, {e->hidden, dim},
                                 {dim, e->hidden}, {pd * L, dim}, {e->vocab, dim}, {pd, dim}, {dim, pd},
                                 {e->qd_max + e->kvd_max, dim}, {2 * e->hidden, dim}};  // + Q4_K pair launches
        for (auto &sh : shapes) {
            part = std::max(part, tc_part_bytes(sh[0], sh[1], e->nsm));
            // BF16 K-split: up to nsm / tiles slices of the whole row set
            const int tiles = (sh[0] + 127) / 128;
            part = std::max(part, (size_t)std::max(1, std::min(sh[1] / 64, e->nsm / tiles)) * 64 * sh[0] * sizeof(float));
        }
        nmax = (nmax + G4_QK - 1) / G4_QK * G4_QK;
        TRY(dalloc_t(e, &e->tcq, tc_operand_bytes(nmax)));
        TRY(dalloc_t(e, &e->tc6, tc6_operand_bytes(nmax)));
        TRY(dalloc_t(e, &e->tcb, bf16tc_operand_bytes((nmax + 63) / 64 * 64)));
        e->tc_part_bytes = std::max(part, (size_t)16);
        TRY(dalloc_t(e, &e->tc_part, e->tc_part_bytes / sizeof(float)));
        TRY(dalloc_t(e, &e->tc_tickets, (size_t)e->vocab / 128 + 4096));  // zeroed; every launch leaves them zero
        e->tc_part2_bytes = std::max(tc_part_bytes(e->kvd_max, dim, e->nsm), (size_t)16);
        TRY(dalloc_t(e, &e->tc_part2, e->tc_part2_bytes / sizeof(float)));
        TRY(dalloc_t(e, &e->tc_tickets2, 4096));
        G4_CUDA(cudaStreamCreateWithFlags(&e->st2, cudaStreamNonBlocking));
        G4_CUDA(cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming));
        G4_CUDA(cudaEventCreateWithFlags(&e->ev_join, cudaEventDisableTiming));
    }
    TRY(dalloc_t(e, &e->attn_ctr, B * e->nkv));
    TRY(dalloc_t(e, &e->d_err, 1));
    G4_CUDA(cudaMallocHost((void **)&e->h_err, sizeof(int)));
    *e->h_err = 0;
    TRY(dalloc_t(e, &e->d_tokens, B)); TRY(dalloc_t(e, &e->d_next, B)); TRY(dalloc_t(e, &e->d_pos, 1));
    TRY(dalloc_t(e, &e->d_hist, (size_t)max_seq * BS));
    TRY(dalloc_t(e, &e->d_rowpos, B)); TRY(dalloc_t(e, &e->d_rowseq, B));
    G4_CUDA(cudaMallocHost((void **)&e->h_rows, sizeof(int) * 3 * B));
    TRY(dalloc_t(e, &e->cand_v, BS * 64)); TRY(dalloc_t(e, &e->cand_i, BS * 64));
    TRY(dalloc_t(e, &e->d_recent, BS * (size_t)max_seq)); TRY(dalloc_t(e, &e->d_nrec, BS));
    G4_CUDA(cudaMallocHost((void **)&e->h_cand_v, sizeof(float) * BS * 64));
    G4_CUDA(cudaMallocHost((void **)&e->h_cand_i, sizeof(int) * BS * 64));
    G4_CUDA(cudaMallocHost((void **)&e->h_pos, sizeof(int) * (size_t)max_seq));
    for (int i = 0; i < max_seq; i++) e->h_pos[i] = i;
    G4_CUDA(cudaMallocHost((void **)&e->h_tok, sizeof(int) * (size_t)max_seq * BS));
    G4_CUDA(cudaStreamSynchronize(e->st));
    return G4_OK;
}

}  // namespace

extern "C" {

g4_engine *g4_engine_create(const g4_model_desc *m, int device, int max_seq, int max_batch) {
    return g4_engine_create_ex(m, device, max_seq, max_batch, 0);
}

g4_engine *g4_engine_create_ex(const g4_model_desc *m, int device, int max_seq, int max_batch, int prefill_rows) {
    g4_engine *e = new g4_engine();
    e->device = device;
    if (create(e, m, max_seq, max_batch, prefill_rows) != G4_OK) {
        const int code = g4_last_error();
        char msg[512];
        snprintf(msg, sizeof msg, "%s", g4_last_error_string());
        destroy(e);
        set_error(code ? code : G4_ERR_CUDA, "%s", msg);
        return nullptr;
    }
    return e;
}

int g4_engine_destroy(g4_engine *e) {
    destroy(e);
    return G4_OK;
}

size_t g4_engine_device_bytes(const g4_engine *e) { return e ? e->dev_bytes : 0; }

size_t g4_model_desc_bytes(void) { return sizeof(g4_model_desc); }

int g4_engine_last_step_kernels(const g4_engine *e) { return e ? e->last_step_kernels : -1; }

int g4_engine_set_tc_min_batch(g4_engine *e, int min_batch) {
    if (!e || min_batch < 1) { set_error(G4_ERR_ARG, "set_tc_min_batch: bad arguments"); return -1; }
    std::lock_guard<std::mutex> lk(e->mu);
    const int prev = e->tc_min_batch;
    if (min_batch != prev) {  // captured steps were built for the old threshold
        cudaSetDevice(e->device);
        cudaStreamSynchronize(e->st);
        for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);
        e->graphs.clear();
        e->graph_kernels.clear();
        e->graph_hidden.clear();
    }
    e->tc_min_batch = min_batch;
    return prev;
}

int g4_engine_set_attn_split(g4_engine *e, int sliding, int global) {
    if (!e || sliding < 0 || global < 0 || sliding % 32 || global % 32) {
        set_error(G4_ERR_ARG, "set_attn_split: rows must be multiples of 32 (0: default)");
        return G4_ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(e->mu);
    if (sliding != e->attn_split_swa || global != e->attn_split_full) {  // captured steps used the old split
        G4_CUDA(cudaSetDevice(e->device));
        G4_CUDA(cudaStreamSynchronize(e->st));
        for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);
        e->graphs.clear();
        e->graph_kernels.clear();
        e->graph_hidden.clear();
    }
    e->attn_split_swa = sliding;
    e->attn_split_full = global;
    return G4_OK;
}

void *g4_engine_stream(g4_engine *e) { return e ? (void *)e->st : nullptr; }

int g4_engine_sync(g4_engine *e) {
    if (!e) { set_error(G4_ERR_ARG, "engine is NULL"); return G4_ERR_ARG; }
    G4_CUDA(cudaSetDevice(e->device));
    TRY(enqueue_err_check(e));
    G4_CUDA(cudaStreamSynchronize(e->st));
    return err_after_sync(e);
}

int g4_forward(g4_engine *e, int token, int pos, int lm_mode, float *logits) {
    if (!e || lm_mode < 0 || lm_mode > 2) { set_error(G4_ERR_ARG, "forward: bad arguments"); return -1; }
    std::lock_guard<std::mutex> lk(e->mu);
    if (cudaSetDevice(e->device) != cudaSuccess) { set_error(G4_ERR_CUDA, "cudaSetDevice failed"); return -1; }
    if (set_pos(e, pos) || stage_tokens(e, &token, 1, pos)) return -1;
    if (run_step(e, 1, lm_mode, false, lm_mode != 0 && logits != nullptr)) return -1;
    int next = 0;
    if (lm_mode) {
        if (cudaMemcpyAsync(&next, e->d_next, 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess) { set_error(G4_ERR_CUDA, "readback failed"); return -1; }
        if (logits && cudaMemcpyAsync(logits, e->logits, sizeof(float) * e->vocab, cudaMemcpyDeviceToHost, e->st) != cudaSuccess) {
            set_error(G4_ERR_CUDA, "logits readback failed");
            return -1;
        }
    }
    if (enqueue_err_check(e)) return -1;
    cudaError_t ce = cudaStreamSynchronize(e->st);
    if (ce != cudaSuccess) { cuda_fail(ce, "forward", __FILE__, __LINE__); return -1; }
    if (err_after_sync(e)) return -1;
    return next;
}

int g4_generate_greedy(g4_engine *e, const int *prompt, int n_prompt, int max_new, int eos, int *out_tokens) {
    if (!e || !prompt || n_prompt <= 0 || max_new < 0 || (max_new > 0 && !out_tokens)) {
        set_error(G4_ERR_ARG, "generate: bad arguments");
        return -1;
    }
    std::lock_guard<std::mutex> lk(e->mu);
    if (cudaSetDevice(e->device) != cudaSuccess) { set_error(G4_ERR_CUDA, "cudaSetDevice failed"); return -1; }
    int total = n_prompt + max_new - 1;  // generate's position loop (main.c:2366-2370)
    if (total > e->max_seq) total = e->max_seq;
    int ngen = 0;
    for (int pos = 0; pos < total; pos++) {
        const int lm = pos < n_prompt - 1 ? 0 : 1;
        if (set_pos(e, pos)) return -1;
        const bool from_keys = pos >= n_prompt;
        if (!from_keys && stage_tokens(e, prompt + pos, 1, pos)) return -1;
        if (run_step(e, 1, lm, from_keys, false)) return -1;
        if (lm) {
            if (cudaMemcpyAsync(e->d_hist + ngen, e->d_next, 4, cudaMemcpyDeviceToDevice, e->st) != cudaSuccess) {
                set_error(G4_ERR_CUDA, "history copy failed");
                return -1;
            }
            ngen++;
        }
    }
    if (ngen && cudaMemcpyAsync(out_tokens, e->d_hist, sizeof(int) * ngen, cudaMemcpyDeviceToHost, e->st) != cudaSuccess) {
        set_error(G4_ERR_CUDA, "history readback failed");
        return -1;
    }
    if (enqueue_err_check(e)) return -1;
    cudaError_t ce = cudaStreamSynchronize(e->st);
    if (ce != cudaSuccess) { cuda_fail(ce, "generate", __FILE__, __LINE__); return -1; }
    if (err_after_sync(e)) return -1;
    for (int i = 0; i < ngen; i++)
        if (out_tokens[i] == eos) return i;  // the reference stops before emitting eos (main.c:2435)
    return ngen;
}

int g4_decode_batch(g4_engine *e, int B, const int *tokens, int pos, int lm_mode, int *next) {
    if (!e || !tokens || B <= 0 || lm_mode < 0 || lm_mode > 2 || (lm_mode && !next)) { set_error(G4_ERR_ARG, "decode_batch: bad arguments"); return G4_ERR_ARG; }
    std::lock_guard<std::mutex> lk(e->mu);
    if (B > e->max_batch) { set_error(G4_ERR_STATE, "batch %d > engine max_batch %d", B, e->max_batch); return G4_ERR_STATE; }
    G4_CUDA(cudaSetDevice(e->device));
    TRY(set_pos(e, pos));
    TRY(stage_tokens(e, tokens, B, pos));
    TRY(run_step(e, B, lm_mode, false, false));
    if (lm_mode) G4_CUDA(cudaMemcpyAsync(next, e->d_next, sizeof(int) * B, cudaMemcpyDeviceToHost, e->st));
    TRY(enqueue_err_check(e));
    G4_CUDA(cudaStreamSynchronize(e->st));
    return err_after_sync(e);
}

int g4_decode_batch_device(g4_engine *e, int B, const int *tokens_dev, int pos, int lm_mode, int *next_dev) {
    if (!e || B <= 0 || lm_mode < 0 || lm_mode > 2) { set_error(G4_ERR_ARG, "decode_batch_device: bad arguments"); return G4_ERR_ARG; }
    std::lock_guard<std::mutex> lk(e->mu);
    if (B > e->max_batch) { set_error(G4_ERR_STATE, "batch %d > engine max_batch %d", B, e->max_batch); return G4_ERR_STATE; }
    G4_CUDA(cudaSetDevice(e->device));
    TRY(set_pos(e, pos));
    if (tokens_dev) G4_CUDA(cudaMemcpyAsync(e->d_tokens, tokens_dev, sizeof(int) * B, cudaMemcpyDeviceToDevice, e->st));
    TRY(run_step(e, B, lm_mode, tokens_dev == nullptr, false));
    if (lm_mode && next_dev) G4_CUDA(cudaMemcpyAsync(next_dev, e->d_next, sizeof(int) * B, cudaMemcpyDeviceToDevice, e->st));
    return G4_OK;
}

int g4_engine_fill_kv(g4_engine *e, int npos, uint64_t seed) {
    if (!e || npos < 0 || npos > e->max_seq) { set_error(G4_ERR_ARG, "fill_kv: bad arguments"); return G4_ERR_ARG; }
    std::lock_guard<std::mutex> lk(e->mu);
    G4_CUDA(cudaSetDevice(e->device));
    for (int l = 0; l < e->L && l < G4_N_LAYER_KV; l++) {
        const LayerDev &ly = e->layers[l];
        TRY(launch_fill_kv(ly.kc, e->max_batch, e->nkv, ly.ring, ly.hd, npos, seed + 2 * (uint64_t)l, e->st));
        TRY(launch_fill_kv(ly.vc, e->max_batch, e->nkv, ly.ring, ly.hd, npos, seed + 2 * (uint64_t)l + 1, e->st));
    }
    G4_CUDA(cudaStreamSynchronize(e->st));
    return G4_OK;
}

int g4_engine_time_attention(g4_engine *e, const int *layers, int n, int batch, int reps, float *ms) {
    if (!e || !layers || n <= 0 || batch <= 0 || batch > e->max_batch || reps <= 0 || !ms) {
        set_error(G4_ERR_ARG, "time_attention: bad arguments");
        return G4_ERR_ARG;
    }
    for (int i = 0; i < n; i++)
        if (layers[i] < 0 || layers[i] >= e->L) { set_error(G4_ERR_ARG, "time_attention: layer %d", layers[i]); return G4_ERR_ARG; }
    std::lock_guard<std::mutex> lk(e->mu);
    G4_CUDA(cudaSetDevice(e->device));
    cudaEvent_t t0 = nullptr, t1 = nullptr;
    cudaError_t ce = cudaEventCreate(&t0);
    if (ce == cudaSuccess) ce = cudaEventCreate(&t1);
    if (ce == cudaSuccess) ce = cudaEventRecord(t0, e->st);
    int rc = ce == cudaSuccess ? G4_OK : G4_ERR_CUDA;
    for (int r = 0; r < reps && rc == G4_OK; r++)  // launch_attention records its own error text
        for (int i = 0; i < n && rc == G4_OK; i++) rc = launch_attention(attn_args(e, layers[i]), batch, e->d_pos, e->max_seq, e->st);
    if (rc == G4_OK) {
        ce = cudaEventRecord(t1, e->st);
        if (ce == cudaSuccess) ce = cudaEventSynchronize(t1);
        if (ce == cudaSuccess) ce = cudaEventElapsedTime(ms, t0, t1);
        if (ce != cudaSuccess) rc = G4_ERR_CUDA;
    }
    if (ce != cudaSuccess) set_error(G4_ERR_CUDA, "time_attention: %s", cudaGetErrorString(ce));
    if (t0) cudaEventDestroy(t0);
    if (t1) cudaEventDestroy(t1);
    if (rc) return rc;
    G4_CUDA(cudaStreamSynchronize(e->st));
    return err_after_sync(e);
}

int g4_engine_get_hidden(g4_engine *e, int b, float *x) {
    if (!e || !x || b < 0 || b >= e->max_batch) { set_error(G4_ERR_ARG, "get_hidden: bad arguments"); return G4_ERR_ARG; }
    std::lock_guard<std::mutex> lk(e->mu);
    G4_CUDA(cudaSetDevice(e->device));
    // after an LM-head step the reference's State.x holds the output-normed vector (main.c:2021)
    const float *src = (e->hidden_src ? e->hidden_src : e->x) + (size_t)b * e->dim;
    G4_CUDA(cudaMemcpyAsync(x, src, sizeof(float) * e->dim, cudaMemcpyDeviceToHost, e->st));
    G4_CUDA(cudaStreamSynchronize(e->st));
    return G4_OK;
}

int g4_engine_set_kv(g4_engine *e, int b, int layer, int pos0, int npos, const float *k, const float *v) {
    if (!e || !k || !v || b < 0 || b >= e->max_batch || layer < 0 || layer >= e->L || layer >= G4_N_LAYER_KV ||
        pos0 < 0 || npos < 0 || pos0 + npos > e->max_seq) {
        set_error(G4_ERR_ARG, "set_kv: bad arguments");
        return G4_ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(e->mu);
    G4_CUDA(cudaSetDevice(e->device));
    const LayerDev &ly = e->layers[layer];
    const size_t rowf = (size_t)e->nkv * ly.hd;  // host row: n_kv heads of hd floats
    // positions map to ring slots pos % ring; copy runs of consecutive slots per head
    for (int p = pos0; p < pos0 + npos;) {
        const int slot = p % ly.ring, run = std::min(pos0 + npos - p, ly.ring - slot);
        for (int h = 0; h < e->nkv; h++) {
            const size_t drow = (((size_t)b * e->nkv + h) * ly.ring + slot) * ly.hd;
            const size_t srow = (size_t)(p - pos0) * rowf + (size_t)h * ly.hd;
            G4_CUDA(cudaMemcpy2DAsync(ly.kc + drow, ly.hd * sizeof(float), k + srow, rowf * sizeof(float),
                                      ly.hd * sizeof(float), run, cudaMemcpyHostToDevice, e->st));
            G4_CUDA(cudaMemcpy2DAsync(ly.vc + drow, ly.hd * sizeof(float), v + srow, rowf * sizeof(float),
                                      ly.hd * sizeof(float), run, cudaMemcpyHostToDevice, e->st));
        }
        p += run;
    }
    G4_CUDA(cudaStreamSynchronize(e->st));
    return G4_OK;
}

int g4_engine_get_kv(g4_engine *e, int b, int layer, int pos, float *k, float *v) {
    if (!e || b < 0 || b >= e->max_batch || layer < 0 || layer >= e->L || layer >= G4_N_LAYER_KV || pos < 0 ||
        pos >= e->max_seq) {
        set_error(G4_ERR_ARG, "get_kv: bad arguments");
        return G4_ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(e->mu);
    G4_CUDA(cudaSetDevice(e->device));
    const LayerDev &ly = e->layers[layer];
    const int slot = pos % ly.ring;
    for (int h = 0; h < e->nkv; h++) {
        const size_t row = (((size_t)b * e->nkv + h) * ly.ring + slot) * ly.hd;
        if (k) G4_CUDA(cudaMemcpyAsync(k + (size_t)h * ly.hd, ly.kc + row, sizeof(float) * ly.hd, cudaMemcpyDeviceToHost, e->st));
        if (v) G4_CUDA(cudaMemcpyAsync(v + (size_t)h * ly.hd, ly.vc + row, sizeof(float) * ly.hd, cudaMemcpyDeviceToHost, e->st));
    }
    G4_CUDA(cudaStreamSynchronize(e->st));
    return G4_OK;
}

int g4_generate(g4_engine *e, const int *prompt, int n_prompt, int max_new, float temp, float topp, int topk,
                float repeat_penalty, int penalty_last_n, uint64_t seed, int eos, int *out_tokens) {
    if (!e || !prompt || n_prompt <= 0 || max_new < 0 || (max_new > 0 && !out_tokens)) {
        set_error(G4_ERR_ARG, "generate: bad arguments");
        return -1;
    }
    const bool plain_greedy = temp <= 0.0f && repeat_penalty <= 1.0f;
    if (plain_greedy) return g4_generate_greedy(e, prompt, n_prompt, max_new, eos, out_tokens);
    std::lock_guard<std::mutex> lk(e->mu);
    if (cudaSetDevice(e->device) != cudaSuccess) { set_error(G4_ERR_CUDA, "cudaSetDevice failed"); return -1; }
    uint64_t rng = seed ? seed : 1;  // main.c:2341
    int total = n_prompt + max_new - 1, token = prompt[0], gen = 0;
    if (total > e->max_seq) total = e->max_seq;
    for (int pos = 0; pos < total; pos++) {
        const bool prefill = pos < n_prompt - 1;
        if (set_pos(e, pos) || stage_tokens(e, &token, 1, pos)) return -1;
        if (run_step(e, 1, prefill ? 0 : 1, false, !prefill)) return -1;
        int next;
        if (prefill) {
            next = prompt[pos + 1];
        } else {
            // the penalty covers the generated tokens only, the last penalty_last_n of them (main.c:2117-2119)
            const int start = (penalty_last_n > 0 && gen > penalty_last_n) ? gen - penalty_last_n : 0;
            const int nrec = gen - start;
            if (sample_after_step(e, 1, temp, topp, topk, repeat_penalty, out_tokens + start, nrec > 0 ? nrec : 1, &nrec,
                                  &rng, &next))
                return -1;
            if (next == eos) break;
            out_tokens[gen++] = next;
        }
        token = next;
    }
    if (!total || total <= n_prompt - 1) {  // prefill only: wait for it
        if (enqueue_err_check(e) || cudaStreamSynchronize(e->st) != cudaSuccess || err_after_sync(e)) return -1;
    }
    return gen;
}

int g4_decode_batch_sample(g4_engine *e, int B, const int *tokens, int pos, float temp, float topp, int topk,
                           float repeat_penalty, const int *recent, int recent_ld, const int *n_recent, uint64_t *rng,
                           int *next) {
    if (!e || !tokens || B <= 0 || !rng || !next || (repeat_penalty > 1.0f && (!recent || !n_recent || recent_ld <= 0))) {
        set_error(G4_ERR_ARG, "decode_batch_sample: bad arguments");
        return G4_ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(e->mu);
    if (B > e->max_batch) { set_error(G4_ERR_STATE, "batch %d > engine max_batch %d", B, e->max_batch); return G4_ERR_STATE; }
    G4_CUDA(cudaSetDevice(e->device));
    TRY(set_pos(e, pos));
    TRY(stage_tokens(e, tokens, B, pos));
    TRY(run_step(e, B, 1, false, true));
    return sample_after_step(e, B, temp, topp, topk, repeat_penalty, recent, recent_ld, n_recent, rng, next);
}

int g4_prefill(g4_engine *e, int n_rows, const int *seq, const int *pos, const int *tokens) {
    if (!e || n_rows <= 0 || !seq || !pos || !tokens) { set_error(G4_ERR_ARG, "prefill: bad arguments"); return G4_ERR_ARG; }
    std::lock_guard<std::mutex> lk(e->mu);
    if (n_rows > e->prefill_cap) {
        set_error(G4_ERR_STATE, "prefill: %d rows > the engine's %d prefill rows (g4_engine_create_ex)", n_rows, e->prefill_cap);
        return G4_ERR_STATE;
    }
    for (int i = 0; i < n_rows; i++) {
        if (seq[i] < 0 || seq[i] >= e->max_batch || pos[i] < 0 || pos[i] >= e->max_seq || tokens[i] < 0 || tokens[i] >= e->vocab) {
            set_error(G4_ERR_ARG, "prefill: row %d (sequence %d, position %d, token %d) out of range", i, seq[i], pos[i], tokens[i]);
            return G4_ERR_ARG;
        }
        for (int j = 0; j < i; j++)  // one row per (sequence, position); a call spans < prefill_cap positions
            if (seq[j] == seq[i] && (pos[j] == pos[i] || abs(pos[j] - pos[i]) >= e->prefill_cap)) {
                set_error(G4_ERR_ARG, "prefill: rows %d and %d of sequence %d at positions %d and %d", j, i, seq[i], pos[j], pos[i]);
                return G4_ERR_ARG;
            }
    }
    G4_CUDA(cudaSetDevice(e->device));
    G4_CUDA(cudaStreamSynchronize(e->st));  // the pinned staging rows are reused
    int *h = e->h_rows;
    memcpy(h, seq, sizeof(int) * n_rows);
    memcpy(h + n_rows, pos, sizeof(int) * n_rows);
    memcpy(h + 2 * n_rows, tokens, sizeof(int) * n_rows);
    G4_CUDA(cudaMemcpyAsync(e->d_rowseq, h, sizeof(int) * n_rows, cudaMemcpyHostToDevice, e->st));
    G4_CUDA(cudaMemcpyAsync(e->d_rowpos, h + n_rows, sizeof(int) * n_rows, cudaMemcpyHostToDevice, e->st));
    G4_CUDA(cudaMemcpyAsync(e->d_tokens, h + 2 * n_rows, sizeof(int) * n_rows, cudaMemcpyHostToDevice, e->st));
    TRY(enqueue_step_unfused(e, n_rows, 0, false, false, true));
    e->hidden_src = e->x;
    TRY(enqueue_err_check(e));
    G4_CUDA(cudaStreamSynchronize(e->st));
    return err_after_sync(e);
}

int g4_nccl_unique_id(void *id) {
    if (!id) { set_error(G4_ERR_ARG, "nccl_unique_id: null"); return G4_ERR_ARG; }
    TRY(nccl_load());
    ncclUniqueId u;
    G4_NCCL(g_nccl.get_unique_id(&u));
    memcpy(id, &u, sizeof u);
    return G4_OK;
}

int g4_lm_split_rows(int vocab, int world, int rank, int *row0, int *row1) {
    if (vocab <= 0 || world <= 0 || rank < 0 || rank >= world || !row0 || !row1) {
        set_error(G4_ERR_ARG, "lm_split_rows: bad arguments");
        return G4_ERR_ARG;
    }
    const int chunk = ((vocab + world - 1) / world + 127) / 128 * 128;  // whole 128-row tiles per rank
    *row0 = std::min(vocab, rank * chunk);
    *row1 = std::min(vocab, *row0 + chunk);
    return chunk;
}

int g4_lm_split_merge(const uint64_t *keys_all, int world, int rank, int B, int chunk, uint64_t *out) {
    if (!keys_all || !out || world <= 0 || rank < 0 || rank >= world || B <= 0 || chunk <= 0) {
        set_error(G4_ERR_ARG, "lm_split_merge: bad arguments");
        return G4_ERR_ARG;
    }
    for (int b = 0; b < B; b++)
        out[b] = lm_split_merge_one((const unsigned long long *)keys_all, world, rank, B, chunk, b);
    return G4_OK;
}

int g4_argmax_keys(const float *logits, int n, int row0, uint64_t *key) {
    if (!logits || n <= 0 || !key) { set_error(G4_ERR_ARG, "argmax_keys: bad arguments"); return G4_ERR_ARG; }
    unsigned long long best = 0ull;
    for (int i = 0; i < n; i++) {  // the device's packed key (argmax_key) computed on the host
        uint32_t b;
        memcpy(&b, logits + i, 4);
        if ((b & 0x7fffffffu) == 0u) b = 0u;
        b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
        const unsigned long long k = ((unsigned long long)b << 32) | (uint32_t)(0xffffffffu - (uint32_t)(i + row0));
        best = k > best ? k : best;
    }
    *key = best;
    return G4_OK;
}

int g4_engine_lm_split(g4_engine *e, const void *nccl_id, int rank, int world) {
    if (!e || !nccl_id || world < 2 || rank < 0 || rank >= world) {
        set_error(G4_ERR_ARG, "lm_split: bad arguments");
        return G4_ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(e->mu);
    if (e->comm) { set_error(G4_ERR_STATE, "lm_split: already split"); return G4_ERR_STATE; }
    TRY(nccl_load());
    G4_CUDA(cudaSetDevice(e->device));
    G4_CUDA(cudaStreamSynchronize(e->st));
    int r0 = 0, r1 = 0;
    const int chunk = g4_lm_split_rows(e->vocab, world, rank, &r0, &r1);
    if (chunk < 0) return G4_ERR_ARG;
    TRY(dalloc_t(e, &e->xf_all, (size_t)world * e->max_batch * e->dim));
    TRY(dalloc_t(e, &e->keys_loc, (size_t)world * e->max_batch));
    TRY(dalloc_t(e, &e->keys_all, (size_t)world * world * e->max_batch));
    ncclUniqueId u;
    memcpy(&u, nccl_id, sizeof u);
    G4_NCCL(g_nccl.comm_init_rank(&e->comm, world, u, rank));
    e->split_rank = rank; e->split_world = world; e->lm_r0 = r0; e->lm_r1 = r1; e->lm_chunk = chunk;
    for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);  // captured without the split
    e->graphs.clear(); e->graph_kernels.clear(); e->graph_hidden.clear();
    return G4_OK;
}

}  // extern "C"
