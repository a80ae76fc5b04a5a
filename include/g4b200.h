/*
 * g4b200.h — C ABI of the B200 (sm_100a) decode engine for the Gemma 4 E4B
 * Q4_K_M hot path of thamada/Gemma4.c.
 *
 * Every entry point is plain C: pointers, sizes and ints, no CUDA or torch types.
 * Two families:
 *
 *  1. Per-call drop-ins for the static functions of
 *     gemma4-4b/cpu-blas/main.c (the reference engine, one translation unit).
 *     They take HOST buffers, run the work on the GPU and copy the result back
 *     before returning, so a C host can swap `mm(...)` for `g4_mm(...)` with
 *     no other change.  Weight pointers are treated like the reference treats
 *     them: read-only views of the GGUF mmap.  The first call that sees a
 *     weight pointer uploads the tensor and later calls reuse the device copy
 *     (keyed by host pointer and byte size).  `g4_registry_clear()` drops the
 *     cache when a host buffer is reused for other contents.
 *     The reference signatures return void and `exit(1)` on bad input; the
 *     drop-ins keep the void signature, record the error instead
 *     (`g4_last_error()`), and never abort.  Each has an `_ex` twin that
 *     returns the status.
 *
 *  2. The device-resident decode engine (`g4_engine_*`, `g4_forward`,
 *     `g4_generate_greedy`, `g4_decode_batch_*`): the whole of `forward`
 *     (main.c:1838-2029) on the GPU with weights, KV cache and activations
 *     resident in HBM.  Only token ids in and logits / argmax out cross PCIe.
 *
 * Threading: one engine per GPU, not re-entrant per engine (the reference's
 * `generate` loop is single-threaded, main.c:2335-2488).  Per-call functions
 * use one internal stream per device and are serialised by a mutex.
 */
#ifndef G4B200_H
#define G4B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G4_QK_K 256

/* ggml tensor type ids, as enumerated in main.c:84-91 (enum ggml_dtype). */
enum g4_dtype {
    G4_F32 = 0,
    G4_F16 = 1,
    G4_Q4_K = 12,
    G4_Q5_K = 13,
    G4_Q6_K = 14,
    G4_BF16 = 30
};

/* Q8_K activation block; byte layout of BlockQ8_K (main.c:118-122), 292 bytes. */
typedef struct {
    float d;
    int8_t qs[G4_QK_K];
    int16_t bsums[G4_QK_K / 16];
} g4_block_q8_K;

/* Status codes.  The reference reports these cases with fprintf+exit(1)
 * (main.c:609-610, 1663-1664, 1676-1678, 1690-1692). */
enum g4_status {
    G4_OK = 0,
    G4_ERR_ARG = 1,        /* bad size / NULL pointer / n % 256 != 0 */
    G4_ERR_TYPE = 2,       /* tensor type not supported by this function */
    G4_ERR_CUDA = 3,       /* a CUDA runtime call failed */
    G4_ERR_OOM = 4,        /* device allocation failed */
    G4_ERR_NO_DEVICE = 5,  /* no usable sm_100 device */
    G4_ERR_STATE = 6,      /* engine misuse (pos beyond max_seq, batch too big...) */
    G4_ERR_TIMEOUT = 7     /* a bounded device-side wait gave up */
};

/* Last error of the calling thread (0 = none) and its message. */
int g4_last_error(void);
const char *g4_last_error_string(void);
void g4_clear_error(void);

/* Select the device used by the per-call API (default: the current device). */
int g4_set_device(int device);
/* Drop every cached device copy of host weight tensors (per-call API). */
int g4_registry_clear(void);
/* Number of cached weight tensors and their device bytes. */
int g4_registry_stats(int *n_tensors, size_t *bytes);
/* Number of kernels this library launched since load (all devices). */
uint64_t g4_kernel_launch_count(void);

/* ------------------------------------------------------------------ */
/* 1. Per-call drop-ins (host buffers in, host buffers out)           */
/* ------------------------------------------------------------------ */

/* quantize_row_q8_K (main.c:282-340; scalar twin 247-279).  k % 256 == 0. */
void g4_quantize_row_q8_K(const float *x, g4_block_q8_K *y, int k);
int g4_quantize_row_q8_K_ex(const float *x, g4_block_q8_K *y, int k);

/* vec_dot_q4_K_q8_K / vec_dot_q5_K_q8_K: one row (main.c:476-529, 531-593). */
void g4_vec_dot_q4_K_q8_K(int n, const void *x, const g4_block_q8_K *y, float *out);
void g4_vec_dot_q5_K_q8_K(int n, const void *x, const g4_block_q8_K *y, float *out);
int g4_vec_dot_q4_K_q8_K_ex(int n, const void *x, const g4_block_q8_K *y, float *out);
int g4_vec_dot_q5_K_q8_K_ex(int n, const void *x, const g4_block_q8_K *y, float *out);

/* Integer partial sums of the Q4_K/Q5_K x Q8_K dot per (row, super-block):
 * sumi_s = sum_j scale[j] * sum_32 q * q8 and sumi_m = sum_j min[j/2]*bsums[j]
 * (main.c:373-399).  Outputs are int32[d * n/256] each, row-major.  Test tap. */
int g4_quant_dot_block_sums(const void *w, int n, int d, int type, const g4_block_q8_K *q8,
                            int32_t *sumi_s, int32_t *sumi_m);

/* mm (main.c:1669-1694): o[d] = W[d x n] * x[n] for F32/F16/BF16/Q4_K/Q5_K/Q6_K.
 * Q4_K/Q5_K: when q8_ready == 0 the activation is quantized into q8 (written
 * back to the host buffer, as the reference does); when 1 the given q8 is used. */
void g4_mm(float *o, const float *x, const void *w, int n, int d, int type,
           g4_block_q8_K *q8, int q8_ready);
int g4_mm_ex(float *o, const float *x, const void *w, int n, int d, int type,
             g4_block_q8_K *q8, int q8_ready);

/* mm_quant_dot_rows (main.c:1558-1566): Q4_K/Q5_K rows against a ready Q8_K. */
void g4_mm_quant_dot_rows(float *o, const void *w, int n, int d, int type, const g4_block_q8_K *q8);
int g4_mm_quant_dot_rows_ex(float *o, const void *w, int n, int d, int type, const g4_block_q8_K *q8);

/* mm_quant_rows (main.c:1539-1556): fp32 dequant-dot of K-quant rows. */
void g4_mm_quant_rows(float *o, const float *x, const void *w, int n, int d, int type);
int g4_mm_quant_rows_ex(float *o, const float *x, const void *w, int n, int d, int type);

/* mm_argmax_row (main.c:1570-1667): index of the largest row dot, lowest
 * index on ties.  Returns the index, or -1 on error. */
int g4_mm_argmax_row(const float *x, const void *w, int n, int d, int type, g4_block_q8_K *q8);

/* apply_rope_neox (main.c:1725-1745), in place on vec[n_heads * head_dim]. */
void g4_apply_rope_neox(float *vec, int n_heads, int head_dim, int n_rot, int pos,
                        float freq_base, float freq_scale, const float *freq_factors);
int g4_apply_rope_neox_ex(float *vec, int n_heads, int head_dim, int n_rot, int pos,
                          float freq_base, float freq_scale, const float *freq_factors);

/* logits_tied (main.c:1780-1796) on an explicit hidden vector x[dim]:
 * logits[vocab] = cap * tanh(W_embd x / cap) (cap <= 0: no softcap).  When
 * argmax is not NULL it receives the first index of the largest logit
 * (sample_token with temp <= 0, main.c:2045-2050).  logits may be NULL. */
int g4_logits_tied(float *logits, int *argmax, const float *x, const void *embd, int embd_type,
                   int dim, int vocab, float softcap);

/* sample_token (main.c:2044-2112) on host logits[n]: temp <= 0 returns the
 * first index of the largest logit; otherwise the top-k candidates (value
 * descending, index ascending, as the reference's insertion sort) are
 * selected on the GPU and the temperature softmax, top-p and xorshift64*
 * draws (*rng is advanced) run on the host with the reference's float
 * expressions, so the token is the reference's.  topk <= 0 means n; k above
 * 64 is rejected.  Returns the token id, or -1 on error. */
int g4_sample_token(const float *logits, int n, float temp, float topp, int topk, uint64_t *rng);

/* Decode attention for one query position over a caller-provided fp32 KV
 * window, laid out like the reference cache rows (main.c:1909-1950):
 *   q[n_heads * hd], k/v rows at k + t * kv_stride (+ kvh * hd), t in [0, nwin).
 * out[n_heads * hd] = softmax(K q) V per head, GQA kv head = h / (n_heads/n_kv). */
int g4_attn_decode(float *out, const float *q, const float *k, const float *v, int nwin,
                   int kv_stride, int n_heads, int n_kv_heads, int hd);

/* Device-pointer forms for callers that keep activations in HBM.  `stream`
 * is a cudaStream_t (NULL = the legacy default stream); nothing is
 * synchronised.  Weight pointers must come from g4d_weight_upload (device
 * layout: GGUF blocks, Q6_K split into planes).  `batch` activation vectors
 * are laid out back to back ([batch][n] in, [batch][d] out). */
int g4d_weight_upload(const void *host, int type, int n, int rows, void **dev);
int g4d_free(void *dev);
/* quantize_row_q8_K on device: y[batch][k/256] from x[batch][k]. */
int g4d_quantize_row_q8_K(const float *x, g4_block_q8_K *y, int k, int batch, void *stream);
/* mm on device (same semantics as g4_mm; q8 is a device buffer). */
int g4d_mm(float *o, const float *x, const void *w, int n, int d, int type, g4_block_q8_K *q8, int q8_ready,
           int batch, void *stream);
/* K-quant and BF16 matrices with batch >= the tensor-core threshold (default
 * 16) run as tcgen05 GEMMs over groups of up to 64 activations: Q4_K as exact
 * fp16 integer products, Q5_K as int8 x int8 -> int32 (both with exact
 * integer block sums and an fp32 block epilogue), Q6_K as int8 x int8 ->
 * int32 on the activation's three fixed-point pieces (exact block dots), BF16
 * on activations split into three bf16 parts; smaller batches use the
 * streaming GEMV (bit-identical to the tensor-core results for the K-quants).  The tensor-core path keeps a per-device scratch
 * (activation operand, K-slice partials) shared by all calls: calls on
 * different streams must be ordered by the caller.  Not part of the
 * reference interface: sets the threshold (>= 1) and returns the previous
 * one, or -1 on a bad value. */
int g4_set_tc_min_batch(int min_batch);

/* Which kernel runs Q4_K/Q5_K GEMVs of one activation vector (g4_mm,
 * g4d_mm with batch 1, the engine's batch-1 step): 1 (default) the row-owner
 * kernel (a warp streams whole rows and folds them in registers), 0 the
 * tiled streaming kernel used for 2..15 activations.  Both give bit-identical
 * results.  Not part of the reference interface; returns the previous value. */
int g4_set_gemv_rows(int on);

/* Decode attention (the result of g4_attn_decode) on DEVICE pointers, for
 * callers that cannot let the library allocate device memory.  This entry
 * point has no counterpart in the reference.  It calls no cudaMalloc/cudaFree:
 * its scratch is a 4 MiB array compiled into the library (held on every GPU
 * that loads it), so n_heads * ceil(nwin/32) * (hd + 2) * 4 bytes plus about
 * 512 must fit in 4 MiB, else G4_ERR_ARG.  k and v are [n_kv_heads][nwin][hd]
 * (each kv head's rows contiguous), q [n_heads * hd], out [n_heads * hd].
 * The first call on a device looks the array up and should precede any
 * stream capture; calls that may overlap on the GPU share the array and must
 * be serialised by the caller.  The call is asynchronous: if a bounded
 * device-side wait gives up (not expected on a healthy GPU), `out` is filled
 * with NaN instead of a status being returned. */
int g4d_attn_decode_noalloc(float *out, const float *q, const float *k, const float *v, int nwin, int n_heads,
                            int n_kv_heads, int hd, void *stream);

/* ------------------------------------------------------------------ */
/* 2. Device-resident engine                                           */
/* ------------------------------------------------------------------ */

/* Model description: the reference's Config + Weights (main.c:623-629, 667-692)
 * as plain fields.  All tensor pointers are HOST pointers (e.g. into the GGUF
 * mmap); the engine copies them to the device at creation. */
typedef struct g4_model_desc {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size;
    int ple_dim, sliding_window;
    int head_dim_swa, head_dim_full, n_rot_swa, n_rot_full;
    float rope_theta, rope_theta_swa, norm_eps, logit_softcapping;
    const int *swa_layers; /* n_layers flags (1 = sliding window) or NULL */
    int swa_pattern;       /* used when swa_layers == NULL (main.c:716-721) */

    const void *embd;      int embd_t;       /* token_embd, tied LM head */
    const void *ple_tok;   int ple_tok_t;    /* per_layer_token_embd */
    const void *ple_proj;  int ple_proj_t;   /* per_layer_model_proj */
    const float *ple_proj_norm;              /* per_layer_proj_norm [ple_dim] */
    const float *rope_freqs;                 /* [n_rot_full/2] or NULL */
    const float *norm_out;                   /* output_norm [dim] */

    /* per-layer arrays, n_layers entries each */
    const float *const *attn_norm;
    const float *const *post_attn_norm;
    const float *const *ffn_norm;
    const float *const *post_ffw_norm;
    const float *const *q_norm;
    const float *const *k_norm;
    const float *const *post_norm;
    const float *const *out_scale;           /* entries may be NULL */
    const void *const *wq;       const int *wq_t;
    const void *const *wk;       const int *wk_t;
    const void *const *wv;       const int *wv_t;
    const void *const *wo;       const int *wo_t;
    const void *const *gate;     const int *gate_t;
    const void *const *up;       const int *up_t;
    const void *const *down;     const int *down_t;
    const void *const *inp_gate; const int *inp_gate_t;
    const void *const *proj;     const int *proj_t;
} g4_model_desc;

typedef struct g4_engine g4_engine;

/* sizeof(g4_model_desc) as compiled into the library (FFI layout check). */
size_t g4_model_desc_bytes(void);

/* Upload the model to `device` and allocate state for `max_batch` sequences
 * of up to `max_seq` positions.  Returns NULL on error (see g4_last_error). */
g4_engine *g4_engine_create(const g4_model_desc *m, int device, int max_seq, int max_batch);
/* As g4_engine_create, plus room for batched prefill: g4_prefill calls of up
 * to prefill_rows rows (sliding-window caches then hold window + prefill_rows
 * slots).  Not part of the reference interface. */
g4_engine *g4_engine_create_ex(const g4_model_desc *m, int device, int max_seq, int max_batch, int prefill_rows);
int g4_engine_destroy(g4_engine *e);
/* Device bytes held by the engine (weights, KV cache, state). */
size_t g4_engine_device_bytes(const g4_engine *e);

/* forward (main.c:1838-2029) for sequence 0 at position pos.
 * lm_mode 0: no LM head (prefill); 1: softcapped logits (copied to `logits`
 * when not NULL); 2: argmax only.  Returns the argmax token for lm_mode 1/2
 * (first index of the largest softcapped logit), 0 for lm_mode 0, -1 on error. */
int g4_forward(g4_engine *e, int token, int pos, int lm_mode, float *logits);

/* Greedy generation for one sequence, the temp <= 0 path of generate
 * (main.c:2335-2488): prefill prompt[0..n_prompt) one position at a time,
 * then max_new greedy tokens.  Stops after emitting `eos` (eos < 0: never).
 * out_tokens receives the generated ids; returns their count or -1. */
int g4_generate_greedy(g4_engine *e, const int *prompt, int n_prompt, int max_new, int eos,
                       int *out_tokens);

/* generate (main.c:2335-2488) with the reference's sampler for one sequence:
 * prefill prompt[0..n_prompt) one position at a time, then up to max_new
 * tokens, each from sample_token(temp, topp, topk) after the repetition
 * penalty over the last penalty_last_n generated tokens (penalty_last_n <= 0:
 * all of them; repeat_penalty <= 1: none).  rng starts at seed (0 -> 1) as in
 * main.c:2341.  The penalty and the top-k candidates run on the GPU; the
 * temperature / top-p tail on the host with the reference's expressions.
 * temp <= 0 is greedy.  Stops before emitting `eos` (eos < 0: never).
 * Returns the number of tokens written to out_tokens, or -1. */
int g4_generate(g4_engine *e, const int *prompt, int n_prompt, int max_new, float temp, float topp, int topk,
                float repeat_penalty, int penalty_last_n, uint64_t seed, int eos, int *out_tokens);

/* Batched prefill (the lm_mode 0 forwards of generate's prompt loop,
 * main.c:2366-2402, for many positions and sequences at once): row i is token
 * tokens[i] of sequence seq[i] at position pos[i].  All rows run through every
 * layer together (tensor-core GEMMs over the rows); each layer stores the K/V
 * rows of all rows, then each row attends over its own causal window with
 * the decode step's arithmetic, so the cache and hidden states equal those of
 * decoding the rows one position at a time, bit for bit.  The rows of one
 * sequence must be distinct positions spanning fewer than prefill_rows, and
 * every earlier position of the sequence must already be in the cache (an
 * earlier call).  No LM head: run the last prompt token through
 * g4_forward / g4_decode_batch.  n_rows <= the engine's prefill_rows. */
int g4_prefill(g4_engine *e, int n_rows, const int *seq, const int *pos, const int *tokens);

/* Batched greedy decode of B independent sequences in lockstep (all at the
 * same position).  tokens[B] in, next[B] out (argmax of each sequence's
 * softcapped logits).  lm_mode 0 skips the LM head (next untouched). */
int g4_decode_batch(g4_engine *e, int B, const int *tokens, int pos, int lm_mode, int *next);

/* One batched step with the sampler: tokens[B] in; for each sequence b the
 * repetition penalty over recent[b * recent_ld .. + n_recent[b]) (host
 * arrays; ignored when repeat_penalty <= 1), then sample_token(temp, topp,
 * topk) with its own rng[b] (advanced); next[B] out.  The logits stay on the
 * GPU; only the top-k candidates reach the host. */
int g4_decode_batch_sample(g4_engine *e, int B, const int *tokens, int pos, float temp, float topp, int topk,
                           float repeat_penalty, const int *recent, int recent_ld, const int *n_recent, uint64_t *rng,
                           int *next);

/* Device-pointer form used by bench loops: tokens/next are DEVICE int32[B]
 * buffers; enqueued on the engine stream, no synchronisation. */
int g4_decode_batch_device(g4_engine *e, int B, const int *tokens_dev, int pos, int lm_mode,
                           int *next_dev);
/* Block until the engine stream is idle. */
int g4_engine_sync(g4_engine *e);
/* The engine's CUDA stream (cudaStream_t as void*) for event timing. */
void *g4_engine_stream(g4_engine *e);

/* Benchmark helper: fill the KV rows of positions [0, npos) of every KV layer
 * and sequence with seeded values in [-1, 1), so decoding can start at a long
 * context without a prefill (a decode step's work does not depend on the
 * cached values).  Not part of the reference interface. */
int g4_engine_fill_kv(g4_engine *e, int npos, uint64_t seed);

/* Benchmark helper: time `reps` rounds of the decode attention of layers[0..n)
 * (in that order) for the first `batch` sequences at the position of the most
 * recent step, on the engine stream with CUDA events; *ms = total milliseconds.
 * Re-running a step's attention rewrites the same K/V row, so the engine state
 * is unchanged.  Not part of the reference interface. */
int g4_engine_time_attention(g4_engine *e, const int *layers, int n, int batch, int reps, float *ms);

/* Batch size from which the engine's step runs the K-quant projections and
 * the LM head on the tensor cores (default 2; below it, streaming GEMVs with
 * the residual/norm work fused in).  Results do not depend on it: both paths
 * compute every row bit-identically.  Not part of the reference interface;
 * returns the previous value, or -1 on a bad argument. */
int g4_engine_set_tc_min_batch(g4_engine *e, int min_batch);

/* Rows of the KV window that one CTA of the decode attention takes, for the
 * sliding-window layers and for the global layers (multiples of 32; 0 keeps
 * the default 64 / 256).  Fixed per engine, never derived from the batch, so
 * a sequence's results do not depend on the batch size; changing it changes
 * the float summation order of attention.  Not part of the reference
 * interface (main.c:1909-1950 has one sequential pass). */
int g4_engine_set_attn_split(g4_engine *e, int sliding, int global);

/* Number of kernels in the most recent step (the nodes of its CUDA graph). */
int g4_engine_last_step_kernels(const g4_engine *e);

/* Optional row-split LM head over `world` GPUs, one engine per GPU (one
 * process per GPU), each decoding its own sequences in lockstep with the
 * others (the same B, positions and lm_mode on every rank).  Rank r owns the
 * vocabulary rows [r*chunk, (r+1)*chunk) (g4_lm_split_rows).  Each step
 * gathers every rank's output-normed hidden states (one NCCL all-gather of
 * B*dim floats), computes its rows for all of them with the softcap and a
 * packed (value, first index) key per sequence, gathers the keys (one
 * all-gather of 8 bytes per sequence and rank) and keeps the largest key of
 * each of its sequences: the first index of the largest logit over the whole
 * vocabulary, as the reference's greedy scan (main.c:2045-2050).  Logits are
 * not returned in this mode.  nccl_id: 128 bytes from g4_nccl_unique_id on
 * one rank, passed to every rank.  NCCL is loaded at run time
 * (libnccl.so.2).  Not part of the reference interface. */
int g4_nccl_unique_id(void *nccl_id);
int g4_engine_lm_split(g4_engine *e, const void *nccl_id, int rank, int world);
/* Host helpers of the split (used by tests): the rows of rank `rank`
 * (returns the rows per rank, -1 on error), the merge of the gathered keys
 * keys_all[world][world*B] into out[B] for rank `rank`, and the packed key of
 * the first largest value of logits[n] with row indices offset by row0. */
int g4_lm_split_rows(int vocab, int world, int rank, int *row0, int *row1);
int g4_lm_split_merge(const uint64_t *keys_all, int world, int rank, int B, int chunk, uint64_t *out);
int g4_argmax_keys(const float *logits, int n, int row0, uint64_t *key);

/* Test taps: hidden state x[dim] of sequence b after the last step, and the
 * K/V rows (n_kv_heads * head_dim floats each) stored for (layer, pos). */
int g4_engine_get_hidden(g4_engine *e, int b, float *x);
int g4_engine_get_kv(g4_engine *e, int b, int layer, int pos, float *k, float *v);
/* Test tap: write the K/V rows of positions [pos0, pos0+npos) of sequence b
 * in a KV layer (< 24) from host rows k/v[npos][n_kv_heads * head_dim], so a
 * test can start the engine and the reference from identical caches. */
int g4_engine_set_kv(g4_engine *e, int b, int layer, int pos0, int npos, const float *k, const float *v);

#ifdef __cplusplus
}
#endif
#endif /* G4B200_H */
