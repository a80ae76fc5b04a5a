// g4_kernels.cuh — launchers of the sm_100a kernels (internal to libg4b200).
#pragma once
#include <cuda.h>  // CUtensorMap

#include "g4_internal.cuh"
#include "g4_prologue.cuh"

namespace g4 {

enum Epilogue {
    EPI_STORE = 0,           // out[row] = acc
    EPI_GELU_MUL = 1,        // out[row] = gelu(acc(w)) * acc(w2)        (FFN, main.c:1973-1978)
    EPI_SOFTCAP_ARGMAX = 2,  // out[row] = cap*tanh(acc/cap); argmax key (LM head, main.c:1780-1796)
    EPI_GELU_SCALE = 3       // out[row] = gelu(acc) * evec[row]           (PLE gate, main.c:1986-1991)
};

constexpr int kMaxJobs = 3;

// Canonical summation order of one output row of a K-quant matrix, shared by
// the streaming GEMV and the tensor-core GEMMs so that a sequence gets
// bit-identical results whether it is decoded alone or in a batch.  Each
// super-block b of the row contributes an exact term pair (a_b, c_b) (Q4_K/
// Q5_K: a = Q8_K block scale, c = d*float(sumi_s) - dmin*sumi_m; Q6_K: a =
// float of the exact integer dot, c = d * activation block scale), and
//   v = 0; P = 0
//   for b = 0 .. nb-1:
//       if b > 0 and seg_start(b): v = v + P; P = 0
//       P = fma(a_b, c_b, P)
//   v = v + P
// The segments are the K ranges a tensor-core launch hands to different
// CTAs: stream-K units of `share` consecutive (row tile, super-block) units
// with this matrix's row tile 0 at unit index tile0 * nb (Q4_K), or uniform
// slices of `kslice` super-blocks (Q5_K, Q6_K).  The plan depends only on the
// matrix shapes and the SM count, never on the batch.
struct RowOrder {
    int tile0;   // global row-tile index of this matrix's row 0 in its tensor-core launch
    int share;   // stream-K units per CTA, or 0
    int kslice;  // super-blocks per uniform K slice, or 0
};
__host__ __device__ __forceinline__ bool seg_start(const RowOrder &o, int row, int nb, int b) {
    if (b == 0) return false;
    if (o.share > 0 && ((long long)(o.tile0 + row / 128) * nb + b) % o.share == 0) return true;
    return o.kslice > 0 && b % o.kslice == 0;
}

// One matrix of a grouped K-quant GEMV launch.
struct GemvJob {
    const void *w;       // device tensor (GGUF blocks; Q6_K as planes)
    const void *w2;      // second matrix of EPI_GELU_MUL (same type and shape) or null
    const void *act;     // Q4/Q5: BlockQ8_K [B][n/256];  Q6: fp32 [B][act_stride]
    float *out;          // [B][out_stride] (may be null for EPI_SOFTCAP_ARGMAX)
    unsigned long long *amax;  // [B] argmax keys for EPI_SOFTCAP_ARGMAX
    const float *evec;   // [B][ld_evec] multiplier of EPI_GELU_SCALE
    int type, n, rows, act_stride, out_stride, epi, rt, cta_begin, ld_evec, ctas;
    float cap;
    RowOrder ord, ord2;  // canonical row order of w (and w2)
    int explicit_order;  // 0: the launcher sets ord (and ord2) for w alone in its own tensor-core launch
};
struct GemvJobs {
    GemvJob j[kMaxJobs];
    int njobs;
    // Optional fused prologue (batch <= 8): the activation of every job is
    // computed per CTA from the residual stream instead of read from `act`.
    Prologue pro;
    int has_pro;     // 1: run `pro`; jobs' act/act_stride are ignored
    int pro_writer;  // 1: CTA 0 of this launch stores x' (pro.x_out)
    int red_floats;  // set by the launcher: offset of the prologue area in shared memory
    int *err;        // device status word: a bounded wait that gave up stores G4_ERR_TIMEOUT
};
constexpr int kFusedMaxBatch = 8;

int launch_quantize_q8k(const float *x, int ldx, void *y, int n, int B, cudaStream_t st);
int launch_gemv_kquant(GemvJobs &jobs, int B, cudaStream_t st);
int set_gemv_rows(int on);  // 1: batch-1 Q4_K/Q5_K GEMVs on gemv_rows_kernel; returns the previous value
int launch_gemv_dense(const void *w, int type, int n, int rows, const float *x, int ldx, float *out, int ldo,
                      int B, int epi, const float *evec, int ld_evec, cudaStream_t st,
                      const Prologue *pro = nullptr, int pro_writer = 0);
int launch_qk_block_sums(const void *w, int type, int n, int rows, const void *q8, int *ss, int *sm,
                         cudaStream_t st);

// ---- attention (k_attn.cu)

// One attention layer for the fused decode-attention kernel.
struct AttnLayer {
    int hd, n_rot, n_heads, n_kv;
    const float *q, *k, *v;         // raw projections [B][n_heads*hd], [B][n_kv*hd]
    int prep;                       // 1: q-norm + RoPE here (0: q is ready)
    const float *q_norm, *k_norm;   // device [hd]
    const float2 *rope;             // device [max_seq][n_rot/2] (cos, sin) or null
    int append;                     // 1: this layer stores K/V (l < 24)
    float *kc, *vc;                 // cache of THIS layer (append target)
    int ring;                       // slots of this layer's cache (window ring or max_seq)
    const float *src_kc, *src_vc;   // cache read by attention (this layer or 22/23)
    int src_ring;                   // slots of the source cache
    int window;                     // 0: full causal, else sliding window
    float eps;
    int *err;                       // status word for bounded waits (may be null)
    float *qo;                      // output [B][n_heads*hd]
    float *part;                    // scratch [B][n_heads][max_chunks][hd+2]
    int *counters;                  // [B][n_kv] zero-initialised tickets
    int max_chunks;
    uint8_t *op_bq;                 // tensor-core operand of qo for a Q4_K output projection (tc4_store_q8
    float *op_yd;                   // layout, one group of op_np <= 64 sequences), written by the merging
    int op_np;                      // CTAs; null: not written
    int split;                      // rows per canonical split of attn_stream_kernel (a multiple of 32);
                                    // 0: 64 for a sliding window, 256 otherwise
    int early;                      // 1: every cache row but `pos` was written before the launch's
                                    //    stream predecessor started (earlier graph launches), so it
                                    //    may be copied before the grid dependency wait
    // Prefill: row b of the launch is the query of cache sequence row_seq[b] at position row_pos[b]
    // (device arrays; null: row b is sequence b at *pos_dev).  The K/V rows of the launch's positions
    // are stored beforehand by launch_kv_append (append = 0 here).
    const int *row_pos, *row_seq;
};
// Store the K/V rows of `rows` prefill rows (k-norm + RoPE of K, norm of V, as the attention kernels
// do for a decode step's new row) into the layer's cache.
int launch_kv_append(const AttnLayer &L, int rows, cudaStream_t st);
int launch_attention(const AttnLayer &L, int B, const int *pos_dev, int max_seq, cudaStream_t st);
int attn_chunk_size();
// Host: reference-exact RoPE table for positions [0, npos).
void rope_table_host(float2 *out, int npos, int n_rot, float base, float freq_scale, const float *ff);

// ---- glue (k_glue.cu)
struct ResNorm {
    const float *x_in;      // [B][dim] residual stream
    const float *delta;     // [B][dim] sublayer output or null
    const float *post_w;    // norm weight for delta
    const float *scale;     // layer_output_scale (device, 1 float) or null
    float *x_out;           // [B][dim] (may alias x_in)
    const float *pre_w;     // pre-norm weight or null
    float *xn_out;          // [B][dim] normed output (pre_w) or null
    void *q8_out;           // [B][dim/256] BlockQ8_K of xn_out or null
    int dim;
    float eps;
    // Tensor-core B operands of the output vector (xn when pre_w is set, else x) for sequence
    // blockIdx.x of one group of tc_np <= 64 sequences, in the layouts of tc4_quant_kernel,
    // tc6_split_kernel and bf3_split_kernel (null: not written).  Padding slots are not written.
    uint8_t *tc4_bq;
    float *tc4_yd;
    uint8_t *tc6_bq;
    float *tc6_ys;
    uint8_t *bf3_bq;
    int tc_np;
};
int launch_resnorm(const ResNorm &r, int B, cudaStream_t st);
int launch_embed_v(const void *embd, int embd_t, int dim, size_t vocab, float emb_scale, const void *ple_tok,
                   int ple_tok_t, int ple_row, float ple_scale, const int *tokens, unsigned long long *keys,
                   float *x, float *ple_out, int B, cudaStream_t st);
int launch_gelu_mul(float *a, const float *b, size_t n, cudaStream_t st);
int launch_softcap_argmax(float *logits, int vocab, int ld, float cap, unsigned long long *keys, int B,
                          cudaStream_t st);
int launch_repack_q6(const void *raw_dev, size_t nblk, size_t blk_offset, void *planes_dev, int nb,
                     cudaStream_t st);
int launch_ple_mix(const float *ple_tok, float *ple_ctx, const float *norm_w, int pd, int L, float ctx_scale,
                   float mix_scale, float eps, float *ple_out, int B, cudaStream_t st);
int launch_keys_to_tokens(const unsigned long long *keys, int *tokens, int B, cudaStream_t st);
int launch_fill_kv(float *c, int B, int n_kv, int ring, int hd, int npos, uint64_t seed, cudaStream_t st);

// ---- sampler (k_sample.cu)
int launch_rep_penalty(float *logits, int ld, const int *recent, int rec_ld, const int *nrec, int vocab, float penalty,
                       int B, cudaStream_t st);
int launch_topk(const float *logits, int ld, int n, int k, float *out_v, int *out_i, int B, cudaStream_t st);
int sample_tail_host(const float *vals, const int *idx, int k, float temp, float topp, uint64_t *rng, float *p);

// ---- batched BF16-weight GEMM on tcgen05 (k_gemm_bf16tc.cu), 16..64 sequences
size_t bf16tc_operand_bytes(int n);
int bf16tc_weight_map(CUtensorMap *m, const void *w, int n, int rows);
int launch_bf3_split(const float *x, int ldx, int B, int n, int np, uint8_t *bq, cudaStream_t st);
int launch_gemm_bf16tc(const CUtensorMap *tm, int n, int rows, const uint8_t *bq, int B, int np, float *out, int ldo,
                       float *part, size_t part_bytes, int *err, int nsm, int epi, const float *evec,
                       int ld_evec, cudaStream_t st);
int prime_bf16tc_attrs();

// ---- batched Q6_K GEMM on tcgen05 (k_gemm_q6tc.cu), 16..64 sequences
size_t tc6_operand_bytes(int n);     // x1/x2 operand + scales of one activation (NP = 64)
size_t tc6_ys_offset(int n);
size_t tc6_maps_bytes();             // bytes of the opaque tensor-map bundle
int tc6_weight_maps(void *maps_out, const void *w, int n, int rows);
int prime_tc6_attrs();
int prime_tc_attrs();
int launch_tc6_split(const float *x, int ldx, int B, int n, int np, uint8_t *bq, float *ys, cudaStream_t st);
int launch_gemm_q6tc(const void *maps, const void *w, int n, int rows, const uint8_t *bq, const float *ys, int B,
                     int np, float *out, int ldo, float *part, size_t part_bytes, int *err, int nsm,
                     int epi, float cap, unsigned long long *keys, cudaStream_t st, int *tickets);

// ---- batched K-quant GEMM on tcgen05 (k_gemm_tc.cu), 16..64 sequences
struct TcPlan {
    int ksplit, kslice, units, grid;  // K-slices per 128-row tile, blocks per slice, work units, CTAs
};
struct Q4Plan {
    int share, grid, nseg_max;        // units per CTA, CTAs, most CTAs sharing one row tile
};
Q4Plan q4_plan(int tiles, int nb, int nsm);
// Row orders of the tensor-core launches (the GEMV follows the same order):
//   Q4_K alone, or the first / second matrix of a pair sharing one launch;
RowOrder q4_row_order(int rows_a, int rows_b, int n, int nsm, int which);  // which: 0 = a, 1 = b (rows_b 0: no pair)
//   Q5_K (uniform K slices of tc_plan);  Q6_K (its own uniform plan; argmax: whole rows).
RowOrder q5_row_order(int rows, int n, int nsm);
RowOrder q6_row_order(int rows, int n, int nsm, bool argmax);
// Q4_K GEMM of one or two matrices (same n, same activation; w2 = null for one) in one launch,
// plus the merge of split row tiles.  epi: EPI_STORE, or EPI_GELU_MUL for a gate/up pair
// (out = GELU(gate) * up; out2 unused).
int launch_gemm_q4tc2(const CUtensorMap *tm, const void *w, int rows, float *out, int ldo, const CUtensorMap *tm2,
                      const void *w2, int rows2, float *out2, int ldo2, int n, const uint8_t *bq, const float *yd, int B,
                      int np, float *part, size_t part_bytes, int *err, int nsm, cudaStream_t st,
                      int epi, int *tickets);
int tc_np(int B);                    // padded sequence count: 16, 32 or 64
size_t tc_operand_bytes(int n);      // B operand + block scales of one activation (NP = 64)
size_t tc_yd_offset(int n);          // where the block scales start inside that buffer
TcPlan tc_plan(int rows, int nb, int nsm);
size_t tc_part_bytes(int rows, int n, int nsm);
int launch_tc_merge(const float *part, int ksplit, int np, int rows, int B, float *out, int ldo, int epi,
                    const float *evec, int ld_evec, cudaStream_t st);
int tc_weight_map(CUtensorMap *m, const void *w, int type, int n, int rows);
int launch_tc_quant(int type, const float *x, int ldx, int B, int n, int np, uint8_t *bq, float *yd, cudaStream_t st);
int launch_tc_from_q8(int type, const void *q8, int B, int n, int np, uint8_t *bq, float *yd, cudaStream_t st);
int launch_gemm_tc(const CUtensorMap *tm, const void *w, int type, int n, int rows, const uint8_t *bq, const float *yd, int B, int np,
                   float *out, int ldo, float *part, size_t part_bytes, int *err, int nsm,
                   cudaStream_t st, int *tickets);

}  // namespace g4
