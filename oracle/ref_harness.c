/*
 * ref_harness.c — TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * Compiles the reference engine gemma4-4b/cpu-blas/main.c UNCHANGED into this
 * translation unit (the path comes from -DG4_REF_MAIN_C=...), so that its
 * `static` functions become callable, and exports thin wrappers with C
 * linkage.  The result is oracle/_ref/libg4ref.so, used to
 *   - pin the C restatement in oracle/g4_oracle.c,
 *   - generate the golden fixtures under tests/golden/,
 *   - time the reference CPU path (bench.py --impl reference).
 * Nothing here reimplements reference arithmetic: each wrapper forwards to the
 * reference function named in its comment.
 */
#define main g4ref_cli_main
#include G4_REF_MAIN_C
#undef main

#include "../include/g4b200.h"

/* OpenBLAS fixed to one thread and OpenMP sized as main() does (main.c:2627). */
void ref_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
    openblas_set_num_threads(1);
}
int ref_max_threads(void) { return omp_get_max_threads(); }

/* quantize_row_q8_K (AVX2 when built with AVX2, main.c:282-340) and the scalar
 * quantize_row_q8_K_ref (main.c:247-279). */
void ref_quantize_row_q8_K(const float *x, void *y, int k) { quantize_row_q8_K(x, (BlockQ8_K *)y, k); }
void ref_quantize_row_q8_K_scalar(const float *x, void *y, int k) { quantize_row_q8_K_ref(x, (BlockQ8_K *)y, k); }

/* vec_dot_q{4,5}_K_q8_K (main.c:476-593) and their generic twins (347-473). */
void ref_vec_dot_q4_K_q8_K(int n, const void *x, const void *y, float *out) {
    vec_dot_q4_K_q8_K(n, (const BlockQ4_K *)x, (const BlockQ8_K *)y, out);
}
void ref_vec_dot_q5_K_q8_K(int n, const void *x, const void *y, float *out) {
    vec_dot_q5_K_q8_K(n, (const BlockQ5_K *)x, (const BlockQ8_K *)y, out);
}
void ref_vec_dot_q4_K_q8_K_generic(int n, const void *x, const void *y, float *out) {
    vec_dot_q4_K_q8_K_generic(n, (const BlockQ4_K *)x, (const BlockQ8_K *)y, out);
}
void ref_vec_dot_q5_K_q8_K_generic(int n, const void *x, const void *y, float *out) {
    vec_dot_q5_K_q8_K_generic(n, (const BlockQ5_K *)x, (const BlockQ8_K *)y, out);
}

/* dequant_one_block_to (main.c:767-776) over nblocks consecutive blocks. */
void ref_dequant(const void *blocks, int type, float *dst, int nblocks) {
    size_t bs = block_size_quant(type);
    for (int b = 0; b < nblocks; b++)
        dequant_one_block_to((const uint8_t *)blocks + (size_t)b * bs, type, dst + (size_t)b * QK_K);
}

/* mm and its row kernels (main.c:1494-1694). */
void ref_mm(float *o, const float *x, const void *w, int n, int d, int type, void *q8, int q8_ready) {
    mm(o, x, w, n, d, type, (BlockQ8_K *)q8, q8_ready);
}
void ref_mm_quant_rows(float *o, const float *x, const void *w, int n, int d, int type) {
    mm_quant_rows(o, x, w, n, d, type);
}
void ref_mm_quant_dot_rows(float *o, const void *w, int n, int d, int type, const void *q8) {
    mm_quant_dot_rows(o, w, n, d, type, (const BlockQ8_K *)q8);
}
int ref_mm_argmax_row(const float *x, const void *w, int n, int d, int type, void *q8) {
    return mm_argmax_row(x, w, n, d, type, (BlockQ8_K *)q8);
}
void ref_set_f32_matmul(int on) { g_f32_matmul = on; }

/* Math primitives (main.c:1451-1492, 1725-1745). */
void ref_rmsnorm(float *o, const float *x, const float *w, int n, float eps) { rmsnorm(o, x, w, n, eps); }
void ref_rmsnorm_head_inplace(float *v, const float *w, int nh, int hd, float eps) {
    rmsnorm_head_inplace(v, w, nh, hd, eps);
}
void ref_rmsnorm_head_noweight_inplace(float *v, int nh, int hd, float eps) {
    rmsnorm_head_noweight_inplace(v, nh, hd, eps);
}
void ref_softmax(float *x, int n) { softmax(x, n); }
float ref_gelu(float x) { return gelu_f32(x); }
void ref_apply_rope_neox(float *vec, int n_heads, int head_dim, int n_rot, int pos, float freq_base,
                         float freq_scale, const float *freq_factors) {
    apply_rope_neox(vec, n_heads, head_dim, n_rot, pos, freq_base, freq_scale, freq_factors);
}
/* sample_token (main.c:2044-2112); temp <= 0 is the greedy first-max scan. */
int ref_sample_token(float *logits, int n, float temp, float topp, int topk, uint64_t *rng) {
    return sample_token(logits, n, temp, topp, topk, rng);
}
float ref_rng_f32(uint64_t *state) { return rng_f32(state); }

/* ---- Model built from a g4_model_desc (fields of Config/Weights) ---- */

void *ref_model_create(const g4_model_desc *dsc, int max_seq) {
    Model *m = (Model *)calloc(1, sizeof(Model));
    Config *c = &m->cfg;
    Weights *w = &m->w;
    int L = dsc->n_layers;
    c->dim = dsc->dim; c->hidden_dim = dsc->hidden_dim; c->n_layers = L;
    c->n_heads = dsc->n_heads; c->n_kv_heads = dsc->n_kv_heads; c->vocab_size = dsc->vocab_size;
    c->max_seq = max_seq; c->ple_dim = dsc->ple_dim; c->sliding_window = dsc->sliding_window;
    c->shared_kv_layers = 18; c->swa_pattern = dsc->swa_pattern;
    c->head_dim_swa = dsc->head_dim_swa; c->head_dim_full = dsc->head_dim_full;
    c->n_rot_swa = dsc->n_rot_swa; c->n_rot_full = dsc->n_rot_full;
    c->rope_theta = dsc->rope_theta; c->rope_theta_swa = dsc->rope_theta_swa;
    c->norm_eps = dsc->norm_eps; c->logit_softcapping = dsc->logit_softcapping;
    c->swa_layers = NULL;
    if (dsc->swa_layers) {
        c->swa_layers = (int *)calloc((size_t)L, sizeof(int));
        for (int l = 0; l < L; l++) c->swa_layers[l] = dsc->swa_layers[l] ? 1 : 0;
    }
    w->embd = (void *)dsc->embd; w->embd_t = dsc->embd_t;
    w->ple_tok = (void *)dsc->ple_tok; w->ple_tok_t = dsc->ple_tok_t;
    w->ple_proj = (void *)dsc->ple_proj; w->ple_proj_t = dsc->ple_proj_t;
    w->ple_proj_norm = (float *)dsc->ple_proj_norm;
    w->rope_freqs = (float *)dsc->rope_freqs;
    w->norm_out = (float *)dsc->norm_out;
#define G4_CP_F(field) do { w->field = (float **)calloc((size_t)L, sizeof(float *)); \
        for (int l = 0; l < L; l++) w->field[l] = dsc->field ? (float *)dsc->field[l] : NULL; } while (0)
#define G4_CP_W(field) do { w->field = (void **)calloc((size_t)L, sizeof(void *)); \
        w->field##_t = (int *)calloc((size_t)L, sizeof(int)); \
        for (int l = 0; l < L; l++) { w->field[l] = dsc->field ? (void *)dsc->field[l] : NULL; \
                                      w->field##_t[l] = dsc->field##_t ? dsc->field##_t[l] : 0; } } while (0)
    G4_CP_F(attn_norm); G4_CP_F(post_attn_norm); G4_CP_F(ffn_norm); G4_CP_F(post_ffw_norm);
    G4_CP_F(q_norm); G4_CP_F(k_norm); G4_CP_F(post_norm); G4_CP_F(out_scale);
    G4_CP_W(wq); G4_CP_W(wk); G4_CP_W(wv); G4_CP_W(wo); G4_CP_W(gate); G4_CP_W(up); G4_CP_W(down);
    G4_CP_W(inp_gate); G4_CP_W(proj);
#undef G4_CP_F
#undef G4_CP_W
    alloc_state(&m->s, c);
    m->tok.bos = 2; m->tok.eos = -1; m->tok.eot = -1;
    return m;
}

void ref_model_free(void *mp) {
    Model *m = (Model *)mp;
    if (!m) return;
    free_state(&m->s);
    free_weight_ptrs(&m->w, m->cfg.n_layers);
    free(m->cfg.swa_layers);
    free(m);
}

/* forward (main.c:1838-2029). */
void ref_forward(void *mp, int token, int pos, int lm_mode) { forward((Model *)mp, token, pos, lm_mode); }
const float *ref_model_logits(void *mp) { return ((Model *)mp)->s.logits; }
int ref_model_argmax(void *mp) { return ((Model *)mp)->s.argmax_tok; }
const float *ref_model_x(void *mp) { return ((Model *)mp)->s.x; }
const float *ref_model_kc(void *mp, int layer, int pos) {
    Model *m = (Model *)mp;
    return kc_at(&m->s, layer, pos, m->cfg.max_seq);
}
const float *ref_model_vc(void *mp, int layer, int pos) {
    Model *m = (Model *)mp;
    return vc_at(&m->s, layer, pos, m->cfg.max_seq);
}

/* The temp <= 0 path of generate (main.c:2335-2488) without the tokenizer
 * printing: same lm_mode choice (2372-2379), same next-token rule
 * (2401-2402, 2427 via sample_token), eos stop (2435). */
int ref_generate_greedy(void *mp, const int *prompt, int n_prompt, int max_new, int eos, int *out) {
    Model *m = (Model *)mp;
    uint64_t rng = 1;
    int fast_argmax = m->cfg.logit_softcapping <= 0.0f;
    int token = prompt[0], gen = 0;
    for (int pos = 0; pos < n_prompt + max_new - 1; pos++) {
        if (pos >= m->cfg.max_seq) break;
        int lm_mode = pos < n_prompt - 1 ? 0 : (fast_argmax ? 2 : 1);
        forward(m, token, pos, lm_mode);
        int next;
        if (pos < n_prompt - 1) {
            next = prompt[pos + 1];
        } else {
            next = fast_argmax ? m->s.argmax_tok
                               : sample_token(m->s.logits, m->cfg.vocab_size, 0.0f, 0.9f, DEFAULT_TOP_K, &rng);
            if (next == eos) break;
            out[gen++] = next;
        }
        token = next;
    }
    return gen;
}

/* apply_repetition_penalty (main.c:2114-2126). */
void ref_apply_repetition_penalty(float *logits, const int *tokens, int n_tokens, float penalty, int last_n) {
    apply_repetition_penalty(logits, tokens, n_tokens, penalty, last_n);
}

/* generate (main.c:2335-2488) with sampling, without the tokenizer output,
 * thinking control or forced tokens: the same lm_mode choice (2372-2379), the
 * repetition penalty over the generated tokens (2403-2405), sample_token with
 * DEFAULT_TOP_K (2427-2429), the eos stop (2435). */
int ref_generate_sample(void *mp, const int *prompt, int n_prompt, int max_new, float temp, float topp,
                        float repeat_penalty, int penalty_last_n, uint64_t seed, int eos, int *out) {
    Model *m = (Model *)mp;
    uint64_t rng = seed ? seed : 1;
    int token = prompt[0], gen = 0;
    int greedy = temp <= 0.0f;
    int fast_argmax = greedy && repeat_penalty <= 1.0f && m->cfg.logit_softcapping <= 0.0f;
    for (int pos = 0; pos < n_prompt + max_new - 1; pos++) {
        if (pos >= m->cfg.max_seq) break;
        int lm_mode = pos < n_prompt - 1 ? 0 : (fast_argmax ? 2 : 1);
        forward(m, token, pos, lm_mode);
        int next;
        if (pos < n_prompt - 1) {
            next = prompt[pos + 1];
        } else {
            if (repeat_penalty > 1.0f) apply_repetition_penalty(m->s.logits, out, gen, repeat_penalty, penalty_last_n);
            if (fast_argmax) next = m->s.argmax_tok;
            else if (greedy) next = sample_token(m->s.logits, m->cfg.vocab_size, 0.0f, topp, DEFAULT_TOP_K, &rng);
            else next = sample_token(m->s.logits, m->cfg.vocab_size, temp, topp, DEFAULT_TOP_K, &rng);
            if (next == eos) break;
            out[gen++] = next;
        }
        token = next;
    }
    return gen;
}

/* Fill the KV cache rows [0, npos) of every KV layer with seeded values in
 * [-1, 1) (xorshift64*).  Used only to time forward() at a long context
 * without running the prefill first: the work of a decode step does not
 * depend on the cached values. */
void ref_model_fill_kv(void *mp, int npos, uint64_t seed) {
    Model *m = (Model *)mp;
    uint64_t s = seed ? seed : 1;
    if (npos > m->cfg.max_seq) npos = m->cfg.max_seq;
    for (int l = 0; l < N_LAYER_KV && l < m->cfg.n_layers; l++)
        for (int p = 0; p < npos; p++) {
            float *k = kc_at(&m->s, l, p, m->cfg.max_seq), *v = vc_at(&m->s, l, p, m->cfg.max_seq);
            for (int i = 0; i < MAX_KV_DIM; i++) {
                k[i] = 2.0f * rng_f32(&s) - 1.0f;
                v[i] = 2.0f * rng_f32(&s) - 1.0f;
            }
        }
}
