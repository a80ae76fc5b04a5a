/*
 * g4_oracle.c — TEST INFRASTRUCTURE ONLY: the CPU restatement of the
 * reference algorithm for the decode hot path of thamada/Gemma4.c
 * (gemma4-4b/cpu-blas/main.c).  It is the checker the CUDA kernels are
 * compared against; nothing in the product links or calls it.
 *
 * Parity pin: every function below is checked against the reference itself,
 * compiled unchanged by oracle/Makefile into oracle/_ref/libg4ref.so, and
 * against the golden fixtures in tests/golden/ that were generated from it
 * (tests/test_oracle_pin.py).  Integer results (Q8_K bytes, per-block integer
 * sums, argmax indices) are bit-exact; float results follow the reference
 * arithmetic and summation order wherever the reference is scalar C (the
 * AVX2 dot kernels and OpenBLAS sgemv differ only by summation order).
 *
 * Each function names the reference lines it restates.  Built with
 * -std=c11 (GCC then does not contract a*b+c into FMA, like the reference).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/g4b200.h"

#define QK 256

#pragma pack(push, 1)
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[128]; } or_q4k;          /* main.c:95-100 */
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qh[32]; uint8_t qs[128]; } or_q5k; /* 102-108 */
typedef struct { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; uint16_t d; } or_q6k;  /* 110-115 */
#pragma pack(pop)
typedef g4_block_q8_K or_q8k;                                                               /* 118-122 */

/* IEEE half -> float (host_f16f32, main.c:128-149): exact for every input. */
float or_f16(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 31u, m = h & 1023u, bits;
    if (e == 0) {
        if (m == 0) bits = sign;
        else { /* subnormal: normalise the mantissa */
            int sh = 0;
            while (!(m & 1024u)) { m <<= 1; sh++; }
            bits = sign | ((uint32_t)(113 - sh) << 23) | ((m & 1023u) << 13);
        }
    } else if (e == 31) bits = sign | 0x7F800000u | (m << 13);
    else bits = sign | ((e + 112u) << 23) | (m << 13);
    float f; memcpy(&f, &bits, 4); return f;
}
/* bf16 -> float (host_bf16f32, main.c:151-156). */
float or_bf16(uint16_t h) { uint32_t b = (uint32_t)h << 16; float f; memcpy(&f, &b, 4); return f; }

/* 6-bit scale/min of sub-block j (get_scale_min_k4, main.c:162-170). */
static void or_scale_min(int j, const uint8_t *s, int *sc, int *mn) {
    if (j < 4) { *sc = s[j] & 63; *mn = s[j + 4] & 63; }
    else { *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4); *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
}

size_t or_block_bytes(int type) {
    return type == G4_Q4_K ? sizeof(or_q4k) : type == G4_Q5_K ? sizeof(or_q5k)
         : type == G4_Q6_K ? sizeof(or_q6k) : 0;
}

/* Dequantize one super-block to 256 floats: dequant_q4_k / q5_k / q6_k
 * (main.c:172-237), same float expressions: d*sc*q - dmin*m, d*sc*(q6-32). */
void or_dequant_block(const void *blk, int type, float *y) {
    if (type == G4_Q4_K || type == G4_Q5_K) {
        const uint8_t *scales, *qs, *qh = NULL;
        uint16_t hd, hm;
        if (type == G4_Q4_K) { const or_q4k *b = (const or_q4k *)blk; scales = b->scales; qs = b->qs; hd = b->d; hm = b->dmin; }
        else { const or_q5k *b = (const or_q5k *)blk; scales = b->scales; qs = b->qs; qh = b->qh; hd = b->d; hm = b->dmin; }
        const float d = or_f16(hd), dmin = or_f16(hm);
        for (int c = 0; c < 4; c++) {              /* 64-element chunks */
            int s0, m0, s1, m1;
            or_scale_min(2 * c, scales, &s0, &m0);
            or_scale_min(2 * c + 1, scales, &s1, &m1);
            const float d1 = d * s0, mm1 = dmin * m0, d2 = d * s1, mm2 = dmin * m1;
            for (int l = 0; l < 32; l++) {
                int lo = qs[32 * c + l] & 15, hi = qs[32 * c + l] >> 4;
                if (qh) { lo += (qh[l] >> (2 * c)) & 1 ? 16 : 0; hi += (qh[l] >> (2 * c + 1)) & 1 ? 16 : 0; }
                y[64 * c + l] = d1 * lo - mm1;
                y[64 * c + 32 + l] = d2 * hi - mm2;
            }
        }
    } else if (type == G4_Q6_K) {
        const or_q6k *b = (const or_q6k *)blk;
        const float d = or_f16(b->d);
        for (int h = 0; h < 2; h++) {              /* 128-element halves */
            const uint8_t *ql = b->ql + 64 * h, *qh = b->qh + 32 * h;
            const int8_t *sc = b->scales + 8 * h;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int q1 = ((ql[l] & 15) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q2 = ((ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[128 * h + l] = d * sc[is] * q1;
                y[128 * h + l + 32] = d * sc[is + 2] * q2;
                y[128 * h + l + 64] = d * sc[is + 4] * q3;
                y[128 * h + l + 96] = d * sc[is + 6] * q4;
            }
        }
    }
}

/* quantize_row_q8_K (main.c:247-340): per block, the FIRST element with the
 * largest |x| gives maxv; iscale = -127/maxv; q = min(rint(iscale*x), 127);
 * bsums over 16; d = 1/iscale; an all-zero block gives all zeros. */
void or_quantize_row_q8_K(const float *x, or_q8k *y, int k) {
    for (int b = 0; b < k / QK; b++, x += QK) {
        float amax = 0.0f, maxv = 0.0f;
        for (int j = 0; j < QK; j++) {
            float a = fabsf(x[j]);
            if (a > amax) { amax = a; maxv = x[j]; }
        }
        if (amax == 0.0f) { memset(&y[b], 0, sizeof(or_q8k)); continue; }
        const float iscale = -127.0f / maxv;
        for (int j = 0; j < QK; j++) {
            long v = lrintf(iscale * x[j]);
            if (v > 127) v = 127;
            if (v < -128) v = -128;
            y[b].qs[j] = (int8_t)v;
        }
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int i = 0; i < 16; i++) s += y[b].qs[16 * g + i];
            y[b].bsums[g] = (int16_t)s;
        }
        y[b].d = 1.0f / iscale;
    }
}

/* Integer partial sums of one Q4_K/Q5_K super-block against Q8_K
 * (main.c:373-399 / 437-465): sumi_s = sum_j sc[j] * sum_{32} q*q8,
 * sumi_m = sum_{g<16} bsums[g] * min[g/2]. */
void or_qk_block_sums(const void *blk, int type, const or_q8k *y, int32_t *sumi_s, int32_t *sumi_m) {
    const uint8_t *scales, *qs, *qh = NULL;
    if (type == G4_Q4_K) { const or_q4k *b = (const or_q4k *)blk; scales = b->scales; qs = b->qs; }
    else { const or_q5k *b = (const or_q5k *)blk; scales = b->scales; qs = b->qs; qh = b->qh; }
    int32_t ss = 0, sm = 0;
    for (int j = 0; j < 8; j++) {
        int sc, mn;
        or_scale_min(j, scales, &sc, &mn);
        int c = j / 2, hi = j & 1, dot = 0;
        for (int l = 0; l < 32; l++) {
            int q = hi ? qs[32 * c + l] >> 4 : qs[32 * c + l] & 15;
            if (qh && ((qh[l] >> j) & 1)) q += 16;
            dot += q * y->qs[32 * j + l];
        }
        ss += sc * dot;
        sm += mn * (y->bsums[2 * j] + y->bsums[2 * j + 1]);
    }
    *sumi_s = ss; *sumi_m = sm;
}

/* vec_dot_q4_K_q8_K / q5 in the generic order (main.c:347-473): eight
 * per-lane int32 accumulators, lane l collecting every element with index
 * % 8 == l scaled by its sub-block scale, then sums[l] += d*lane and
 * sumf -= dmin*sumi_m per block, lanes added last. */
float or_vec_dot_qk(int n, const void *row, int type, const or_q8k *y) {
    const size_t bs = or_block_bytes(type);
    float sums[8] = {0}, sumf = 0.0f;
    for (int b = 0; b < n / QK; b++) {
        const uint8_t *blk = (const uint8_t *)row + (size_t)b * bs;
        const uint8_t *scales, *qs, *qh = NULL;
        uint16_t hd, hm;
        if (type == G4_Q4_K) { const or_q4k *p = (const or_q4k *)blk; scales = p->scales; qs = p->qs; hd = p->d; hm = p->dmin; }
        else { const or_q5k *p = (const or_q5k *)blk; scales = p->scales; qs = p->qs; qh = p->qh; hd = p->d; hm = p->dmin; }
        int32_t lane[8] = {0}, sumi_m = 0;
        for (int j = 0; j < 8; j++) {
            int sc, mn;
            or_scale_min(j, scales, &sc, &mn);
            sumi_m += mn * (y[b].bsums[2 * j] + y[b].bsums[2 * j + 1]);
            int c = j / 2, hi = j & 1;
            for (int l = 0; l < 32; l++) {
                int q = hi ? qs[32 * c + l] >> 4 : qs[32 * c + l] & 15;
                if (qh && ((qh[l] >> j) & 1)) q += 16;
                lane[l % 8] += sc * (q * y[b].qs[32 * j + l]);
            }
        }
        const float d = or_f16(hd) * y[b].d;
        for (int l = 0; l < 8; l++) sums[l] += d * (float)lane[l];
        const float dmin = or_f16(hm) * y[b].d;
        sumf -= dmin * (float)sumi_m;
    }
    for (int l = 0; l < 8; l++) sumf += sums[l];
    return sumf;
}

static size_t or_row_bytes(int type, int n) {
    if (type == G4_F32) return (size_t)n * 4;
    if (type == G4_F16 || type == G4_BF16) return (size_t)n * 2;
    return (size_t)(n / QK) * or_block_bytes(type);
}

/* One row of the fp32 GEMVs: mm_f16 / mm_bf16 (main.c:1519-1537, x[j]*w[j]
 * summed in order), mm_quant_rows (1539-1556: dequantize a block, then
 * val += x*w in order), mm_f32 row (OpenBLAS sgemv; restated as an in-order
 * sum, which matches OpenBLAS only to rounding). */
float or_row_dot_f32(const float *x, const void *row, int n, int type) {
    float val = 0.0f;
    if (type == G4_F32) { const float *w = (const float *)row; for (int j = 0; j < n; j++) val += x[j] * w[j]; }
    else if (type == G4_F16) { const uint16_t *w = (const uint16_t *)row; for (int j = 0; j < n; j++) val += x[j] * or_f16(w[j]); }
    else if (type == G4_BF16) { const uint16_t *w = (const uint16_t *)row; for (int j = 0; j < n; j++) val += x[j] * or_bf16(w[j]); }
    else {
        float blk[QK];
        const size_t bs = or_block_bytes(type);
        for (int b = 0; b < n / QK; b++) {
            or_dequant_block((const uint8_t *)row + (size_t)b * bs, type, blk);
            for (int j = 0; j < QK; j++) val += x[b * QK + j] * blk[j];
        }
    }
    return val;
}

/* mm (main.c:1669-1694): Q4_K/Q5_K through Q8_K integer dots (quantizing x
 * into q8 unless q8_ready), Q6_K/F32/F16/BF16 through fp32 dots.  Returns 0,
 * or -1 for an unsupported type / n % 256 (where the reference exits). */
int or_mm(float *o, const float *x, const void *w, int n, int d, int type, or_q8k *q8, int q8_ready) {
    const size_t rb = or_row_bytes(type, n);
    if (type == G4_Q4_K || type == G4_Q5_K) {
        if (n % QK) return -1;
        if (!q8_ready) or_quantize_row_q8_K(x, q8, n);
        #pragma omp parallel for schedule(static)
        for (int i = 0; i < d; i++) o[i] = or_vec_dot_qk(n, (const uint8_t *)w + (size_t)i * rb, type, q8);
        return 0;
    }
    if (type != G4_Q6_K && type != G4_F32 && type != G4_F16 && type != G4_BF16) return -1;
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < d; i++) o[i] = or_row_dot_f32(x, (const uint8_t *)w + (size_t)i * rb, n, type);
    return 0;
}

/* First index of the maximum: sample_token with temp <= 0 (main.c:2045-2050)
 * and the merge rule of mm_argmax_row (1570-1667, lowest index among equals). */
int or_argmax_first(const float *v, int n) {
    int best = 0;
    for (int i = 1; i < n; i++) if (v[i] > v[best]) best = i;
    return best;
}

/* rmsnorm family (main.c:1451-1476). */
void or_rmsnorm(float *o, const float *x, const float *w, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    ss = 1.0f / sqrtf(ss / n + eps);
    for (int i = 0; i < n; i++) o[i] = x[i] * ss * w[i];
}
void or_rmsnorm_heads(float *v, const float *w, int nh, int hd, float eps) {
    for (int h = 0; h < nh; h++) {
        float *s = v + (size_t)h * hd, ss = 0.0f;
        for (int i = 0; i < hd; i++) ss += s[i] * s[i];
        ss = 1.0f / sqrtf(ss / hd + eps);
        for (int i = 0; i < hd; i++) s[i] *= w ? ss * w[i] : ss;
    }
}
/* tanh GELU (main.c:1490-1492). */
float or_gelu(float x) { return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * x * (1.0f + 0.044715f * x * x))); }

/* Neox RoPE (main.c:1725-1745): pairs (j, j + head_dim/2) for j < n_rot/2;
 * theta starts at pos and is multiplied by theta_scale once per pair. */
void or_rope_neox(float *vec, int n_heads, int hd, int n_rot, int pos, float base, float fscale,
                  const float *ff) {
    const float theta_scale = powf(base, -2.0f / (float)n_rot);
    for (int h = 0; h < n_heads; h++) {
        float *s = vec + (size_t)h * hd, theta = (float)pos;
        for (int j = 0; j < n_rot / 2; j++) {
            const float angle = fscale * theta / (ff ? ff[j] : 1.0f);
            const float c = cosf(angle), sn = sinf(angle);
            const float v0 = s[j], v1 = s[j + hd / 2];
            s[j] = v0 * c - v1 * sn;
            s[j + hd / 2] = v0 * sn + v1 * c;
            theta *= theta_scale;
        }
    }
}

/* Decode attention for one position (the per-head block of forward,
 * main.c:1924-1950, with softmax 1478-1488): scores over nwin cached rows
 * (row stride kv_stride floats), scale 1, max-subtracted expf softmax, then
 * the probability-weighted sum of V rows.  Summation in row order. */
void or_attention(float *out, const float *q, const float *k, const float *v, int nwin, int kv_stride,
                  int n_heads, int n_kv, int hd) {
    float *att = (float *)malloc(sizeof(float) * (nwin > 0 ? nwin : 1));
    const int group = n_heads / n_kv;
    for (int h = 0; h < n_heads; h++) {
        const float *qh = q + (size_t)h * hd;
        const int kvh = h / group;
        float *oh = out + (size_t)h * hd;
        if (nwin <= 0) { memset(oh, 0, sizeof(float) * hd); continue; }
        for (int t = 0; t < nwin; t++) {
            const float *kr = k + (size_t)t * kv_stride + (size_t)kvh * hd;
            float s = 0.0f;
            for (int i = 0; i < hd; i++) s += kr[i] * qh[i];
            att[t] = s;
        }
        float mx = att[0], sum = 0.0f;
        for (int t = 1; t < nwin; t++) if (att[t] > mx) mx = att[t];
        for (int t = 0; t < nwin; t++) { att[t] = expf(att[t] - mx); sum += att[t]; }
        for (int t = 0; t < nwin; t++) att[t] /= sum;
        for (int i = 0; i < hd; i++) oh[i] = 0.0f;
        for (int t = 0; t < nwin; t++) {
            const float *vr = v + (size_t)t * kv_stride + (size_t)kvh * hd;
            for (int i = 0; i < hd; i++) oh[i] += att[t] * vr[i];
        }
    }
    free(att);
}

/* logits_tied (main.c:1780-1796): tied-embedding GEMV then cap*tanh(l/cap). */
void or_logits_tied(float *logits, const float *x, const void *embd, int type, int dim, int vocab, float cap,
                    or_q8k *q8) {
    or_mm(logits, x, embd, dim, vocab, type, q8, 0);
    if (cap > 0.0f) {
        const float inv = 1.0f / cap;
        for (int i = 0; i < vocab; i++) logits[i] = cap * tanhf(logits[i] * inv);
    }
}

/* ------------------------------------------------------------------ */
/* Whole decode step: forward (main.c:1838-2029) with build_ple (1747-1778)
 * and emb_lookup (1696-1723), on a model given as a g4_model_desc.          */
/* ------------------------------------------------------------------ */

#define OR_N_LAYER_KV 24 /* main.c:77 */

typedef struct {
    g4_model_desc m;
    int max_seq, kv_dim_max;
    float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *qo, *ple, *ple_ctx, *gate, *logits, *kc, *vc;
    or_q8k *q8;
} or_model;

static int or_is_swa(const g4_model_desc *m, int l) { /* main.c:716-721 */
    if (m->swa_layers) return m->swa_layers[l] != 0;
    if (m->swa_pattern <= 0) return 0;
    return (l % m->swa_pattern) < (m->swa_pattern - 1);
}

void *or_model_create(const g4_model_desc *m, int max_seq) {
    or_model *s = (or_model *)calloc(1, sizeof(or_model));
    s->m = *m; s->max_seq = max_seq; s->kv_dim_max = 1024; /* MAX_KV_DIM, main.c:74 */
    const int L = m->n_layers, pd = m->ple_dim;
    s->x = calloc(m->dim, 4); s->xb2 = calloc(m->dim, 4);
    s->hb = calloc(m->hidden_dim, 4); s->hb2 = calloc(m->hidden_dim, 4);
    s->q = calloc(4096, 4); s->k = calloc(1024, 4); s->v = calloc(1024, 4); s->qo = calloc(4096, 4);
    s->ple = calloc((size_t)pd * L, 4); s->ple_ctx = calloc((size_t)pd * L, 4); s->gate = calloc(pd, 4);
    s->logits = calloc(m->vocab_size, 4);
    s->kc = calloc((size_t)OR_N_LAYER_KV * max_seq * 1024, 4);
    s->vc = calloc((size_t)OR_N_LAYER_KV * max_seq * 1024, 4);
    int qb = m->hidden_dim > 4096 ? m->hidden_dim : 4096;
    s->q8 = calloc(qb / QK + 1, sizeof(or_q8k));
    return s;
}

void or_model_free(void *p) {
    or_model *s = (or_model *)p;
    if (!s) return;
    free(s->x); free(s->xb2); free(s->hb); free(s->hb2); free(s->q); free(s->k); free(s->v); free(s->qo);
    free(s->ple); free(s->ple_ctx); free(s->gate); free(s->logits); free(s->kc); free(s->vc); free(s->q8);
    free(s);
}

const float *or_model_logits(void *p) { return ((or_model *)p)->logits; }
const float *or_model_x(void *p) { return ((or_model *)p)->x; }
const float *or_model_kc(void *p, int l, int pos) { or_model *s = p; return s->kc + ((size_t)l * s->max_seq + pos) * 1024; }
const float *or_model_vc(void *p, int l, int pos) { or_model *s = p; return s->vc + ((size_t)l * s->max_seq + pos) * 1024; }

/* Row `id` of an embedding table as floats (emb_lookup, main.c:1696-1723). */
static void or_emb_row(float *o, const void *w, int type, int id, int dim) {
    const uint8_t *row = (const uint8_t *)w + (size_t)id * or_row_bytes(type, dim);
    if (type == G4_F32) memcpy(o, row, (size_t)dim * 4);
    else if (type == G4_F16) for (int i = 0; i < dim; i++) o[i] = or_f16(((const uint16_t *)row)[i]);
    else if (type == G4_BF16) for (int i = 0; i < dim; i++) o[i] = or_bf16(((const uint16_t *)row)[i]);
    else for (int b = 0; b < dim / QK; b++) or_dequant_block(row + (size_t)b * or_block_bytes(type), type, o + b * QK);
}

/* Returns the argmax token for lm_mode != 0 (first max of the softcapped
 * logits, main.c:2045-2050), 0 for lm_mode 0. */
int or_forward(void *p, int token, int pos, int lm_mode) {
    or_model *s = (or_model *)p;
    const g4_model_desc *m = &s->m;
    const int dim = m->dim, hid = m->hidden_dim, nh = m->n_heads, nkv = m->n_kv_heads, pd = m->ple_dim;
    const int L = m->n_layers, group = nh / nkv;
    const float eps = m->norm_eps;

    or_emb_row(s->x, m->embd, m->embd_t, token, dim);                    /* 1849-1854 */
    { const float sc = sqrtf((float)dim); for (int i = 0; i < dim; i++) s->x[i] *= sc; }

    {   /* build_ple (1747-1778) */
        const int rd = pd * L;
        float *row = (float *)malloc((size_t)rd * 4);
        or_emb_row(row, m->ple_tok, m->ple_tok_t, token, rd);
        const float st = sqrtf((float)pd);
        for (int i = 0; i < rd; i++) row[i] *= st;
        or_mm(s->ple_ctx, s->x, m->ple_proj, dim, rd, m->ple_proj_t, s->q8, 0);
        const float sc = 1.0f / sqrtf((float)dim);
        for (int i = 0; i < rd; i++) s->ple_ctx[i] *= sc;
        for (int l = 0; l < L; l++) or_rmsnorm(s->ple_ctx + (size_t)l * pd, s->ple_ctx + (size_t)l * pd, m->ple_proj_norm, pd, eps);
        const float mix = 1.0f / sqrtf(2.0f);
        for (int i = 0; i < rd; i++) s->ple[i] = (row[i] + s->ple_ctx[i]) * mix;
        free(row);
    }

    float *xb = (float *)malloc((size_t)dim * 4);
    float *att_k = NULL, *att_v = NULL;
    for (int l = 0; l < L; l++) {
        const int swa = or_is_swa(m, l);
        const int hd = swa ? m->head_dim_swa : m->head_dim_full;
        const int nrot = swa ? m->n_rot_swa : m->n_rot_full;
        const int qd = nh * hd, kvd = nkv * hd;
        const float base = swa ? m->rope_theta_swa : m->rope_theta;
        const float *ff = swa ? NULL : m->rope_freqs;
        memcpy(xb, s->x, (size_t)dim * 4);                               /* x_before */

        or_rmsnorm(s->xb2, s->x, m->attn_norm[l], dim, eps);            /* 1878-1886 */
        const int q8a = m->wq_t[l] == G4_Q4_K || m->wq_t[l] == G4_Q5_K;
        if (q8a) or_quantize_row_q8_K(s->xb2, s->q8, dim);
        or_mm(s->q, s->xb2, m->wq[l], dim, qd, m->wq_t[l], s->q8, q8a);
        or_rmsnorm_heads(s->q, m->q_norm[l], nh, hd, eps);
        or_rope_neox(s->q, nh, hd, nrot, pos, base, 1.0f, ff);

        int src = l;                                                     /* kv_source_for_layer 743-746 */
        if (l < OR_N_LAYER_KV) {                                         /* 1889-1907 */
            or_mm(s->k, s->xb2, m->wk[l], dim, kvd, m->wk_t[l], s->q8, q8a);
            or_mm(s->v, s->xb2, m->wv[l], dim, kvd, m->wv_t[l], s->q8, q8a);
            or_rmsnorm_heads(s->k, m->k_norm[l], nkv, hd, eps);
            or_rmsnorm_heads(s->v, NULL, nkv, hd, eps);
            or_rope_neox(s->k, nkv, hd, nrot, pos, base, 1.0f, ff);
            memcpy(s->kc + ((size_t)l * s->max_seq + pos) * 1024, s->k, (size_t)kvd * 4);
            memcpy(s->vc + ((size_t)l * s->max_seq + pos) * 1024, s->v, (size_t)kvd * 4);
        } else {
            src = swa ? 22 : 23;
        }
        const int src_hd = or_is_swa(m, src) ? m->head_dim_swa : m->head_dim_full;
        int t0 = 0;                                                      /* 1909-1915 */
        if (swa) { t0 = pos + 1 - m->sliding_window; if (t0 < 0) t0 = 0; }
        const int nwin = pos + 1 - t0;
        (void)att_k; (void)att_v;
        {
            const float *kb = s->kc + ((size_t)src * s->max_seq + t0) * 1024;
            const float *vb = s->vc + ((size_t)src * s->max_seq + t0) * 1024;
            /* per q head, kv head h / group, head slice at kvh * src_hd (1924-1950) */
            float *att = (float *)malloc(sizeof(float) * (nwin > 0 ? nwin : 1));
            for (int h = 0; h < nh; h++) {
                const float *qh = s->q + (size_t)h * hd;
                float *oh = s->qo + (size_t)h * hd;
                const int kvh = h / group;
                if (nwin <= 0) { memset(oh, 0, (size_t)hd * 4); continue; }
                for (int t = 0; t < nwin; t++) {
                    const float *kr = kb + (size_t)t * 1024 + (size_t)kvh * src_hd;
                    float sc = 0.0f;
                    for (int i = 0; i < hd; i++) sc += kr[i] * qh[i];
                    att[t] = sc;
                }
                float mx = att[0], sum = 0.0f;
                for (int t = 1; t < nwin; t++) if (att[t] > mx) mx = att[t];
                for (int t = 0; t < nwin; t++) { att[t] = expf(att[t] - mx); sum += att[t]; }
                for (int t = 0; t < nwin; t++) att[t] /= sum;
                for (int i = 0; i < hd; i++) oh[i] = 0.0f;
                for (int t = 0; t < nwin; t++) {
                    const float *vr = vb + (size_t)t * 1024 + (size_t)kvh * src_hd;
                    for (int i = 0; i < hd; i++) oh[i] += att[t] * vr[i];
                }
            }
            free(att);
        }

        or_mm(s->xb2, s->qo, m->wo[l], qd, dim, m->wo_t[l], s->q8, 0);  /* 1959-1962 */
        or_rmsnorm(s->xb2, s->xb2, m->post_attn_norm[l], dim, eps);
        for (int i = 0; i < dim; i++) s->x[i] = xb[i] + s->xb2[i];
        memcpy(xb, s->x, (size_t)dim * 4);

        or_rmsnorm(s->xb2, s->x, m->ffn_norm[l], dim, eps);             /* 1973-1984 */
        const int q8f = m->gate_t[l] == G4_Q4_K || m->gate_t[l] == G4_Q5_K;
        if (q8f) or_quantize_row_q8_K(s->xb2, s->q8, dim);
        or_mm(s->hb, s->xb2, m->gate[l], dim, hid, m->gate_t[l], s->q8, q8f);
        or_mm(s->hb2, s->xb2, m->up[l], dim, hid, m->up_t[l], s->q8, q8f);
        for (int i = 0; i < hid; i++) s->hb[i] = or_gelu(s->hb[i]) * s->hb2[i];
        or_mm(s->xb2, s->hb, m->down[l], hid, dim, m->down_t[l], s->q8, 0);
        or_rmsnorm(s->xb2, s->xb2, m->post_ffw_norm[l], dim, eps);
        for (int i = 0; i < dim; i++) s->x[i] = xb[i] + s->xb2[i];
        memcpy(xb, s->x, (size_t)dim * 4);

        or_mm(s->gate, s->x, m->inp_gate[l], dim, pd, m->inp_gate_t[l], s->q8, 0); /* 1986-1997 */
        for (int i = 0; i < pd; i++) s->gate[i] = or_gelu(s->gate[i]);
        for (int i = 0; i < pd; i++) s->gate[i] *= s->ple[(size_t)l * pd + i];
        or_mm(s->xb2, s->gate, m->proj[l], pd, dim, m->proj_t[l], s->q8, 0);
        or_rmsnorm(s->xb2, s->xb2, m->post_norm[l], dim, eps);
        for (int i = 0; i < dim; i++) s->x[i] = xb[i] + s->xb2[i];
        if (m->out_scale && m->out_scale[l]) {                           /* 1999-2003 */
            const float sc = m->out_scale[l][0];
            for (int i = 0; i < dim; i++) s->x[i] *= sc;
        }
    }
    free(xb);
    if (lm_mode == 0) return 0;
    or_rmsnorm(s->x, s->x, m->norm_out, dim, eps);                       /* 2021 */
    or_logits_tied(s->logits, s->x, m->embd, m->embd_t, dim, m->vocab_size, m->logit_softcapping, s->q8);
    return or_argmax_first(s->logits, m->vocab_size);
}

/* Greedy generation (generate, main.c:2335-2488, temp <= 0). */
int or_generate_greedy(void *p, const int *prompt, int n_prompt, int max_new, int eos, int *out) {
    or_model *s = (or_model *)p;
    int token = prompt[0], gen = 0;
    for (int pos = 0; pos < n_prompt + max_new - 1; pos++) {
        if (pos >= s->max_seq) break;
        const int lm = pos < n_prompt - 1 ? 0 : 1;
        const int am = or_forward(s, token, pos, lm);
        int next;
        if (pos < n_prompt - 1) next = prompt[pos + 1];
        else {
            next = am;
            if (next == eos) break;
            out[gen++] = next;
        }
        token = next;
    }
    return gen;
}
