/*
 * qwen3_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the almostrealism/common Qwen3 forward step, used as the
 * parity checker for the CUDA library and as the timed CPU baseline.  Nothing in
 * the product path links or calls this file; only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference legs load it.
 *
 * Compiled twice: with -DORACLE_REAL=double (the reference's default JNI precision,
 * base/hardware/src/main/java/org/almostrealism/hardware/Hardware.java:684) and with
 * -DORACLE_REAL=float (AR_HARDWARE_PRECISION=FP32).
 *
 * Semantics follow the reference exactly (all paths relative to the reference root):
 *   rmsnorm           domain/graph/src/main/java/org/almostrealism/layers/NormalizationLayerFeatures.java:587-603
 *   dense (y = W x)   domain/graph/src/main/java/org/almostrealism/layers/LayerFeatures.java:785-830
 *   attention block   engine/ml/src/main/java/org/almostrealism/ml/AttentionFeatures.java:785-929
 *   QK-norm           AttentionFeatures.java:840-845, 886-891 (norm over the WHOLE q / k vector)
 *   split-half RoPE   AttentionFeatures.java:195-237, RotationFeatures.java:124-170
 *   freqCis           RotationFeatures.java:189-208
 *   GQA expand        AttentionFeatures.java:372-391 (expanded at cache-write time)
 *   scores / PV       AttentionFeatures.java:531-616
 *   causal mask       AttentionFeatures.java:906-917 (-10000 for t > position)
 *   softmax           domain/graph/src/main/java/org/almostrealism/layers/ActivationFeatures.java:126-143
 *   silu              ActivationFeatures.java:263-265
 *   feed-forward      engine/ml/src/main/java/org/almostrealism/ml/FeedForwardFeatures.java:140-157
 *   transformer/accum AttentionFeatures.java:1688-1708, domain/graph/.../model/SequentialBlock.java:413-429
 *   model assembly    engine/ml/src/main/java/org/almostrealism/ml/qwen3/Qwen3.java:334-415
 *   indexOfMax        compute/algebra/src/main/java/org/almostrealism/collect/AggregationFeatures.java:111-121
 *
 * Extensions beyond the reference (clearly flagged by config fields):
 *   - q_dim = heads*head_dim may differ from dim (Qwen3-0.6B / 32B geometry); the
 *     reference requires heads*headSize == dim (TransformerConfig.java:104).
 *   - qk_norm_mode 2 = per-head QK-norm (HuggingFace Qwen3).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#ifndef ORACLE_REAL
#define ORACLE_REAL double
#endif
typedef ORACLE_REAL real;

#define CAT2(a, b) a##b
#define CAT(a, b) CAT2(a, b)
#ifdef ORACLE_F32
#define SFX _f32
#define RSQRT(x) (1.0f / sqrtf(x))
#define EXP(x) expf(x)
#define LOG(x) logf(x)
#define SQRT(x) sqrtf(x)
#else
#define SFX _f64
#define RSQRT(x) (1.0 / sqrt(x))
#define EXP(x) exp(x)
#define LOG(x) log(x)
#define SQRT(x) sqrt(x)
#endif
#define API(name) CAT(name, SFX)

typedef struct {
    int dim, hidden_dim, layers, heads, kv_heads, head_dim, vocab, seq_len;
    int shared_weights;   /* lm_head tied to embed_tokens (Qwen3.java:344-345) */
    int qk_norm_mode;     /* 0 none, 1 reference (whole vector), 2 per head */
    int has_qkv_bias;     /* Qwen2.5-style biases on q/k/v (Qwen3.java:370-373) */
    int share_layers;     /* CPU-baseline memory saver: every layer uses layer 0's weights */
    double rope_theta;
    double eps;
} oref_config;

typedef struct {
    real *rms_att, *rms_ffn, *wq, *wk, *wv, *wo, *bq, *bk, *bv, *qn, *kn, *w1, *w2, *w3;
    real *kcache, *vcache; /* (seq_len, heads, head_dim), GQA-expanded, zero-filled */
} oref_layer;

typedef struct {
    oref_config c;
    int q_dim, kv_dim;
    real *embed, *wcls, *rms_final, *freq; /* freq: (seq_len, head_dim/2, 2) */
    oref_layer *L;
    /* scratch */
    real *x, *xb, *q, *k, *v, *att, *o, *hb, *hb2, *logits;
} oref_model;

/* ---------------- component functions (also exported for KAT tests) ---------------- */

/* rmsnorm: out_i = w_i * x_i * (sum_j x_j^2 / n + eps)^-1/2  (NormalizationLayerFeatures.java:587-603) */
static void rmsnorm_(real *out, const real *x, const real *w, int n, real eps) {
    real ss = 0;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    ss = ss / (real)n + eps;
    real s = (real)1 / (real)SQRT(ss);
    for (int i = 0; i < n; i++) out[i] = w[i] * x[i] * s;
}

/* y = W x, W (out, in) row-major (LayerFeatures.dense / MatrixFeatures.matmul) */
static void matvec_(real *y, const real *W, const real *x, const real *bias, int out, int in) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < out; r++) {
        const real *w = W + (size_t)r * in;
        real acc = 0;
        for (int i = 0; i < in; i++) acc += w[i] * x[i];
        y[r] = acc + (bias ? bias[r] : (real)0);
    }
}

/* freqCis[pos, f, 0|1] = cos|sin(pos * exp(-2 f ln(theta) / d))  (RotationFeatures.java:189-208) */
void API(oref_rope_freqs)(double theta, int head_dim, int seq_len, double *out) {
    int fd = head_dim / 2;
    double lt = log(theta);
    for (int p = 0; p < seq_len; p++)
        for (int f = 0; f < fd; f++) {
            real inv = (real)EXP((real)f * (real)(-2.0 * lt / head_dim));
            real ang = (real)p * inv;
#ifdef ORACLE_F32
            out[((size_t)p * fd + f) * 2 + 0] = cosf(ang);
            out[((size_t)p * fd + f) * 2 + 1] = sinf(ang);
#else
            out[((size_t)p * fd + f) * 2 + 0] = cos(ang);
            out[((size_t)p * fd + f) * 2 + 1] = sin(ang);
#endif
        }
}

/* split-half RoPE on (heads, head_dim) in place: for f < d/2,
 * o[f] = x[f] c - x[f+d/2] s ; o[f+d/2] = x[f+d/2] c + x[f] s
 * (reshapeToSplitHalfRope -> ropeRotation -> reshapeFromSplitHalfRope,
 *  AttentionFeatures.java:195-237, RotationFeatures.java:143-166) */
static void rope_(real *x, int heads, int head_dim, const real *freq_row) {
    int fd = head_dim / 2;
    for (int h = 0; h < heads; h++) {
        real *v = x + (size_t)h * head_dim;
        for (int f = 0; f < fd; f++) {
            real c = freq_row[2 * f], s = freq_row[2 * f + 1];
            real x1 = v[f], x2 = v[f + fd];
            v[f] = x1 * c - x2 * s;
            v[f + fd] = x2 * c + x1 * s;
        }
    }
}

/* gqaExpand: out[h*d + i] = in[(h / (H/Hkv))*d + i]  (AttentionFeatures.java:372-391) */
void API(oref_gqa_expand)(const double *in, int kv_heads, int heads, int head_dim, double *out) {
    int g = heads / kv_heads;
    for (int h = 0; h < heads; h++)
        for (int i = 0; i < head_dim; i++) out[(size_t)h * head_dim + i] = in[(size_t)(h / g) * head_dim + i];
}

/* attentionKeysStandard: s[h, t] = sum_i q[h,i] K[t,h,i] / sqrt(d)  (AttentionFeatures.java:531-559) */
void API(oref_attention_keys)(const double *q, const double *K, int heads, int head_dim, int seq_len, double *s) {
    for (int h = 0; h < heads; h++)
        for (int t = 0; t < seq_len; t++) {
            real acc = 0;
            for (int i = 0; i < head_dim; i++)
                acc += (real)q[(size_t)h * head_dim + i] * (real)K[((size_t)t * heads + h) * head_dim + i];
            s[(size_t)h * seq_len + t] = acc / (real)SQRT((real)head_dim);
        }
}

/* attentionValuesStandard: o[h, i] = sum_t a[h,t] V[t,h,i]  (AttentionFeatures.java:572-616) */
void API(oref_attention_values)(const double *a, const double *V, int heads, int head_dim, int seq_len, double *o) {
    for (int h = 0; h < heads; h++)
        for (int i = 0; i < head_dim; i++) {
            real acc = 0;
            for (int t = 0; t < seq_len; t++)
                acc += (real)a[(size_t)h * seq_len + t] * (real)V[((size_t)t * heads + h) * head_dim + i];
            o[(size_t)h * head_dim + i] = acc;
        }
}

/* causal mask: s[h, t] += (t > pos) ? -10000 : 0  (AttentionFeatures.java:906-917) */
void API(oref_causal_mask)(double *s, int heads, int seq_len, int pos) {
    for (int h = 0; h < heads; h++)
        for (int t = 0; t < seq_len; t++) s[(size_t)h * seq_len + t] = (real)s[(size_t)h * seq_len + t] + (t > pos ? (real)-10000.0 : (real)0);
}

/* log-stable softmax along the last axis: exp(x - m - log(sum exp(x - m)))  (ActivationFeatures.java:136-142) */
static void softmax_(real *x, int n) {
    real m = x[0];
    for (int i = 1; i < n; i++) if (x[i] > m) m = x[i];
    real sum = 0;
    for (int i = 0; i < n; i++) sum += (real)EXP(x[i] - m);
    real ls = (real)LOG(sum);
    for (int i = 0; i < n; i++) x[i] = (real)EXP(x[i] - m - ls);
}
void API(oref_softmax)(double *x, int rows, int n) {
    real *t = (real *)malloc(sizeof(real) * n);
    for (int r = 0; r < rows; r++) {
        for (int i = 0; i < n; i++) t[i] = (real)x[(size_t)r * n + i];
        softmax_(t, n);
        for (int i = 0; i < n; i++) x[(size_t)r * n + i] = t[i];
    }
    free(t);
}

void API(oref_rmsnorm)(const double *x, const double *w, int n, double eps, double *out) {
    real *a = (real *)malloc(sizeof(real) * n * 3);
    for (int i = 0; i < n; i++) { a[i] = (real)x[i]; a[n + i] = (real)w[i]; }
    rmsnorm_(a + 2 * n, a, a + n, n, (real)eps);
    for (int i = 0; i < n; i++) out[i] = a[2 * n + i];
    free(a);
}

/* indexOfMax: the first index holding the maximum (strict greaterThan, AggregationFeatures.java:111-121) */
int API(oref_argmax)(const float *v, int n) {
    int best = 0;
    for (int i = 1; i < n; i++) if (v[i] > v[best]) best = i;
    return best;
}

/* ---------------- model ---------------- */

static real *zalloc(size_t n) {
    real *p = (real *)calloc(n ? n : 1, sizeof(real));
    if (!p) { fprintf(stderr, "oracle: out of memory (%zu elements)\n", n); abort(); }
    return p;
}

void *API(oref_create)(const oref_config *c) {
    oref_model *m = (oref_model *)calloc(1, sizeof(oref_model));
    m->c = *c;
    m->q_dim = c->heads * c->head_dim;
    m->kv_dim = c->kv_heads * c->head_dim;
    int D = c->dim, Q = m->q_dim, KV = m->kv_dim, F = c->hidden_dim;
    m->L = (oref_layer *)calloc(c->layers, sizeof(oref_layer));
    for (int l = 0; l < c->layers; l++) {
        oref_layer *L = &m->L[l];
        if (c->share_layers && l > 0) {
            *L = m->L[0];
            L->kcache = zalloc((size_t)c->seq_len * Q);
            L->vcache = zalloc((size_t)c->seq_len * Q);
            continue;
        }
        L->rms_att = zalloc(D); L->rms_ffn = zalloc(D);
        L->wq = zalloc((size_t)Q * D); L->wk = zalloc((size_t)KV * D); L->wv = zalloc((size_t)KV * D);
        L->wo = zalloc((size_t)D * Q);
        L->qn = zalloc(Q); L->kn = zalloc(KV);
        if (c->has_qkv_bias) { L->bq = zalloc(Q); L->bk = zalloc(KV); L->bv = zalloc(KV); }
        L->w1 = zalloc((size_t)F * D); L->w3 = zalloc((size_t)F * D); L->w2 = zalloc((size_t)D * F);
        L->kcache = zalloc((size_t)c->seq_len * Q);
        L->vcache = zalloc((size_t)c->seq_len * Q);
    }
    m->embed = zalloc((size_t)c->vocab * D);
    m->wcls = c->shared_weights ? m->embed : zalloc((size_t)c->vocab * D);
    m->rms_final = zalloc(D);
    m->freq = zalloc((size_t)c->seq_len * c->head_dim);
    {
        double *f = (double *)malloc(sizeof(double) * (size_t)c->seq_len * c->head_dim);
        API(oref_rope_freqs)(c->rope_theta, c->head_dim, c->seq_len, f);
        for (size_t i = 0; i < (size_t)c->seq_len * c->head_dim; i++) m->freq[i] = (real)f[i];
        free(f);
    }
    int mx = D > Q ? D : Q;
    m->x = zalloc(D); m->xb = zalloc(mx); m->q = zalloc(Q); m->k = zalloc(KV); m->v = zalloc(KV);
    m->att = zalloc((size_t)c->heads * c->seq_len); m->o = zalloc(Q);
    m->hb = zalloc(F); m->hb2 = zalloc(F); m->logits = zalloc(c->vocab);
    return m;
}

void API(oref_destroy)(void *mp) {
    oref_model *m = (oref_model *)mp;
    if (!m) return;
    for (int l = 0; l < m->c.layers; l++) {
        oref_layer *L = &m->L[l];
        if (m->c.share_layers && l > 0) { free(L->kcache); free(L->vcache); continue; }
        free(L->rms_att); free(L->rms_ffn); free(L->wq); free(L->wk); free(L->wv); free(L->wo);
        free(L->qn); free(L->kn); free(L->bq); free(L->bk); free(L->bv);
        free(L->w1); free(L->w2); free(L->w3); free(L->kcache); free(L->vcache);
    }
    free(m->L);
    if (m->wcls != m->embed) free(m->wcls);
    free(m->embed); free(m->rms_final); free(m->freq);
    free(m->x); free(m->xb); free(m->q); free(m->k); free(m->v); free(m->att); free(m->o);
    free(m->hb); free(m->hb2); free(m->logits);
    free(m);
}

/* Resolve an HF state-dict key (Qwen3.java:361-382) to a buffer and its element count. */
static real *lookup(oref_model *m, const char *key, size_t *n) {
    const oref_config *c = &m->c;
    int D = c->dim, Q = m->q_dim, KV = m->kv_dim, F = c->hidden_dim, l;
    char rest[128];
    if (!strcmp(key, "model.embed_tokens.weight")) { *n = (size_t)c->vocab * D; return m->embed; }
    if (!strcmp(key, "lm_head.weight")) { *n = (size_t)c->vocab * D; return c->shared_weights ? NULL : m->wcls; }
    if (!strcmp(key, "model.norm.weight")) { *n = D; return m->rms_final; }
    /* an explicit RoPE table (seq_len, head_dim/2, 2), as Llama2 checkpoints carry (Llama2Weights.java:108-110) */
    if (!strcmp(key, "rope.freq_cis")) { *n = (size_t)c->seq_len * c->head_dim; return m->freq; }
    if (sscanf(key, "model.layers.%d.%127s", &l, rest) != 2 || l < 0 || l >= c->layers) return NULL;
    if (c->share_layers && l > 0) return NULL;
    oref_layer *L = &m->L[l];
    if (!strcmp(rest, "input_layernorm.weight")) { *n = D; return L->rms_att; }
    if (!strcmp(rest, "post_attention_layernorm.weight")) { *n = D; return L->rms_ffn; }
    if (!strcmp(rest, "self_attn.q_proj.weight")) { *n = (size_t)Q * D; return L->wq; }
    if (!strcmp(rest, "self_attn.k_proj.weight")) { *n = (size_t)KV * D; return L->wk; }
    if (!strcmp(rest, "self_attn.v_proj.weight")) { *n = (size_t)KV * D; return L->wv; }
    if (!strcmp(rest, "self_attn.o_proj.weight")) { *n = (size_t)D * Q; return L->wo; }
    if (!strcmp(rest, "self_attn.q_proj.bias")) { *n = Q; return L->bq; }
    if (!strcmp(rest, "self_attn.k_proj.bias")) { *n = KV; return L->bk; }
    if (!strcmp(rest, "self_attn.v_proj.bias")) { *n = KV; return L->bv; }
    if (!strcmp(rest, "self_attn.q_norm.weight")) { *n = Q; return L->qn; }
    if (!strcmp(rest, "self_attn.k_norm.weight")) { *n = KV; return L->kn; }
    if (!strcmp(rest, "mlp.gate_proj.weight")) { *n = (size_t)F * D; return L->w1; }
    if (!strcmp(rest, "mlp.up_proj.weight")) { *n = (size_t)F * D; return L->w3; }
    if (!strcmp(rest, "mlp.down_proj.weight")) { *n = (size_t)D * F; return L->w2; }
    return NULL;
}

/* Copy one fp32 host tensor in.  Returns 0 on success, -1 unknown key, -2 size mismatch. */
int API(oref_set)(void *mp, const char *key, const float *data, long long n) {
    oref_model *m = (oref_model *)mp;
    size_t want = 0;
    real *dst = lookup(m, key, &want);
    if (!dst) return -1;
    if ((size_t)n != want) return -2;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < n; i++) dst[i] = (real)data[i];
    return 0;
}

/* Counter-based synthetic generator shared bit-for-bit with the CUDA library:
 * splitmix64 of (seed, tensor id, index) -> Irwin-Hall sum of four 16-bit uniforms,
 * scaled to the requested standard deviation.  Integer arithmetic + one fp32 multiply,
 * so host and device produce identical values. */
static uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
float API(oref_synth_value)(uint64_t seed, uint32_t tensor_id, uint64_t idx, float scale) {
    uint64_t h = splitmix64(seed ^ ((uint64_t)tensor_id << 40) ^ splitmix64(idx));
    int s = (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) + (int)(h >> 48) - 2 * 65535;
    return (float)s * scale;
}

void API(oref_reset)(void *mp) {
    oref_model *m = (oref_model *)mp;
    size_t n = (size_t)m->c.seq_len * m->q_dim;
    for (int l = 0; l < m->c.layers; l++) {
        memset(m->L[l].kcache, 0, n * sizeof(real));
        memset(m->L[l].vcache, 0, n * sizeof(real));
    }
}

/* One transformer layer at position `pos` on m->x (AttentionFeatures.transformer, :1688-1708). */
static void layer_(oref_model *m, int l, int pos) {
    const oref_config *c = &m->c;
    int D = c->dim, H = c->heads, Hkv = c->kv_heads, d = c->head_dim, S = c->seq_len;
    int Q = m->q_dim, KV = m->kv_dim, F = c->hidden_dim, grp = H / Hkv;
    real eps = (real)c->eps;
    const real *fr = m->freq + (size_t)pos * d;
    real *x = m->x;
    oref_layer *L = &m->L[l];
    /* attention: rmsnorm -> q/k/v dense -> qk-norm -> rope -> cache write -> scores -> mask -> softmax -> PV -> wo */
    rmsnorm_(m->xb, x, L->rms_att, D, eps);
    matvec_(m->q, L->wq, m->xb, L->bq, Q, D);
    matvec_(m->k, L->wk, m->xb, L->bk, KV, D);
    matvec_(m->v, L->wv, m->xb, L->bv, KV, D);
    if (c->qk_norm_mode == 1) {
        rmsnorm_(m->q, m->q, L->qn, Q, (real)1e-6);
        rmsnorm_(m->k, m->k, L->kn, KV, (real)1e-6);
    } else if (c->qk_norm_mode == 2) {
        for (int h = 0; h < H; h++) rmsnorm_(m->q + h * d, m->q + h * d, L->qn + h * d, d, (real)1e-6);
        for (int h = 0; h < Hkv; h++) rmsnorm_(m->k + h * d, m->k + h * d, L->kn + h * d, d, (real)1e-6);
    }
    rope_(m->q, H, d, fr);
    rope_(m->k, Hkv, d, fr);
    for (int h = 0; h < H; h++)
        for (int i = 0; i < d; i++) {
            L->kcache[((size_t)pos * H + h) * d + i] = m->k[(h / grp) * d + i];
            L->vcache[((size_t)pos * H + h) * d + i] = m->v[(h / grp) * d + i];
        }
    real isd = (real)SQRT((real)d);
#pragma omp parallel for schedule(static)
    for (int h = 0; h < H; h++) {
        real *a = m->att + (size_t)h * S;
        const real *qh = m->q + (size_t)h * d;
        for (int t = 0; t < S; t++) {
            const real *kt = L->kcache + ((size_t)t * H + h) * d;
            real acc = 0;
            for (int i = 0; i < d; i++) acc += qh[i] * kt[i];
            a[t] = acc / isd + (t > pos ? (real)-10000.0 : (real)0);
        }
        softmax_(a, S);
        real *oh = m->o + (size_t)h * d;
        for (int i = 0; i < d; i++) oh[i] = 0;
        for (int t = 0; t < S; t++) {
            const real *vt = L->vcache + ((size_t)t * H + h) * d;
            real p = a[t];
            for (int i = 0; i < d; i++) oh[i] += p * vt[i];
        }
    }
    matvec_(m->xb, L->wo, m->o, NULL, D, Q);
    for (int i = 0; i < D; i++) x[i] += m->xb[i];
    /* feed-forward: rmsnorm -> w3 b * silu(w1 b) -> w2, accumulated */
    rmsnorm_(m->xb, x, L->rms_ffn, D, eps);
    matvec_(m->hb, L->w1, m->xb, NULL, F, D);
    matvec_(m->hb2, L->w3, m->xb, NULL, F, D);
    for (int i = 0; i < F; i++) {
        real g = m->hb[i];
        real sg = (real)1 / ((real)1 + (real)EXP(-g));
        m->hb[i] = m->hb2[i] * (g * sg);
    }
    matvec_(m->xb, L->w2, m->hb, NULL, D, F);
    for (int i = 0; i < D; i++) x[i] += m->xb[i];
}

/* final rmsnorm + lm_head rows [r0, r1) (Qwen3.java:402-405) */
static void head_(oref_model *m, int r0, int r1, float *logits_out) {
    const oref_config *c = &m->c;
    rmsnorm_(m->xb, m->x, m->rms_final, c->dim, (real)c->eps);
    matvec_(m->logits + r0, m->wcls + (size_t)r0 * c->dim, m->xb, NULL, r1 - r0, c->dim);
    if (logits_out)
        for (int i = r0; i < r1; i++) logits_out[i] = (float)m->logits[i];
}

/* One compiled-model forward (CompiledModel.forward, CompiledModel.java:189-198):
 * x_in (dim) at `pos` -> logits (vocab), following the semantics above. */
static void forward_(oref_model *m, int pos, float *logits_out) {
    for (int l = 0; l < m->c.layers; l++) layer_(m, l, pos);
    head_(m, 0, m->c.vocab, logits_out);
}

/* CPU-baseline sample: one layer of the step plus a slice of the lm_head rows, on the
 * current hidden state.  `layers` such slices with lm rows split evenly = one token. */
int API(oref_bench_slice)(void *mp, int layer, int pos, int lm_r0, int lm_r1) {
    oref_model *m = (oref_model *)mp;
    if (layer < 0 || layer >= m->c.layers || pos < 0 || pos >= m->c.seq_len || lm_r0 < 0 || lm_r1 > m->c.vocab ||
        lm_r0 > lm_r1)
        return -1;
    layer_(m, layer, pos);
    head_(m, lm_r0, lm_r1, NULL);
    return 0;
}

/* token path: in.setFrom(embed.range((1,dim), t*dim)) (AutoregressiveModel.java:430, Qwen3.java:414) */
int API(oref_forward_token)(void *mp, int token, int pos, float *logits_out) {
    oref_model *m = (oref_model *)mp;
    if (token < 0 || token >= m->c.vocab || pos < 0 || pos >= m->c.seq_len) return -1;
    for (int i = 0; i < m->c.dim; i++) m->x[i] = m->embed[(size_t)token * m->c.dim + i];
    forward_(m, pos, logits_out);
    return 0;
}

int API(oref_forward_hidden)(void *mp, const float *x_in, int pos, float *logits_out) {
    oref_model *m = (oref_model *)mp;
    if (pos < 0 || pos >= m->c.seq_len) return -1;
    for (int i = 0; i < m->c.dim; i++) m->x[i] = (real)x_in[i];
    forward_(m, pos, logits_out);
    return 0;
}

/* AutoregressiveModel.next() loop (AutoregressiveModel.java:295-308) with greedy sampling:
 * prompt tokens fed one per step; afterwards the token is argmax of the previous logits.
 * tokens_out[i] = the token fed at step i (what next() returns). */
int API(oref_generate)(void *mp, const int *prompt, int prompt_len, int steps, int *tokens_out, float *last_logits) {
    oref_model *m = (oref_model *)mp;
    float *lg = (float *)malloc(sizeof(float) * m->c.vocab);
    int cur = 0;
    for (int s = 0; s < steps; s++) {
        cur = s < prompt_len ? prompt[s] : API(oref_argmax)(lg, m->c.vocab);
        if (API(oref_forward_token)(mp, cur, s, lg)) { free(lg); return -1; }
        tokens_out[s] = cur;
    }
    if (last_logits) memcpy(last_logits, lg, sizeof(float) * m->c.vocab);
    free(lg);
    return 0;
}

/* host threads for the timed CPU baseline (a torchrun launch sets OMP_NUM_THREADS=1 in the environment) */
void API(oref_set_threads)(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int API(oref_num_threads)(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Fill every tensor from the synthetic generator with the CUDA library's tensor ids:
 * embed 0, lm_head 1, final norm 2, layer l kind k -> 16 + 16 l + k with kinds
 * rms_att 0, rms_ffn 1, wq 2, wk 3, wv 4, wo 5, bq 6, bk 7, bv 8, q_norm 9, k_norm 10,
 * gate 11, up 12, down 13.  Norm weights are 1; element index = row-major index in the
 * full (unsharded) tensor. */
static void synth_fill(real *dst, size_t n, uint64_t seed, uint32_t tid, float scale) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) dst[i] = (real)API(oref_synth_value)(seed, tid, i, scale);
}
static void ones(real *dst, size_t n) { for (size_t i = 0; i < n; i++) dst[i] = 1; }

void API(oref_init_synthetic)(void *mp, uint64_t seed, float stdv) {
    oref_model *m = (oref_model *)mp;
    const oref_config *c = &m->c;
    size_t D = c->dim, Q = m->q_dim, KV = m->kv_dim, F = c->hidden_dim;
    float scale = (float)(stdv / sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0));
    synth_fill(m->embed, (size_t)c->vocab * D, seed, 0, scale);
    if (!c->shared_weights) synth_fill(m->wcls, (size_t)c->vocab * D, seed, 1, scale);
    ones(m->rms_final, D);
    for (int l = 0; l < (c->share_layers ? 1 : c->layers); l++) {
        oref_layer *L = &m->L[l];
        uint32_t b = 16u + 16u * (uint32_t)l;
        ones(L->rms_att, D); ones(L->rms_ffn, D);
        synth_fill(L->wq, Q * D, seed, b + 2, scale);
        synth_fill(L->wk, KV * D, seed, b + 3, scale);
        synth_fill(L->wv, KV * D, seed, b + 4, scale);
        synth_fill(L->wo, D * Q, seed, b + 5, scale);
        if (c->has_qkv_bias) {
            synth_fill(L->bq, Q, seed, b + 6, scale);
            synth_fill(L->bk, KV, seed, b + 7, scale);
            synth_fill(L->bv, KV, seed, b + 8, scale);
        }
        ones(L->qn, Q); ones(L->kn, KV);
        synth_fill(L->w1, F * D, seed, b + 11, scale);
        synth_fill(L->w3, F * D, seed, b + 12, scale);
        synth_fill(L->w2, D * F, seed, b + 13, scale);
    }
}

/* Round every stored weight to bf16 (round-to-nearest-even): the values a bf16-weight
 * run of the CUDA library holds, so both sides compute on identical weights. */
static void bf16_round_buf(real *p, size_t n) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) {
        float f = (float)p[i];
        uint32_t u;
        memcpy(&u, &f, 4);
        if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
        memcpy(&f, &u, 4);
        p[i] = (real)f;
    }
}
void API(oref_round_weights_bf16)(void *mp) {
    oref_model *m = (oref_model *)mp;
    const oref_config *c = &m->c;
    size_t D = c->dim, Q = m->q_dim, KV = m->kv_dim, F = c->hidden_dim;
    bf16_round_buf(m->embed, (size_t)c->vocab * D);
    if (!c->shared_weights) bf16_round_buf(m->wcls, (size_t)c->vocab * D);
    for (int l = 0; l < (c->share_layers ? 1 : c->layers); l++) {
        oref_layer *L = &m->L[l];
        bf16_round_buf(L->wq, Q * D); bf16_round_buf(L->wk, KV * D); bf16_round_buf(L->wv, KV * D);
        bf16_round_buf(L->wo, D * Q); bf16_round_buf(L->w1, F * D); bf16_round_buf(L->w3, F * D);
        bf16_round_buf(L->w2, D * F);
    }
}
