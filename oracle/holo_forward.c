/*
 * holo_forward.c -- CPU restatement of holo's llm_forward (checker only).
 *
 * TEST INFRASTRUCTURE ONLY: see holo_oracle.h.  Nothing in the product
 * library links this file.
 *
 * ho_fwd_forward restates src/ai/llm.c:1015-1269 (llm_forward) for the llama
 * architecture (no Gemma scaling, no QK-norm, no biases), one position per
 * call, with two switches the device engine has:
 *
 *   act_mode HO_ACT_F32 : every matmul_q (llm.c:770-926) is the fp32-activation
 *                         restatement ho_matvec_f32act.  With kv_f16 = 0 this
 *                         is the reference's arithmetic, operation for
 *                         operation (pinned bit-exact to the compiled
 *                         llm_forward by tests/test_forward_oracle.py).
 *   act_mode HO_ACT_Q8  : every matmul_q input is quantized to Q8 per
 *                         32-block (ho_quantize_act_q8) and the product is the
 *                         integer block dot ho_matvec_q8act -- the device's
 *                         HOLO_ACT_Q8 matvec.  F16/F32 weights keep fp32
 *                         activations, as on the device.
 *   kv_f16              : K and V are rounded to binary16 (nearest even) when
 *                         stored in the cache and widened exactly when read,
 *                         as the device's fp16 cache stores them.
 *
 * The vector helpers follow src/ai/tensor.c as the reference is built here
 * (-mavx2 -mfma): vec_dot (tensor.c:129-157) accumulates 8 lanes with fused
 * multiply-adds and then sums them as _mm256_extractf128_ps + _mm_add_ps +
 * two _mm_hadd_ps do; rms_norm (tensor.c:242-255), softmax (tensor.c:300-319)
 * and silu (tensor.c:218-222) are sequential.  RoPE is the rotate-half loop
 * of llm.c:1135-1163 (powf, cosf, sinf per pair).  Compiled with
 * -ffp-contract=off, so each written operation rounds once, as in the
 * reference build.
 */
#include "holo_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

struct ho_fwd_layer {
    const float *attn_norm, *ffn_norm;
    const void *wq, *wk, *wv, *wo, *w1, *w2, *w3;
    int wv_type, w2_type;    /* -1: the model's */
};

struct ho_fwd_model {
    int n_layers, dim, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_seq;
    float rope_base, eps;
    int act_mode, kv_f16, nthreads;
    unsigned f32_roles;      /* diagnostics: bit r set -> role r keeps fp32 activations in HO_ACT_Q8 */
    /* weight types: wq/wk/wo/w1/w3 (g_weight_type), wv (wv_type), w2
     * (w2_type), embeddings (g_emb_type), output (g_output_type); llm.c:335-342 */
    int layer_type, wv_type, w2_type, emb_type, out_type;
    struct ho_fwd_layer *layers;
    const void *tok_emb, *output;
    const float *final_norm;
    int pos;
    float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits;
    void *kcache, *vcache;                 /* float or uint16_t, [layer][pos][kv_dim] */
    int8_t *qa;                            /* Q8 activation scratch */
    float *da;
    int32_t *sa;
};

/* ---- tensor.c helpers, as built with -mavx2 -mfma ------------------------- */

static float fwd_vec_dot(const float *a, const float *b, int n) {
    float l[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int j = 0; j < 8; j++) l[j] = fmaf(a[i + j], b[i + j], l[j]);
    /* _mm256_extractf128_ps / _mm_add_ps, then _mm_hadd_ps twice */
    float s0 = l[0] + l[4], s1 = l[1] + l[5], s2 = l[2] + l[6], s3 = l[3] + l[7];
    float r = (s0 + s1) + (s2 + s3);
    for (; i < n; i++) r += a[i] * b[i];
    return r;
}

static void fwd_rms_norm(float *dst, const float *x, const float *w, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float rms = sqrtf(ss / n + eps);
    float scale = 1.0f / rms;
    for (int i = 0; i < n; i++) dst[i] = x[i] * scale * w[i];
}

static void fwd_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    float scale = 1.0f / sum;
    for (int i = 0; i < n; i++) x[i] *= scale;
}

static void fwd_rope(float *v, int n_heads, int head_dim, int pos, float base) {
    int half = head_dim / 2;
    for (int h = 0; h < n_heads; h++) {
        float *vh = v + (size_t)h * head_dim;
        for (int i = 0; i < half; i++) {
            float freq = 1.0f / powf(base, (float)(2 * i) / head_dim);
            float theta = pos * freq;
            float c = cosf(theta), s = sinf(theta);
            float a = vh[i], b = vh[i + half];
            vh[i] = a * c - b * s;
            vh[i + half] = a * s + b * c;
        }
    }
}

static void fwd_embedding(struct ho_fwd_model *m, int token) {
    int dim = m->dim;
    if (m->emb_type == HO_TYPE_F32) {
        memcpy(m->x, (const float *)m->tok_emb + (size_t)token * dim, sizeof(float) * dim);
    } else if (m->emb_type == HO_TYPE_F16) {
        const uint16_t *e = (const uint16_t *)m->tok_emb + (size_t)token * dim;
        for (int i = 0; i < dim; i++) m->x[i] = ho_f16_to_f32(e[i]);
    } else {
        /* quantized tables: the dequantized values of the token's row */
        int64_t rb = ho_row_bytes(m->emb_type, dim);
        ho_dequant_row(m->emb_type, (const uint8_t *)m->tok_emb + (size_t)token * rb, m->x, dim, HO_Q4K_REF);
    }
}

/* matmul roles (for ho_fwd_set_f32_roles) */
enum { R_Q, R_K, R_V, R_O, R_W1, R_W3, R_W2, R_OUT };

/* matmul_q (llm.c:770-926) in the model's activation mode */
static void fwd_matmul(struct ho_fwd_model *m, float *y, const void *W, const float *x, int rows, int cols,
                       int type, int role) {
    if (m->act_mode == HO_ACT_Q8 && type != HO_TYPE_F16 && type != HO_TYPE_F32 && !((m->f32_roles >> role) & 1u)) {
        ho_quantize_act_q8(x, cols, m->qa, m->da, m->sa);
        ho_matvec_q8act(type, W, m->qa, m->da, m->sa, y, rows, cols, HO_Q4K_REF, NULL, m->nthreads);
    } else if (type == HO_TYPE_F32) {
        for (int r = 0; r < rows; r++) y[r] = fwd_vec_dot((const float *)W + (size_t)r * cols, x, cols);
    } else {
        ho_matvec_f32act(type, W, x, y, rows, cols, HO_Q4K_REF, m->nthreads);
    }
}

/* ---- model ------------------------------------------------------------------ */

struct ho_fwd_model *ho_fwd_create(int n_layers, int dim, int n_heads, int n_kv_heads, int head_dim,
                                   int ffn_dim, int vocab, int max_seq, float rope_base, float eps,
                                   int act_mode, int kv_f16, int nthreads) {
    struct ho_fwd_model *m = (struct ho_fwd_model *)calloc(1, sizeof(*m));
    if (!m) return NULL;
    m->n_layers = n_layers; m->dim = dim; m->n_heads = n_heads; m->n_kv_heads = n_kv_heads;
    m->head_dim = head_dim; m->ffn_dim = ffn_dim; m->vocab = vocab; m->max_seq = max_seq;
    m->rope_base = rope_base; m->eps = eps;
    m->act_mode = act_mode; m->kv_f16 = kv_f16; m->nthreads = nthreads < 1 ? 1 : nthreads;
    m->layer_type = m->wv_type = m->w2_type = HO_TYPE_Q4_K;
    m->emb_type = HO_TYPE_F16;
    m->out_type = HO_TYPE_Q8_0;
    int q_dim = n_heads * head_dim, kv_dim = n_kv_heads * head_dim;
    int big = dim > q_dim ? dim : q_dim;
    big = big > ffn_dim ? big : ffn_dim;
    m->layers = (struct ho_fwd_layer *)calloc((size_t)n_layers, sizeof(struct ho_fwd_layer));
    for (int l = 0; m->layers && l < n_layers; l++) m->layers[l].wv_type = m->layers[l].w2_type = -1;
    m->x = (float *)calloc(big, 4); m->xb = (float *)calloc(big, 4); m->xb2 = (float *)calloc(big, 4);
    m->hb = (float *)calloc(ffn_dim, 4); m->hb2 = (float *)calloc(ffn_dim, 4);
    m->q = (float *)calloc(q_dim, 4); m->k = (float *)calloc(kv_dim, 4); m->v = (float *)calloc(kv_dim, 4);
    m->att = (float *)calloc((size_t)max_seq, 4);
    m->logits = (float *)calloc(vocab, 4);
    size_t kv = (size_t)n_layers * max_seq * kv_dim;
    m->kcache = calloc(kv, kv_f16 ? 2 : 4);
    m->vcache = calloc(kv, kv_f16 ? 2 : 4);
    m->qa = (int8_t *)calloc(big, 1);
    m->da = (float *)calloc(big / 32 + 1, 4);
    m->sa = (int32_t *)calloc(big / 32 + 1, 4);
    if (!m->layers || !m->x || !m->xb || !m->xb2 || !m->hb || !m->hb2 || !m->q || !m->k || !m->v || !m->att ||
        !m->logits || !m->kcache || !m->vcache || !m->qa || !m->da || !m->sa) {
        ho_fwd_free(m);
        return NULL;
    }
    return m;
}

void ho_fwd_set_types(struct ho_fwd_model *m, int layer_type, int wv_type, int w2_type, int emb_type,
                      int out_type) {
    m->layer_type = layer_type; m->wv_type = wv_type; m->w2_type = w2_type;
    m->emb_type = emb_type; m->out_type = out_type;
}

void ho_fwd_set_layer_types(struct ho_fwd_model *m, int l, int wv_type, int w2_type) {
    m->layers[l].wv_type = wv_type;
    m->layers[l].w2_type = w2_type;
}

void ho_fwd_set_layer(struct ho_fwd_model *m, int l, const float *attn_norm, const void *wq, const void *wk,
                      const void *wv, const void *wo, const float *ffn_norm, const void *w1, const void *w2,
                      const void *w3) {
    struct ho_fwd_layer *L = &m->layers[l];
    L->attn_norm = attn_norm; L->wq = wq; L->wk = wk; L->wv = wv; L->wo = wo;
    L->ffn_norm = ffn_norm; L->w1 = w1; L->w2 = w2; L->w3 = w3;
}

void ho_fwd_set_globals(struct ho_fwd_model *m, const void *tok_emb, const float *final_norm, const void *output) {
    m->tok_emb = tok_emb; m->final_norm = final_norm; m->output = output;
}

void ho_fwd_reset(struct ho_fwd_model *m) { m->pos = 0; }
void ho_fwd_set_f32_roles(struct ho_fwd_model *m, unsigned mask) { m->f32_roles = mask; }

int ho_fwd_debug_vector(const struct ho_fwd_model *m, int which, float *dst) {
    const int q_dim = m->n_heads * m->head_dim, kv_dim = m->n_kv_heads * m->head_dim;
    switch (which) {
    case 0: memcpy(dst, m->x, sizeof(float) * m->dim); return m->dim;
    case 1:
        memcpy(dst, m->q, sizeof(float) * q_dim);
        memcpy(dst + q_dim, m->k, sizeof(float) * kv_dim);
        memcpy(dst + q_dim + kv_dim, m->v, sizeof(float) * kv_dim);
        return q_dim + 2 * kv_dim;
    case 2: memcpy(dst, m->xb2, sizeof(float) * q_dim); return q_dim;
    case 3: memcpy(dst, m->hb, sizeof(float) * m->ffn_dim); return m->ffn_dim;
    case 4: memcpy(dst, m->logits, sizeof(float) * m->vocab); return m->vocab;
    default: return -1;
    }
}
int ho_fwd_pos(const struct ho_fwd_model *m) { return m->pos; }
const float *ho_fwd_logits(const struct ho_fwd_model *m) { return m->logits; }

static void kv_store(struct ho_fwd_model *m, void *cache, size_t off, const float *src, int n) {
    if (m->kv_f16) {
        uint16_t *c = (uint16_t *)cache + off;
        for (int i = 0; i < n; i++) c[i] = ho_f32_to_f16_rn(src[i]);
    } else {
        memcpy((float *)cache + off, src, sizeof(float) * n);
    }
}

/* row `off` of the cache, widened into tmp when it is binary16 */
static const float *kv_row(struct ho_fwd_model *m, const void *cache, size_t off, float *tmp, int n) {
    if (!m->kv_f16) return (const float *)cache + off;
    const uint16_t *c = (const uint16_t *)cache + off;
    for (int i = 0; i < n; i++) tmp[i] = ho_f16_to_f32(c[i]);
    return tmp;
}

/* One position: llm.c:1049-1266 with matmul_q in the model's mode. */
int ho_fwd_forward(struct ho_fwd_model *m, int token) {
    if (token < 0 || token >= m->vocab || m->pos >= m->max_seq) return -1;
    const int dim = m->dim, hd = m->head_dim, nh = m->n_heads, nkv = m->n_kv_heads;
    const int q_dim = nh * hd, kv_dim = nkv * hd, ffn = m->ffn_dim, pos = m->pos;
    const size_t layer_size = (size_t)m->max_seq * kv_dim;
    float tmp_k[1024], tmp_v[1024];
    if (hd > 1024) return -1;
    fwd_embedding(m, token);
    for (int l = 0; l < m->n_layers; l++) {
        const struct ho_fwd_layer *L = &m->layers[l];
        fwd_rms_norm(m->xb, m->x, L->attn_norm, dim, m->eps);
        fwd_matmul(m, m->q, L->wq, m->xb, q_dim, dim, m->layer_type, R_Q);
        fwd_matmul(m, m->k, L->wk, m->xb, kv_dim, dim, m->layer_type, R_K);
        fwd_matmul(m, m->v, L->wv, m->xb, kv_dim, dim, L->wv_type >= 0 ? L->wv_type : m->wv_type, R_V);
        fwd_rope(m->q, nh, hd, pos, m->rope_base);
        fwd_rope(m->k, nkv, hd, pos, m->rope_base);
        kv_store(m, m->kcache, l * layer_size + (size_t)pos * kv_dim, m->k, kv_dim);
        kv_store(m, m->vcache, l * layer_size + (size_t)pos * kv_dim, m->v, kv_dim);
        const int group = nkv > 0 ? nh / nkv : 1;
        memset(m->xb2, 0, sizeof(float) * q_dim);
        for (int h = 0; h < nh; h++) {
            const float *qh = m->q + (size_t)h * hd;
            float *out = m->xb2 + (size_t)h * hd;
            const int kvh = h / group;
            for (int p = 0; p <= pos; p++) {
                const float *kp = kv_row(m, m->kcache, l * layer_size + (size_t)p * kv_dim + (size_t)kvh * hd,
                                         tmp_k, hd);
                float score = fwd_vec_dot(qh, kp, hd);
                m->att[p] = score / sqrtf((float)hd);
            }
            fwd_softmax(m->att, pos + 1);
            for (int p = 0; p <= pos; p++) {
                const float *vp = kv_row(m, m->vcache, l * layer_size + (size_t)p * kv_dim + (size_t)kvh * hd,
                                         tmp_v, hd);
                const float a = m->att[p];
                for (int d = 0; d < hd; d++) out[d] += a * vp[d];
            }
        }
        fwd_matmul(m, m->xb, L->wo, m->xb2, dim, q_dim, m->layer_type, R_O);
        for (int i = 0; i < dim; i++) m->x[i] = m->x[i] + m->xb[i];
        fwd_rms_norm(m->xb, m->x, L->ffn_norm, dim, m->eps);
        fwd_matmul(m, m->hb, L->w1, m->xb, ffn, dim, m->layer_type, R_W1);
        fwd_matmul(m, m->hb2, L->w3, m->xb, ffn, dim, m->layer_type, R_W3);
        for (int i = 0; i < ffn; i++) m->hb[i] = m->hb[i] / (1.0f + expf(-m->hb[i]));
        for (int i = 0; i < ffn; i++) m->hb[i] = m->hb[i] * m->hb2[i];
        fwd_matmul(m, m->xb, L->w2, m->hb, dim, ffn, L->w2_type >= 0 ? L->w2_type : m->w2_type, R_W2);
        for (int i = 0; i < dim; i++) m->x[i] = m->x[i] + m->xb[i];
    }
    /* the final norm into xb (the reference normalises x in place; the values
     * are the same, and x stays the residual stream for ho_fwd_debug_vector) */
    fwd_rms_norm(m->xb, m->x, m->final_norm, dim, m->eps);
    fwd_matmul(m, m->logits, m->output, m->xb, m->vocab, dim, m->out_type, R_OUT);
    m->pos++;
    return 0;
}

void ho_fwd_free(struct ho_fwd_model *m) {
    if (!m) return;
    free(m->layers); free(m->x); free(m->xb); free(m->xb2); free(m->hb); free(m->hb2);
    free(m->q); free(m->k); free(m->v); free(m->att); free(m->logits);
    free(m->kcache); free(m->vcache); free(m->qa); free(m->da); free(m->sa);
    free(m);
}
