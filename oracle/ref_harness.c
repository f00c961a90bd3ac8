/*
 * ref_harness.c -- drives the reference engine's own C code (test
 * infrastructure only).
 *
 * oracle/Makefile compiles this file together with the reference sources
 * src/ai/{quant,tensor,gguf,llm}.c, taken where they lie, into
 * oracle/_ref/libholo_ref.so.  The functions here only fill the reference's
 * public structs (src/ai/llm.h:22-200) in memory, so no GGUF file is needed,
 * and call the reference's own entry points: matmul_q (llm.c:770),
 * llm_forward (llm.c:1015), llm_sample (llm.c:1281), llm_reset (llm.c:732),
 * llm_tokenize (llm.c:178), and gguf.c's metadata readers.
 */
#include "gguf.h"
#include "llm.h"
#include "quant.h"

#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* weight-type globals of src/ai/llm.c:335-342 */
extern int g_emb_type, g_weight_type, g_v_weight_type, g_w1_weight_type;
extern int g_w2_weight_type, g_w3_weight_type, g_output_type, g_emb_vocab_size;
extern void matmul_q(float *dst, const void *M, const float *v,
                     int out_dim, int in_dim, int quant_type);

/* Reference matmul_q over row slices, one slice per thread.  matmul_q itself
 * is unchanged; each row's arithmetic is the same whatever the slicing. */
void href_matmul_q_threads(float *dst, const void *M, const float *v,
                           int out_dim, int in_dim, int qtype, int nthreads) {
    size_t row_bytes = quant_row_size(qtype, in_dim);
    if (qtype == GGML_TYPE_F32) row_bytes = (size_t)in_dim * 4;
    if (nthreads <= 1) { matmul_q(dst, M, v, out_dim, in_dim, qtype); return; }
#pragma omp parallel num_threads(nthreads)
    {
        int t = omp_get_thread_num(), n = omp_get_num_threads();
        int r0 = (int)((long long)out_dim * t / n), r1 = (int)((long long)out_dim * (t + 1) / n);
        if (r1 > r0)
            matmul_q(dst + r0, (const char *)M + (size_t)r0 * row_bytes, v, r1 - r0, in_dim, qtype);
    }
}

typedef struct {
    llm_ctx_t ctx;
} href_model_t;

href_model_t *href_model_create(int n_layers, int dim, int n_heads, int n_kv_heads,
                                int head_dim, int ffn_dim, int vocab, int max_seq,
                                float rope_base, float eps) {
    href_model_t *m = (href_model_t *)calloc(1, sizeof(href_model_t));
    llm_ctx_t *c = &m->ctx;
    strcpy(c->config.arch, "llama");
    c->config.vocab_size = vocab;
    c->config.context_length = max_seq;
    c->config.embedding_dim = dim;
    c->config.n_layers = n_layers;
    c->config.n_heads = n_heads;
    c->config.n_kv_heads = n_kv_heads;
    c->config.head_dim = head_dim;
    c->config.ffn_dim = ffn_dim;
    c->config.rope_freq_base = rope_base;
    c->config.rms_norm_eps = eps;
    c->config.eos_token = -1;
    c->weights.n_layers = n_layers;
    c->weights.layers = calloc(n_layers, sizeof(*c->weights.layers));
    int q_dim = n_heads * head_dim, kv_dim = n_kv_heads * head_dim;
    int big = dim > q_dim ? dim : q_dim;
    /* buffer sizes follow alloc_state (llm.c:534-560) */
    c->state.x = calloc(big, 4);
    c->state.xb = calloc(big, 4);
    c->state.xb2 = calloc(big, 4);
    c->state.hb = calloc(ffn_dim, 4);
    c->state.hb2 = calloc(ffn_dim, 4);
    c->state.q = calloc(big, 4);
    c->state.k = calloc(big > kv_dim ? big : kv_dim, 4);
    c->state.v = calloc(big > kv_dim ? big : kv_dim, 4);
    c->state.att = calloc((size_t)n_heads * max_seq, 4);
    c->state.logits = calloc(vocab, 4);
    size_t kv = (size_t)n_layers * max_seq * kv_dim;
    c->kv_cache.key_cache = calloc(kv, 4);
    c->kv_cache.value_cache = calloc(kv, 4);
    c->kv_cache.max_seq_len = max_seq;
    c->kv_cache.n_layers = n_layers;
    c->kv_cache.n_kv_heads = n_kv_heads;
    c->kv_cache.head_dim = head_dim;
    c->max_tokens = max_seq;
    c->tokens = calloc(max_seq, sizeof(int));
    c->loaded = true;
    return m;
}

/* Types of the weight globals llm_forward reads (llm.c:1035, 1107, 1250). */
void href_model_set_types(href_model_t *m, int layer_type, int emb_type, int out_type) {
    (void)m;
    g_weight_type = g_v_weight_type = layer_type;
    g_w1_weight_type = g_w2_weight_type = g_w3_weight_type = layer_type;
    g_emb_type = emb_type;
    g_output_type = out_type;
    g_emb_vocab_size = m->ctx.config.vocab_size;
    for (int l = 0; l < m->ctx.weights.n_layers; l++) {
        m->ctx.weights.layers[l].wv_type = layer_type;
        m->ctx.weights.layers[l].w2_type = layer_type;
    }
}

/* Per-tensor types as llm.c:335-342 binds them for mixed files: wq/wk/wo/w1/w3
 * share g_weight_type, each layer's wv and w2 carry their own type. */
void href_model_set_types_mixed(href_model_t *m, int layer_type, int wv_type, int w2_type, int emb_type,
                                int out_type) {
    href_model_set_types(m, layer_type, emb_type, out_type);
    g_v_weight_type = wv_type;
    g_w2_weight_type = w2_type;
    for (int l = 0; l < m->ctx.weights.n_layers; l++) {
        m->ctx.weights.layers[l].wv_type = wv_type;
        m->ctx.weights.layers[l].w2_type = w2_type;
    }
}

/* One layer's wv / w2 types, as load_weights binds them per tensor
 * (llm.c:445-447, 505-507: the globals follow layer 0). */
void href_model_set_layer_types(href_model_t *m, int l, int wv_type, int w2_type) {
    m->ctx.weights.layers[l].wv_type = wv_type;
    m->ctx.weights.layers[l].w2_type = w2_type;
    if (l == 0) {
        g_v_weight_type = wv_type;
        g_w2_weight_type = w2_type;
    }
}

void href_model_set_layer(href_model_t *m, int l, void *attn_norm, void *wq, void *wk,
                          void *wv, void *wo, void *ffn_norm, void *w1, void *w2, void *w3) {
    typeof(m->ctx.weights.layers[0]) *L = &m->ctx.weights.layers[l];
    L->attn_norm = attn_norm; L->wq = wq; L->wk = wk; L->wv = wv; L->wo = wo;
    L->ffn_norm = ffn_norm; L->w1 = w1; L->w2 = w2; L->w3 = w3;
}

void href_model_set_globals(href_model_t *m, void *tok_emb, void *final_norm, void *output) {
    m->ctx.weights.tok_embeddings = tok_emb;
    m->ctx.weights.norm = final_norm;
    m->ctx.weights.output = output;
}

int href_forward(href_model_t *m, int token) { return llm_forward(&m->ctx, &token, 1); }
float *href_logits(href_model_t *m) { return m->ctx.state.logits; }
int href_pos(href_model_t *m) { return m->ctx.pos; }
void href_reset(href_model_t *m) { llm_reset(&m->ctx); }

/* token history used by the repetition penalty (llm.c:1292-1298) */
void href_push_token(href_model_t *m, int token) {
    if (m->ctx.n_tokens < m->ctx.max_tokens) m->ctx.tokens[m->ctx.n_tokens++] = token;
}

int href_sample(href_model_t *m, float temperature, float top_p, int top_k,
                float repeat_penalty, int repeat_last_n) {
    llm_sampler_t s;
    s.temperature = temperature;
    s.top_p = top_p;
    s.top_k = top_k;
    s.repeat_penalty = repeat_penalty;
    s.repeat_last_n = repeat_last_n;
    s.seed = 0;
    return llm_sample(&m->ctx, &s);
}

void href_model_free(href_model_t *m) {
    llm_ctx_t *c = &m->ctx;
    free(c->state.x); free(c->state.xb); free(c->state.xb2); free(c->state.hb);
    free(c->state.hb2); free(c->state.q); free(c->state.k); free(c->state.v);
    free(c->state.att); free(c->state.logits);
    free(c->kv_cache.key_cache); free(c->kv_cache.value_cache);
    free(c->weights.layers); free(c->tokens);
    free(m);
}

/* The reference's GGUF parser (gguf_open, gguf.c:280-395; gguf_mmap;
 * gguf_get_tensor_data, gguf.c:504-510) on a file: the bytes its loader
 * would hand to upload_tensor for tensor `name`, copied into dst (at most
 * cap).  Returns the byte count, or -1 (open), -2 (map), -3 (no such
 * tensor), -4 (cap too small); *type gets the tensor's ggml type. */
long long href_gguf_tensor(const char *path, const char *name, void *dst, long long cap, int *type) {
    gguf_ctx_t *g = gguf_open(path);
    if (!g) return -1;
    if (gguf_mmap(g) != 0) { gguf_close(g); return -2; }
    const gguf_tensor_info_t *t = gguf_find_tensor(g, name);
    if (!t) { gguf_close(g); return -3; }
    long long n = (long long)t->size_bytes;
    if (n > cap) { gguf_close(g); return -4; }
    memcpy(dst, gguf_get_tensor_data(g, t), (size_t)n);
    *type = (int)t->type;
    gguf_close(g);
    return n;
}

/* gguf_get_int / gguf_get_float (gguf.c) on a file's metadata */
long long href_gguf_int(const char *path, const char *key, long long dflt) {
    gguf_ctx_t *g = gguf_open(path);
    if (!g) return dflt;
    long long v = (long long)gguf_get_int(g, key, dflt);
    gguf_close(g);
    return v;
}
double href_gguf_float(const char *path, const char *key, double dflt) {
    gguf_ctx_t *g = gguf_open(path);
    if (!g) return dflt;
    double v = (double)gguf_get_float(g, key, (float)dflt);
    gguf_close(g);
    return v;
}

/* llm_tokenize (llm.c:178-221) with the tokenizer fields load_tokenizer
 * fills (llm.c:61-100) set in memory; vocab entries may be NULL. */
int href_tokenize(char **vocab, int vocab_size, int bos, int unk, const char *text, int *tokens,
                  int max_tokens, int add_bos) {
    llm_ctx_t *c = (llm_ctx_t *)calloc(1, sizeof(llm_ctx_t));
    if (!c) return -1;
    c->tokenizer.vocab = vocab;
    c->tokenizer.vocab_size = vocab_size;
    c->tokenizer.bos_token = bos;
    c->tokenizer.unk_token = unk;
    int n = llm_tokenize(c, text, tokens, max_tokens, add_bos != 0);
    free(c);
    return n;
}

/* Entry i of a GGUF string array as load_tokenizer copies it (strdup of the
 * entry's data, llm.c:78-81): its length, -1 if the key or entry is absent,
 * -2 if cap is too small (dst gets a NUL-terminated copy). */
long long href_gguf_string_at(const char *path, const char *key, long long i, char *dst, long long cap) {
    gguf_ctx_t *g = gguf_open(path);
    if (!g) return -1;
    uint64_t len = 0;
    const gguf_string_t *arr = (const gguf_string_t *)gguf_get_array(g, key, &len);
    long long r = -1;
    if (arr && i >= 0 && (uint64_t)i < len) {
        size_t n = strlen(arr[i].data);
        if ((long long)n + 1 > cap) r = -2;
        else { memcpy(dst, arr[i].data, n + 1); r = (long long)n; }
    }
    gguf_close(g);
    return r;
}

/* length of a GGUF metadata array (gguf_get_array), 0 if absent */
long long href_gguf_array_len(const char *path, const char *key) {
    gguf_ctx_t *g = gguf_open(path);
    if (!g) return 0;
    uint64_t len = 0;
    gguf_get_array(g, key, &len);
    gguf_close(g);
    return (long long)len;
}

#ifdef HOLO_USE_CUDA
/* The reference's GPU host path (src/ai/llm_cuda.c), built only into the
 * drop-in library (oracle/Makefile `dropin`, linked to this repository's
 * libholo_cuda.so in place of the reference's cuda_ops.cu): llm_cuda_init
 * uploads the model with its own upload_tensor (cuda_malloc +
 * cuda_memcpy_h2d, llm_cuda.c:189-196), llm_forward_cuda runs one position
 * (llm_cuda.c:558-946) and leaves the logits in ctx->state.logits. */
extern int llm_cuda_init(llm_ctx_t *ctx);
extern int llm_forward_cuda(llm_ctx_t *ctx, const int *tokens, int n_tokens);
extern void llm_cuda_cleanup(void);
extern void llm_cuda_reset(void);

int href_cuda_init(href_model_t *m) { return llm_cuda_init(&m->ctx); }
int href_cuda_forward(href_model_t *m, int token) { return llm_forward_cuda(&m->ctx, &token, 1); }
void href_cuda_reset(href_model_t *m) { llm_reset(&m->ctx); llm_cuda_reset(); }
void href_cuda_cleanup(void) { llm_cuda_cleanup(); }
#endif
