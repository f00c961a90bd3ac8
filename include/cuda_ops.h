/*
 * cuda_ops.h -- the C ABI of holo's CUDA op library, served by the B200
 * decode-path library (libholo_cuda.so).
 *
 * Every declaration here has the name, parameter list and meaning of the
 * reference header include/cuda_ops.h of privuser2738/google-classic (the
 * line numbers below are that file's), so the reference's host code
 * (src/ai/llm_cuda.c) compiles and links against this library unchanged.
 * Additive entry points (repacked-weight upload, activation mode, status,
 * multi-GPU, the fused decode step, the device sampler) are declared in
 * holo_b200.h.
 *
 * Conventions kept from the reference:
 *   - all tensor pointers are device pointers, normally from cuda_malloc;
 *   - calls are ordered with respect to each other (one implicit stream per
 *     device); cuda_memcpy_h2d/d2h/d2d, cuda_vec_dot and cuda_argmax return
 *     only after the device work they depend on has finished;
 *   - errors never abort: the reference prints and returns; this library
 *     also records a sticky status readable with cuda_last_status().
 */
#ifndef HOLO_CUDA_OPS_H
#define HOLO_CUDA_OPS_H

#ifdef __cplusplus
extern "C" {
#endif

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

/* -- device set-up (reference cuda_ops.h:18-26) ---------------------------- */
int cuda_init(void);                      /* 0 on success, -1 without a device */
void cuda_cleanup(void);
bool cuda_available(void);
void cuda_print_info(void);
int cuda_get_device_count(void);
size_t cuda_get_free_memory(void);
const char *cuda_get_device_name(void);

/* -- memory (reference cuda_ops.h:29-36); cuda_malloc returns NULL on failure */
void *cuda_malloc(size_t size);
void cuda_free(void *ptr);
void cuda_memcpy_h2d(void *dst, const void *src, size_t size);
void cuda_memcpy_d2h(void *dst, const void *src, size_t size);
void cuda_memcpy_d2d(void *dst, const void *src, size_t size);
void cuda_memcpy_d2d_async(void *dst, const void *src, size_t size);
void cuda_memcpy_d2h_async(void *dst, const void *src, size_t size);
void cuda_memset(void *ptr, int value, size_t size);

/* -- synchronisation (reference cuda_ops.h:39-40) --------------------------- */
void cuda_sync(void);
void cuda_sync_copy(void);

/* -- fp32 vectors (reference cuda_ops.h:43-46) ------------------------------ */
void cuda_vec_add(float *dst, const float *a, const float *b, int n);
void cuda_vec_mul(float *dst, const float *a, const float *b, int n);
void cuda_vec_scale(float *dst, const float *a, float scale, int n);
float cuda_vec_dot(const float *a, const float *b, int n);

/* -- matrix x vector (reference cuda_ops.h:50-57) ---------------------------
 * dst[out_dim] = M[out_dim][in_dim] . v[in_dim], M in GGUF row order.  For
 * the quantized types M is either raw GGUF blocks (as uploaded with
 * cuda_malloc + cuda_memcpy_h2d) or a pointer returned by cuda_upload_quant
 * (holo_b200.h), which selects the tiled fast path. */
void cuda_matmul_f32(float *dst, const float *M, const float *v, int out_dim, int in_dim);
void cuda_matmul_f16(float *dst, const void *M, const float *v, int out_dim, int in_dim);
void cuda_matmul_q8_0(float *dst, const void *M, const float *v, int out_dim, int in_dim);
void cuda_matmul_q4_0(float *dst, const void *M, const float *v, int out_dim, int in_dim);
void cuda_matmul_q4_k(float *dst, const void *M, const float *v, int out_dim, int in_dim);
void cuda_matmul_q6_k(float *dst, const void *M, const float *v, int out_dim, int in_dim);

/* Q, K and V projections of one input in a single launch (reference 60-62) */
void cuda_batched_qkv_q8_0(float *q_out, float *k_out, float *v_out,
                           const void *Wq, const void *Wk, const void *Wv,
                           const float *x, int q_dim, int kv_dim, int in_dim);

/* out = silu(W1.x) * (W3.x) in a single launch (reference 65-66) */
void cuda_batched_ffn_gate_up_q8_0(float *out, const void *W1, const void *W3,
                                   const float *x, int ffn_dim, int in_dim);

/* -- activations (reference cuda_ops.h:69-72) ------------------------------- */
void cuda_silu(float *x, int n);
void cuda_silu_mul(float *dst, const float *a, const float *b, int n);
void cuda_gelu(float *x, int n);
void cuda_relu(float *x, int n);

/* -- normalisation (reference cuda_ops.h:75-76).  As in the reference
 * (src/ai/cuda_ops.cu:1506-1511), cuda_layer_norm applies RMS normalisation
 * and ignores `bias`. */
void cuda_rms_norm(float *dst, const float *x, const float *weight, int n, float eps);
void cuda_layer_norm(float *dst, const float *x, const float *weight, const float *bias,
                     int n, float eps);

/* -- softmax (reference cuda_ops.h:79-80) ----------------------------------- */
void cuda_softmax(float *dst, const float *x, int n);
void cuda_softmax_inplace(float *x, int n);

/* -- attention (reference cuda_ops.h:83-114) --------------------------------
 * Caches are fp32 [max_seq][n_kv_heads*head_dim]; query head h reads KV head
 * h / (n_heads / n_kv_heads). */
void cuda_attention_scores(float *dst, const float *Q, const float *K,
                           int seq_len, int kv_len, int head_dim, float scale);
void cuda_attention_apply(float *dst, const float *scores, const float *V,
                          int seq_len, int kv_len, int head_dim);
void cuda_attention_single(float *dst, const float *q,
                           const float *k_cache, const float *v_cache,
                           float *att_buf, int kv_len, int head_dim,
                           int kv_head, int kv_dim);
void cuda_multi_head_attention(float *dst, const float *q,
                               const float *k_cache, const float *v_cache,
                               int kv_len, int head_dim, int n_heads, int n_kv_heads);

/* -- rotary embedding, rotate-half pairing (i, i + head_dim/2) (reference 117) */
void cuda_rope_apply(float *q, float *k, int pos, int head_dim, int n_heads,
                     int n_kv_heads, float freq_base);

/* -- embedding rows, table [vocab][dim] (reference cuda_ops.h:121-130) ------ */
void cuda_get_embedding_f32(float *dst, const float *embeddings, int token, int dim, int vocab_size);
void cuda_get_embedding_f16(float *dst, const void *embeddings, int token, int dim, int vocab_size);
void cuda_get_embedding_q8_0(float *dst, const void *embeddings, int token, int dim, int vocab_size);
void cuda_get_embedding_q4_0(float *dst, const void *embeddings, int token, int dim, int vocab_size);
void cuda_get_embedding_q6_k(float *dst, const void *embeddings, int token, int dim, int vocab_size);

/* -- sampling helper: index of the first maximum (reference cuda_ops.h:133) - */
int cuda_argmax(const float *x, int n);

#ifdef __cplusplus
}
#endif

#endif /* HOLO_CUDA_OPS_H */
