/*
 * holo_oracle.h -- CPU restatement of holo's quantized decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path is
 * compared against; it is never linked into, called by, or shipped with the
 * product library.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg load it.
 *
 * Every function restates an algorithm of the reference engine (holo, in
 * privuser2738/google-classic) and names the file:line it follows.  Paths are
 * relative to that project's root.  Where the reference has no code for a
 * step (Q8 activation quantization and the integer block dot), the function
 * says so and defines the arithmetic order it uses.
 *
 * Build: oracle/Makefile (gcc -O2 -std=gnu11 -ffp-contract=off, no fast-math),
 * so every float operation below rounds exactly once, as written.
 */
#ifndef HOLO_ORACLE_H
#define HOLO_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids, as in src/ai/quant.h:20-33 */
#define HO_TYPE_F32  0
#define HO_TYPE_F16  1
#define HO_TYPE_Q4_0 2
#define HO_TYPE_Q8_0 8
#define HO_TYPE_Q4_K 12
#define HO_TYPE_Q6_K 14

/* Q4_K semantics of the 144-byte super-block.
 * HO_Q4K_REF : src/ai/quant.c:277-311 (6-bit unpack quant.c:290-297,
 *              sub-block j = 16 bytes, low nibble -> j*32+l, high -> j*32+l+16).
 * HO_Q4K_GGML: src/ai/cuda_ops.cu:684-732 (get_scale_min_k4 unpack, 32 bytes
 *              per 64 values, low nibbles -> first 32, high -> next 32). */
#define HO_Q4K_REF  0
#define HO_Q4K_GGML 1

/* exact binary16 -> binary32 (src/ai/quant.c:44-82) */
float ho_f16_to_f32(uint16_t h);
/* binary32 -> binary16, round to nearest even (used by the generators only) */
uint16_t ho_f32_to_f16_rn(float f);

/* bytes of one row of `cols` values in GGUF packing (src/ai/quant.c:710-719) */
int64_t ho_row_bytes(int type, int64_t cols);

/* dequantized values (src/ai/quant.c:118-128, 136-153, 277-311) */
void ho_dequant_row(int type, const void *row, float *y, int64_t cols, int q4k_layout);

/* fp32-activation matvec, the arithmetic of src/ai/llm.c:770-926 (matmul_q):
 *   Q8_0 : llm.c:836-874 (8 lane accumulators, then the horizontal sum)
 *   Q4_0 : llm.c:893-915
 *   Q4_K : quant.c:541-580 via llm.c:916-918 (or the ggml layout, same order)
 *   F16  : llm.c:817-827
 * rows run in parallel with OpenMP when nthreads > 1; each row's arithmetic is
 * unchanged. */
void ho_matvec_f32act(int type, const void *W, const float *x, float *y,
                      int rows, int cols, int q4k_layout, int nthreads);

/* Q8 activation quantizer.  The reference has no such code (its matvecs take
 * fp32 activations), so this is the build's own definition, per block of 32:
 *   amax = max |x|;  d = amax / 127 (fp32);  id = d != 0 ? 1/d : 0;
 *   q = rint(x * id)  (round half to even; x*id rounded once)
 *   asum = sum of q (int32)  */
void ho_quantize_act_q8(const float *x, int64_t n, int8_t *q, float *d, int32_t *asum);

/* Q8-activation matvec.  Per 32-block integer dot, exact:
 *   Q8_0 : isum = sum qw*qa
 *   Q4_0 : isum = sum (nib-8)*qa
 *   Q4_K : isum = sum nib*qa  (the min term uses asum)
 * then float, in this fixed order, accumulated over blocks in K order:
 *   Q8_0, Q4_0 : y += (dw*da) * (float)isum
 *   Q4_K       : y += da * ((d*sc)*(float)isum - (dmin*m)*(float)asum)
 * If isums != NULL it receives the integer sums, [rows][cols/32]. */
void ho_matvec_q8act(int type, const void *W, const int8_t *q, const float *d,
                     const int32_t *asum, float *y, int rows, int cols,
                     int q4k_layout, int32_t *isums, int nthreads);

/* Rewrite one Q4_K super-block of either semantics into the reference
 * (quant.c) semantics with identical dequantized values. */
void ho_q4k_to_ref_layout(const void *src_block, void *dst_block, int src_layout);

/* The reference's tokenizer (llm_tokenize, src/ai/llm.c:178-221, with its
 * byte fallback find_byte_token, llm.c:113-175), restated literally: every
 * position scans the whole vocabulary.  vocab entries may be NULL. */
int ho_tokenize(const char *const *vocab, int vocab_size, int bos, int unk, const char *text,
                int *tokens, int max_tokens, int add_bos);

/* ---- end-to-end forward (holo_forward.c) -----------------------------------
 * llm_forward (src/ai/llm.c:1015-1269) restated for the llama architecture,
 * one position per call, with the device engine's activation mode (HO_ACT_F32:
 * matmul_q's arithmetic; HO_ACT_Q8: Q8 activations and integer block dots)
 * and KV cache precision (kv_f16: binary16, nearest even).  Weights are raw
 * GGUF blocks read in place; norms are fp32. */
#define HO_ACT_F32 0
#define HO_ACT_Q8  1
struct ho_fwd_model;
struct ho_fwd_model *ho_fwd_create(int n_layers, int dim, int n_heads, int n_kv_heads, int head_dim,
                                   int ffn_dim, int vocab, int max_seq, float rope_base, float eps,
                                   int act_mode, int kv_f16, int nthreads);
/* weight types per tensor role (llm.c:335-342): wq/wk/wo/w1/w3, wv, w2,
 * token embeddings, output matrix */
void ho_fwd_set_types(struct ho_fwd_model *m, int layer_type, int wv_type, int w2_type, int emb_type,
                      int out_type);
/* one layer's wv / w2 types (per tensor, llm.c:445-507); default the model's */
void ho_fwd_set_layer_types(struct ho_fwd_model *m, int l, int wv_type, int w2_type);
void ho_fwd_set_layer(struct ho_fwd_model *m, int l, const float *attn_norm, const void *wq, const void *wk,
                      const void *wv, const void *wo, const float *ffn_norm, const void *w1, const void *w2,
                      const void *w3);
void ho_fwd_set_globals(struct ho_fwd_model *m, const void *tok_emb, const float *final_norm, const void *output);
/* one position (the next one); 0, or -1 for a bad token or a full cache */
int ho_fwd_forward(struct ho_fwd_model *m, int token);
const float *ho_fwd_logits(const struct ho_fwd_model *m);
int ho_fwd_pos(const struct ho_fwd_model *m);
void ho_fwd_reset(struct ho_fwd_model *m);
/* diagnostics: in HO_ACT_Q8, the matmuls of the roles whose bit is set keep
 * fp32 activations (bits 0..7: q, k, v, o, w1, w3, w2, output) */
void ho_fwd_set_f32_roles(struct ho_fwd_model *m, unsigned mask);
/* diagnostics: the last layer's vectors after a forward -- 0 x (residual
 * stream), 1 q|k|v (q, k rotated), 2 attention output, 3 SwiGLU output,
 * 4 logits; returns the length */
int ho_fwd_debug_vector(const struct ho_fwd_model *m, int which, float *dst);
void ho_fwd_free(struct ho_fwd_model *m);

#ifdef __cplusplus
}
#endif
#endif
