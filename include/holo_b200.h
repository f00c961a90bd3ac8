/*
 * holo_b200.h -- additive entry points of the B200 decode-path library.
 *
 * None of these exist in the reference ABI (include/cuda_ops.h of
 * privuser2738/google-classic); each comment names the reference code whose
 * job it takes over or extends.  Plain C types only.
 */
#ifndef HOLO_B200_H
#define HOLO_B200_H

#ifdef __cplusplus
extern "C" {
#endif

#include <stddef.h>
#include <stdint.h>

/* ---- status ----------------------------------------------------------------
 * The reference's ops return void and ignore launch errors
 * (src/ai/cuda_ops.cu:21-37).  Every entry point here records the first
 * failure in a sticky status: a cudaError_t value, or one of the HOLO_E_*
 * codes below.  cuda_last_status() also collects the device-side error word
 * written by kernels whose bounded waits timed out (it synchronises). */
#define HOLO_STATUS_OK        0   /* success (not HOLO_OK: the reference's holo.h
                                     declares that name as an enumerator of
                                     holo_result_t, include/holo.h:28-35) */
#define HOLO_E_ARG         1001   /* bad shape / type / pointer               */
#define HOLO_E_NOMEM       1002   /* device allocation failed                 */
#define HOLO_E_UNSUPPORTED 1003   /* shape beyond a kernel's limits           */
#define HOLO_E_TIMEOUT     1004   /* a kernel's bounded wait gave up          */
#define HOLO_E_COMM        1005   /* collective failed or timed out           */
int cuda_last_status(void);
const char *cuda_last_status_string(void);
void cuda_clear_status(void);

/* ---- activation mode of the quantized matvecs -------------------------------
 * HOLO_ACT_F32: fp32 activations, the reference's arithmetic
 *               (src/ai/llm.c:770-926, src/ai/quant.c:541-580).
 * HOLO_ACT_Q8 : activations quantized per 32-element block to int8 with an
 *               fp32 scale inside the matvec; per-block integer dot products.
 * Default from env HOLO_ACT=f32|q8 (q8 when unset). */
#define HOLO_ACT_F32 0
#define HOLO_ACT_Q8  1
void cuda_set_act_mode(int mode);
int cuda_get_act_mode(void);

/* ---- Q4_K block semantics of uploaded weights ---------------------------
 * HOLO_Q4K_REF : src/ai/quant.c:277-311 (the CPU engine's decoding)
 * HOLO_Q4K_GGML: src/ai/cuda_ops.cu:684-732 (llama.cpp decoding)
 * The repacker rewrites either into one device layout.  Default from env
 * HOLO_Q4K_LAYOUT=ref|ggml (ref when unset). */
#define HOLO_Q4K_REF  0
#define HOLO_Q4K_GGML 1
void cuda_set_q4k_layout(int layout);
int cuda_get_q4k_layout(void);
/* Embedding row of a Q4_K table (raw GGUF blocks, token x dim, dim % 256 ==
 * 0), decoded in the current Q4_K layout.  Completes the embedding lookups of
 * cuda_ops.h: the reference's dispatcher (src/ai/llm_cuda.c:166-186) has no
 * Q4_K case and falls through to the F32 lookup. */
void cuda_get_embedding_q4_k(float *dst, const void *embeddings, int token, int dim, int vocab_size);

/* ---- repacked weights (replaces upload_tensor, src/ai/llm_cuda.c:189-196) ---
 * Uploads `rows` x `cols` values of GGUF blocks of `ggml_type` (Q8_0, Q4_0,
 * Q4_K) from host memory, repacks them once on the device into the tiled
 * layout, and returns the device pointer (free with cuda_free).  Passing it
 * as M to cuda_matmul_* selects the tiled kernels.  NULL on failure. */
void *cuda_upload_quant(const void *host_blocks, int ggml_type, int rows, int cols);
/* Same, from raw GGUF blocks already in device memory (left untouched). */
void *cuda_repack_quant(const void *dev_blocks, int ggml_type, int rows, int cols);
/* Bytes of the tiled copy of a rows x cols matrix (rows padded to 32). */
size_t cuda_quant_tiled_bytes(int ggml_type, int rows, int cols);

/* ---- programmatic dependent launch ------------------------------------------
 * When on, the tiled matvecs are launched with programmatic stream
 * serialisation: a matvec may start streaming its weights while the previous
 * kernel on the stream is still running, and waits for that kernel only
 * before it reads activations or writes outputs.  Safe when the weights are
 * not written by the kernel just before the matvec (they never are after
 * cuda_upload_quant returns).  Default off; env HOLO_PDL=1 turns it on. */
void cuda_set_pdl(int on);
int cuda_get_pdl(void);

/* ---- explicit matvec -------------------------------------------------------
 * dst = M . v (+ residual when residual != NULL, may alias dst), with the
 * activation mode given per call.  M raw or tiled as for cuda_matmul_*. */
void cuda_matvec(float *dst, const void *M, const float *v, int out_dim, int in_dim,
                 int ggml_type, int act_mode, const float *residual);

/* ---- independent matvecs in one launch ------------------------------------
 * No counterpart in the reference.  dst[i] = M[i] . v[i] for i < n, each M[i]
 * a tiled weight from cuda_upload_quant (its registered shape gives out_dim
 * and in_dim), activations per act_mode.  The matvecs must not depend on one
 * another (no v[j] is any dst[i]); their units form one sequence that one
 * persistent launch per weight type splits evenly over the SMs, so the
 * activation staging, quantization and split-K fix-up of each matrix stay off
 * a chain of per-matrix launches.  Every output row has the arithmetic of
 * cuda_matvec (within 1e-6: only the split points differ).  Returns 0 or the
 * error code it records (HOLO_E_ARG: a pointer is not a tiled weight;
 * HOLO_E_UNSUPPORTED: more than 65536 row-blocks of one type in a call). */
int cuda_matvec_batch(int n, float *const *dst, const void *const *M, const float *const *v, int act_mode);

/* ---- matvec without allocation ------------------------------------------------
 * No counterpart in the reference.  dst = M . v like cuda_matvec (no residual)
 * for a tiled weight M from cuda_upload_quant, but its split-K scratch is
 * static device memory (file-scope arrays found with cudaGetSymbolAddress),
 * so the call allocates and frees nothing.  It is for callers that cannot
 * allocate device memory once they are running: a host engine whose memory
 * budget is fixed and fully handed out at start-up (another allocator, such
 * as a framework's caching pool, owns the rest of the device), or a latency
 * loop where cudaMalloc/cudaFree would synchronise the device mid-token.
 * The caller still owns dst, M and v.  Limits: out_dim <= 262144 (8192
 * row-blocks; larger shapes are rejected with HOLO_E_UNSUPPORTED); the grid
 * is capped at 296 CTAs.  The static scratch (about 44 KB) is held by every
 * GPU that loads the library, until the process exits.
 * The first call on a device does the set-up (symbol addresses, status word
 * cleared), so make that first call before any stream capture.  Runs on the
 * thread's cuda_set_stream stream, else the library stream if the device is
 * initialised, else the legacy default stream.  Every call clears the
 * counters it uses first.  The scratch is shared by all calls on a device:
 * calls that overlap on the GPU (other streams or threads) race.  Returns 0,
 * or the error code it also records (HOLO_E_ARG, HOLO_E_UNSUPPORTED, a CUDA
 * error).  A launch whose bounded wait gave up leaves HOLO_E_TIMEOUT in the
 * path's status word: cuda_last_status reports it, cuda_clear_status resets it. */
int cuda_matvec_noalloc(float *dst, const void *M, const float *v, int out_dim, int in_dim,
                        int ggml_type, int act_mode);
/* Device address of that status word on the current device (doing the
 * set-up if needed; NULL if it failed).  For diagnostics and tests. */
void *cuda_matvec_noalloc_status_word(void);

/* ---- parity probes (run the device decode code on their own) ------------- */
/* dst[rows][cols] = dequantized values of M (raw or tiled). */
void cuda_dequantize_rows(float *dst, const void *M, int ggml_type, int rows, int cols);
/* Q8 activation quantizer: q[n], d[n/32], asum[n/32]. */
void cuda_quantize_act_q8(int8_t *q, float *d, int32_t *asum, const float *x, int n);
/* Per-32-block integer dot products of M (raw or tiled) with the Q8
 * quantization of v: dst[rows][cols/32] (int32). */
void cuda_block_sums_q8(int32_t *dst, const void *M, const float *v, int ggml_type,
                        int rows, int cols);

/* ---- streams ---------------------------------------------------------------
 * The library enqueues all work of the current device on one stream
 * (created by cuda_init).  cuda_get_stream returns it as a cudaStream_t;
 * cuda_set_stream(NULL) restores the library's own stream. */
void *cuda_get_stream(void);
/* Stream-ordered copies on that stream (the reference's cuda_memcpy_h2d/d2h
 * wait for the copy; these return at once): a batch of host inputs, the
 * kernels that read them and the copy of their results back can be enqueued
 * (or captured into one CUDA graph) and waited for once with cuda_sync().
 * The host buffer must stay valid until then; with pinned host memory the
 * copies overlap nothing else of the host. */
void cuda_memcpy_h2d_stream(void *dst, const void *src, size_t size);
void cuda_memcpy_d2h_stream(void *dst, const void *src, size_t size);
void cuda_set_stream(void *stream);
/* Select device `local_rank` for this thread and initialise it (one process
 * or thread per GPU); cuda_init() is cuda_init_rank(0, 1). */
int cuda_init_rank(int local_rank, int world_size);
/* Number of SMs of the current device (grid sizing). */
int cuda_sm_count(void);

/* ---- batch-1 decode engine ----------------------------------------------------
 * The decode call sequence of the reference -- llm_forward for one token
 * (src/ai/llm.c:1015-1269; its GPU twin llm_forward_cuda, llm_cuda.c:558-946)
 * and llm_sample (llm.c:1281-1328) -- as one model object whose token step is
 * a single CUDA graph: RMSNorm fused into the QKV, gate/up and output
 * matvecs, [Wq;Wk;Wv] and [W1;W3] each one weight, residual adds and SwiGLU
 * in matvec epilogues, the KV cache resident on the device, and the sampler on
 * the device.  Weights are given as pointers (host or device memory) to GGUF
 * blocks laid out as the reference loader reads them (row-major, rows of
 * in-dim values); they are copied and repacked, not kept. */
typedef struct {
    int n_layers, dim, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_seq;
    float rope_base;     /* RoPE frequency base (llm_config_t.rope_freq_base) */
    float eps;           /* RMSNorm epsilon */
    int layer_type;      /* GGUF type of wq wk wv wo w1 w2 w3: 8 Q8_0, 2 Q4_0, 12 Q4_K */
    int emb_type;        /* token embedding table: 0 F32, 1 F16, or GGUF blocks of Q8_0 (8),
                          * Q4_0 (2), Q4_K (12), Q6_K (14), dequantized once by
                          * holo_model_set_globals as get_embedding decodes them */
    int out_type;        /* GGUF type of the output (lm_head) matrix */
    int kv_f16;          /* 1: fp16 KV cache, 0: fp32 (the reference's) */
    int act_mode;        /* HOLO_ACT_Q8 or HOLO_ACT_F32 for every matvec */
    int world;           /* row sharding over this many GPUs (one process each); 0 or 1: none */
    int rank;            /* this process's shard, 0 <= rank < world */
    int batch;           /* sequences decoded together (2..64, one GPU) by the *_batch calls; 0 or 1: none */
    int rope_mode;       /* HOLO_ROPE_HALF (0): pairs (i, i + hd/2), the reference's rotation
                          * (src/ai/llm.c:1135-1163); HOLO_ROPE_ADJACENT (1): pairs (2i, 2i+1),
                          * the rotation llama.cpp applies to Llama weights converted to GGUF */
} holo_model_desc;
#define HOLO_ROPE_HALF 0
#define HOLO_ROPE_ADJACENT 1

typedef struct {         /* llm_sampler_t (src/ai/llm.h:167-174) without the seed */
    float temperature;   /* 0: greedy */
    float top_p;         /* in (0,1): nucleus; otherwise off */
    int top_k;           /* > 0: top-k; 0: off */
    float repeat_penalty;
    int repeat_last_n;
} holo_sampler_desc;

/* NULL on failure (status set).  head_dim 64/128/256, ffn_dim % 16 == 0. */
void *holo_model_create(const holo_model_desc *desc);
/* Layer weights: attn_norm/ffn_norm fp32 [dim]; wq [n_heads*hd][dim], wk wv
 * [n_kv_heads*hd][dim], wo [dim][n_heads*hd], w1 w3 [ffn][dim], w2 [dim][ffn];
 * GGUF blocks of layer_type, wv and w2 of the layer's types (below). */
/* GGUF types of one layer's wv and w2 (Q8_0, Q4_0, Q4_K or Q6_K; default
 * layer_type), set before that layer's holo_model_set_layer.  The reference
 * binds these two per layer (src/ai/llm.c:445-507: Q4_K_M files keep some
 * layers' attn_v / ffn_down in Q6_K) and dispatches each matmul on the
 * tensor's type (llm_cuda.c:140-163).  A model whose layers mix types runs
 * the one-launch-per-op graph and prompts one position a step; batch 1 on one
 * GPU only (HOLO_E_UNSUPPORTED otherwise). */
int holo_model_set_layer_types(void *model, int layer, int wv_type, int w2_type);
int holo_model_set_layer(void *model, int layer, const float *attn_norm, const void *wq, const void *wk,
                         const void *wv, const void *wo, const float *ffn_norm, const void *w1, const void *w2,
                         const void *w3);
/* tok_embeddings [vocab][dim] (emb_type), final_norm [dim], output [vocab][dim]. */
int holo_model_set_globals(void *model, const void *tok_embeddings, const float *final_norm, const void *output);
/* One position (llm_forward with n_tokens = 1): token at the current position,
 * position + 1; logits (host, vocab floats) copied out when not NULL. */
int holo_model_forward(void *model, int token, float *logits);
/* Prompt pass: tokens[0..n) at the positions pos .. pos+n-1 (llm_forward over
 * a prompt, llm.c:1049), position + n.  Each layer's projections over the n
 * rows are one tensor-core matmul (M = n, cuda_matmul_quant_batched's
 * arithmetic), the attention causal over the cache.  A batched model takes
 * tokens[batch][n] and passes all batch * n rows together.  One GPU,
 * HOLO_ACT_Q8 at batch 1, Q8_0/Q4_0/Q4_K layer matrices, head_dim
 * 64/128/256, n_heads / n_kv_heads <= 16; else
 * HOLO_E_UNSUPPORTED.  logits (host, [batch][vocab] floats) of each
 * sequence's last position when not NULL. */
int holo_model_prefill(void *model, const int *tokens, int n, float *logits);
/* How holo_model_generate / holo_model_generate_batch run the prompt before
 * its last token: 1 (default) holo_model_prefill's row passes where
 * supported, 0 one position a step. */
int holo_model_set_prompt_mode(void *model, int rows);
/* Replace the current logits (vocab host floats), e.g. to sample logits
 * computed elsewhere. */
int holo_model_load_logits(void *model, const float *logits);
/* Append a token to the repetition-penalty history (ctx->tokens). */
int holo_model_push_token(void *model, int token);
/* llm_sample on the current logits and history with the uniform draw r
 * ((float)rand() / RAND_MAX in the reference); returns the token, -1 on error.
 * Unlike the reference, the logits are left unmodified (temperature and
 * penalty are applied to a copy). */
int holo_model_sample(void *model, const holo_sampler_desc *s, float r);
/* llm_generate without tokenizer and EOS: reset, prefill the prompt, then
 * n_new sample + forward steps, all as graph replays; srand(seed) and one
 * rand() per sampled token when temperature != 0.  out[n_new]; returns n_new
 * or -1. */
int holo_model_generate(void *model, const int *prompt, int n_prompt, int n_new, const holo_sampler_desc *s,
                        int seed, int *out);
/* Replays n more steps of the last holo_model_generate's graph without
 * synchronising (for timing); the sampled tokens past n_new are discarded. */
int holo_model_launch_steps(void *model, int n_steps);
/* Diagnostics: a working vector of the last layer of the one-launch-per-op
 * graph (HOLO_STEP=graph, or head_dim 64/256) after a forward, copied to the
 * host: 0 x (residual stream, dim), 1 q|k|v (q rotated, k before rotation,
 * q_dim + 2*kv_dim), 2 attention output, 3 SwiGLU output (ffn_dim), 4 logits.
 * Returns the length, or -1.  The persistent step kernel keeps its vectors
 * elsewhere; there only the logits (4) are current. */
int holo_model_debug_vector(void *model, int which, float *dst);
int holo_model_pos(void *model);
/* Device time of the last holo_model_generate: prefill (the steps before the
 * first draw) and decode (n_new steps of forward + sample), in ms. */
int holo_model_last_timing(void *model, float *prefill_ms, float *decode_ms);
/* Sharded decode (world > 1; head_dim 128): rank r holds query heads
 * [r*n_heads/world, ...) with their KV heads and cache, a 1/world slice of
 * the rows of wo, w2, w1/w3 (in 16-row bands) and output; every phase stores
 * its slice of x, the attention output, the SwiGLU output and the logits into
 * every rank's copy over NVLink, and the step's barriers span the GPUs.  Each
 * rank creates its model with the same desc (rank differing) and passes the
 * full, unsharded weights to set_layer / set_globals, which keep the rank's
 * slice.  Then the ranks exchange handles (all-gather of
 * HOLO_COMM_HANDLE_BYTES each, in rank order) and open them.  Every call that
 * runs a step (forward, generate, launch_steps) must then be made by every
 * rank with the same arguments; a rank that recorded an error (a barrier
 * time-out) leaves the group unusable -- free and recreate it on every rank.
 * No counterpart in the reference (single-device only). */
/* Batched decode (desc.batch = B > 1, one GPU): B sequences in lockstep,
 * each projection one tensor-core matmul with M = B (cuda_matmul_quant_batched's
 * kernel), attention and the sampler per sequence, own KV caches.
 * forward_batch: tokens[B] at the current position of every sequence,
 * logits[B][vocab] copied out when not NULL.  generate_batch: prompts
 * [B][n_prompt] (equal lengths), llm_generate per sequence with seeds[B]
 * (srand(seed), one rand() per draw when T != 0), out[B][n_new]; returns n_new
 * or -1.  The step is a CUDA graph (prompt steps skip the output matrix and
 * the sampler).  No counterpart in the reference (batch 1 only). */
int holo_model_forward_batch(void *model, const int *tokens, float *logits);
int holo_model_generate_batch(void *model, const int *prompts, int n_prompt, int n_new, const holo_sampler_desc *s,
                              const int *seeds, int *out);

#define HOLO_COMM_HANDLE_BYTES 128
/* The rows desc->rank holds (host only, no device needed): ranges[10] =
 * first and count of query heads, KV heads, rows of wo/w2, SwiGLU outputs
 * (rows of w1/w3; whole 16-row bands), rows of output. */
int holo_model_shard(const holo_model_desc *desc, int *ranges);
int holo_model_comm_handle(void *model, void *handle);
int holo_model_open_peers(void *model, const void *handles);
void holo_model_reset(void *model);
void holo_model_free(void *model);

/* Batched quantized matmul for prompt processing (no counterpart in the
 * reference, whose prefill runs llm_forward one token at a time,
 * src/ai/llm.c:1049): Y[M][N] = X[M][K] . W^T on the tensor cores, W an N x K
 * Q8_0, Q4_0 or Q4_K weight from cuda_upload_quant (any N; K a whole number
 * of tiled units: 128 values for Q8_0, 256 for Q4_0/Q4_K), X fp32.  Up to 16
 * rows of X run on the CUDA cores (each weight unit read once for all rows,
 * the Q8 matvec's integer block dots per row).
 * X is quantized to Q8 per 32-block as the matvecs do; the dequantized
 * activations and weights are rounded to fp16 and multiplied with fp32
 * accumulation.  Device pointers; HOLO_STATUS_OK or an error status. */
int cuda_matmul_quant_batched(float *Y, const void *W, const float *X, int M, int N, int K);

/* Seeded synthetic weights on the device: rows x cols values N(0, std) from a
 * counter-based generator, written to dst as raw GGUF blocks of ggml_type
 * (0 F32, 1 F16 plain values; 8 Q8_0, 2 Q4_0, 12 Q4_K round-to-nearest), the
 * layout holo_model_set_layer and the reference loader read.  No counterpart
 * in the reference (it has no f32 -> Q8_0/Q4_0/Q4_K quantizer). */
int cuda_synth_weights(void *dst, int ggml_type, int rows, int cols, unsigned long long seed, float std);

/* ---- tokenizer (host; replaces llm_tokenize, src/ai/llm.c:178-221) ----------
 * The reference's greedy longest-match tokenizer with the same output: at
 * each position the longest vocabulary string that prefixes the remaining
 * text (the lowest index among equal strings; empty and NULL entries never
 * match), else the byte's fallback -- the first "<0xNN>" token, else the
 * first token equal to the byte's GPT-2 byte-level string as
 * find_byte_token builds it (llm.c:113-175), else unk_token -- one byte at a
 * time.  The reference rescans the vocabulary at every position; here it is a
 * byte trie built once by holo_tokenizer_create (which keeps no pointer into
 * vocab: the strings may be freed afterwards; NULL for vocab_size < 0, a NULL
 * vocab with vocab_size > 0, 2 GiB or more of token strings, or no memory).
 * holo_tokenize mirrors llm_tokenize(ctx, text, tokens, max_tokens, add_bos):
 * bos_token first when add_bos and max_tokens > 0, at most max_tokens ids,
 * returns the count; -1 for a NULL tokenizer or text, or NULL tokens with
 * max_tokens > 0.  No CUDA involved; a tokenizer may be used from several
 * threads at once. */
typedef struct holo_tokenizer holo_tokenizer;
holo_tokenizer *holo_tokenizer_create(const char *const *vocab, int vocab_size, int bos_token, int unk_token);
int holo_tokenize(const holo_tokenizer *t, const char *text, int *tokens, int max_tokens, int add_bos);
void holo_tokenizer_free(holo_tokenizer *t);

/* ---- CUDA graphs of the library stream --------------------------------------
 * The reference launches every op separately on the legacy stream
 * (src/ai/llm_cuda.c:558-946, ~13 launches per layer).  Calls made between
 * cuda_capture_begin and cuda_capture_end are recorded, not run, and come
 * back as one replayable graph.  Only launch-only calls may be captured
 * (no cuda_memcpy_h2d/d2h, cuda_argmax, cuda_vec_dot, cuda_upload_quant);
 * call each captured op once outside capture first so its one-time set-up
 * is done. */
int cuda_capture_begin(void);             /* 0 on success */
void *cuda_capture_end(void);             /* executable graph, NULL on failure */
void cuda_graph_launch(void *graph);      /* enqueue one replay on the library stream */
void cuda_graph_free(void *graph);

#ifdef __cplusplus
}
#endif

#endif /* HOLO_B200_H */
