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
#define HOLO_OK               0
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

/* ---- matvec without allocation ------------------------------------------------
 * No counterpart in the reference.  dst = M . v like cuda_matvec (no residual)
 * for a tiled weight M from cuda_upload_quant, but its split-K scratch is
 * static device memory (file-scope arrays found with cudaGetSymbolAddress),
 * so the call allocates and frees nothing: for callers that must not touch
 * the allocator after set-up.  Limits: out_dim <= 262144 (8192 row-blocks);
 * the grid is capped at 296 CTAs.  Runs on the thread's cuda_set_stream
 * stream, else the library stream if the device is initialised, else the
 * legacy default stream.  Every call clears the counters it uses first.
 * The scratch is shared by all calls on a device: overlapping calls (other
 * streams or threads) race.  Returns 0, or the error code it also records
 * (HOLO_E_ARG, HOLO_E_UNSUPPORTED for the row limit, a CUDA error). */
int cuda_matvec_noalloc(float *dst, const void *M, const float *v, int out_dim, int in_dim,
                        int ggml_type, int act_mode);

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
void cuda_set_stream(void *stream);
/* Select device `local_rank` for this thread and initialise it (one process
 * or thread per GPU); cuda_init() is cuda_init_rank(0, 1). */
int cuda_init_rank(int local_rank, int world_size);
/* Number of SMs of the current device (grid sizing). */
int cuda_sm_count(void);

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
