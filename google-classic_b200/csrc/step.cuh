// step.cuh -- arguments of the persistent decode-step kernels (step.cu), built
// by the model object (decode.cu).
#pragma once
#include "holo_common.cuh"
#include "sampler.cuh"

constexpr int STEP_MAX_RANKS = 8;

struct StepLayer {
    const uint8_t *wqkv, *wo, *w13, *w2;
    const float *attn_norm, *ffn_norm;
};

// an L2 prefetch of a byte range, split evenly over the CTAs
struct StepPrefetch {
    const uint8_t *ptr;
    unsigned long long bytes;
};
constexpr int STEP_PF_MAX = 4;            // prefetch ranges per phase

// The vectors passed between phases (x, the QKV output, the attention
// output, the SwiGLU output, the logits) are "LL" vectors: one 64-bit word per
// element, the float in the low half and the epoch of the phase that wrote it
// in the high half.  A single 8-byte store publishes a value and its
// readiness together, so readers need neither fences nor grid barriers: they
// poll the words they need until the epochs match.
typedef unsigned long long StepWord;

// Row sharding over `world` GPUs (rank `rank`): this rank holds query heads
// [h0, h0 + n_heads) and their KV heads, rows [d0, d0 + dim_loc) of Wo and
// W2, outputs [f0, f0 + ffn_loc) of the SwiGLU, rows [v0, v0 + vocab_loc) of
// the output matrix.  Every rank keeps full copies of x, the attention
// output, the SwiGLU output and the logits; each phase stores its slice into
// every rank's copy (peer stores over NVLink, LL words).  world == 1: the
// copies are this rank's only.
struct StepArgs {
    int n_layers, dim, hd, ffn, vocab, max_seq;
    int n_heads, n_kv_heads, h0;          // local heads, first global head
    int n_heads_g;                        // all heads (Wo's input is every rank's attention output)
    int dim_loc, d0, ffn_loc, f0, vocab_loc, v0;
    float eps, rope_base;
    int out_type, emb_f16;
    int rope_mode;                        // HOLO_ROPE_HALF / HOLO_ROPE_ADJACENT
    const StepLayer *layers;              // device array [n_layers] (this rank's shards)
    const void *emb;
    const float *final_norm;
    const uint8_t *out_w;
    StepWord *qkv;                        // LL, local heads' q, k, v
    float *logits;                        // plain copy of the logits (sampler, host)
    void *kc, *vc;                        // [layer][max_seq][local kv_dim]
    float *att_part;                      // [local heads][max_splits][hd + 4]
    int *att_cnt;                         // [local heads], zero between phases
    int per_split, max_splits;
    int *pos, *seq, *hist, *nhist, *out_tokens, *last;
    const float *rvals;
    float *probs, *kept_p;
    int *kept_idx;
    holo_dec::SampleArgs sa;
    int sample;                           // run the sampler (generation steps)
    const StepPrefetch *prefetch;         // [phases][STEP_PF_MAX]
    unsigned long long *bar;              // [1] launches of the layers kernel, [3] of the output kernel
    int *status;
    int grid;
    int mv_depth;                         // weight units in flight per warp (set per kernel at launch)
    int world, rank;
    // LL vectors of every rank (index rank: this rank's own)
    StepWord *px[STEP_MAX_RANKS], *patt[STEP_MAX_RANKS], *ph[STEP_MAX_RANKS], *plog[STEP_MAX_RANKS];
};

// phases of one step: embed, 5 per layer, output matrix
__host__ __device__ inline int step_phases(int n_layers) { return 2 + 5 * n_layers; }

// launch one step (the two persistent kernels); false with the status set on error
bool holo_step_launch(const StepArgs &a, int layer_type, int act, int kv_f16, cudaStream_t st);
