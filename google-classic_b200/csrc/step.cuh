// step.cuh -- arguments of the persistent decode-step kernel (step.cu), built
// by the model object (decode.cu).
#pragma once
#include "holo_common.cuh"
#include "sampler.cuh"

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

struct StepArgs {
    int n_layers, dim, n_heads, n_kv_heads, hd, ffn, vocab, max_seq;
    float eps, rope_base;
    int out_type, emb_f16;
    const StepLayer *layers;              // device array [n_layers]
    const void *emb;
    const float *final_norm;
    const uint8_t *out_w;
    float *x, *qkv, *att, *h, *logits;
    void *kc, *vc;                        // [layer][max_seq][kv_dim]
    float *att_part;                      // [n_heads][max_splits][hd + 2]
    int *att_cnt;                         // [n_heads], zero between phases
    int per_split, max_splits;
    int *pos, *seq, *hist, *nhist, *out_tokens, *last;
    const float *rvals;
    float *probs, *kept_p;
    int *kept_idx;
    holo_dec::SampleArgs sa;
    int sample;                           // run the sampler (generation steps)
    const StepPrefetch *prefetch;         // [phases][STEP_PF_MAX]
    unsigned long long *bar;              // layers kernel [0] arrivals [1] launches; output kernel [2] [3]
    int *status;
    int grid;
};

// phases of one step: embed, 5 per layer, output matrix
__host__ __device__ inline int step_phases(int n_layers) { return 2 + 5 * n_layers; }

// launch one step (the two persistent kernels); false with the status set on error
bool holo_step_launch(const StepArgs &a, int layer_type, int act, int kv_f16, cudaStream_t st);
