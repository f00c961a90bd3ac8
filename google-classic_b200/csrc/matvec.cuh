// matvec.cuh -- launch interface of the tiled matvec (matvec.cu) for the
// other modules of the library (the fused decode step).
#pragma once
#include "holo_common.cuh"

enum { MV_EPI_STORE = 0, MV_EPI_ADD = 1, MV_EPI_SILU_MUL = 2 };

struct MvLaunch {
    const float *x = nullptr;         // fp32 activations [in_dim]
    float *y = nullptr;               // output [out_dim] (SILU_MUL: [out_dim/2])
    const float *residual = nullptr;  // MV_EPI_ADD: y = residual + W.x (may alias y)
    const float *norm_w = nullptr;    // non-NULL: x := rmsnorm(x) * norm_w in the prologue
    float eps = 1e-5f;
    int act = HOLO_ACT_Q8;
    int epi = MV_EPI_STORE;
    bool pdl = false;                 // programmatic dependent launch (graph step)
    float *partials = nullptr;        // split-K scratch (NULL: the device's)
    int *counters = nullptr;
};

// Where a launch finds its scratch and limits: partials [max_ctas][2][32] f32,
// counters [max_rowblocks] i32 (zero between launches), the device status word.
struct MvScratch {
    float *partials = nullptr;
    int *counters = nullptr;
    int *status = nullptr;
    int sms = 0;
    int max_ctas = 0;
    int max_rowblocks = 0;
};

// launch on the current device's state (initialises it on first use)
bool holo_matvec_launch(const void *M, const WeightInfo &wi, const MvLaunch &L, cudaStream_t st);
// one-time set-up (kernel attributes) of the variant a launch of L on wi uses;
// call before capturing such a launch into a graph
bool holo_matvec_prepare(const WeightInfo &wi, const MvLaunch &L);
// launch with caller-provided scratch; touches no per-device state
bool holo_matvec_launch_with(const void *M, const WeightInfo &wi, const MvLaunch &L, cudaStream_t st,
                             const MvScratch &S);
