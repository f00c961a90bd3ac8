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

bool holo_matvec_launch(const void *M, const WeightInfo &wi, const MvLaunch &L, cudaStream_t st);
