// noalloc.cu -- cuda_matvec_noalloc: the tiled matvec of matvec.cu with its
// split-K scratch in file-scope device arrays instead of per-device
// allocations, so the call allocates and frees nothing.
//
// Scratch (fixed at build time):
//   partials [NA_MAX_CTAS][2][32] f32  -- 296 CTAs (two per SM of a 148-SM part)
//   counters [NA_MAX_ROWBLOCKS] i32     -- 8192 row-blocks = 262144 output rows;
//                                          must be zero when a launch starts
//   status   [4] i32                    -- bounded-wait error word; starts at zero
// Set-up, once per device, done by the first call on that device: it takes
// the arrays' addresses with cudaGetSymbolAddress and clears the status word
// (so that first call should come before any stream capture).  Every call
// clears the counters of the row-blocks it uses before its launch.  All calls
// on one device share these arrays: calls that overlap in time (other streams
// or host threads) race and must not be issued.
//
// A launch whose bounded wait gives up writes HOLO_E_TIMEOUT into the status
// word; cuda_last_status collects it (holo_noalloc_collect_status) and
// cuda_clear_status resets it.
#include "holo_common.cuh"
#include "matvec.cuh"

#include <atomic>
#include <mutex>

namespace {

constexpr int NA_MAX_CTAS = 296;
constexpr int NA_MAX_ROWBLOCKS = 8192;
constexpr int NA_MAX_DEVICES = 16;

__device__ __align__(256) float g_na_partials[NA_MAX_CTAS * 2 * 32];
__device__ __align__(256) int g_na_counters[NA_MAX_ROWBLOCKS];
__device__ __align__(256) int g_na_status[4];

struct NaDevice {
    std::atomic<bool> ready{false};   // release-stored after the fields below are set
    float *partials = nullptr;
    int *counters = nullptr;
    int *status = nullptr;
    int sms = 0;
};
NaDevice g_na[NA_MAX_DEVICES];
std::mutex g_na_mu;

// Per-device set-up: symbol addresses (checked), SM count, status cleared.
NaDevice *na_device(int dev, cudaStream_t st) {
    if (dev < 0 || dev >= NA_MAX_DEVICES) return nullptr;
    NaDevice &N = g_na[dev];
    if (N.ready.load(std::memory_order_acquire)) return &N;
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (N.ready.load(std::memory_order_relaxed)) return &N;
    cudaError_t e = cudaGetSymbolAddress((void **)&N.partials, g_na_partials);
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void **)&N.counters, g_na_counters);
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void **)&N.status, g_na_status);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&N.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaMemsetAsync(N.status, 0, sizeof(int) * 4, st);
    if (e != cudaSuccess) {
        cudaGetLastError();
        holo_set_status((int)e, "cuda_matvec_noalloc: scratch set-up (cudaGetSymbolAddress)");
        return nullptr;
    }
    N.ready.store(true, std::memory_order_release);
    return &N;
}

}  // namespace

// Bounded-wait status of the static scratch on device `dev`: waits for the
// device's queued work, returns the word (0 when the no-allocation path was
// never set up there) and, with `clear`, resets it.
int holo_noalloc_collect_status(int dev, bool clear) {
    if (dev < 0 || dev >= NA_MAX_DEVICES) return 0;
    NaDevice &N = g_na[dev];
    if (!N.ready.load(std::memory_order_acquire)) return 0;
    int word = 0;
    // the call may have run on any stream of the device
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(&word, N.status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (clear && word != 0 && cudaMemset(N.status, 0, sizeof(int) * 4) != cudaSuccess) cudaGetLastError();
    return word;
}

extern "C" int cuda_matvec_noalloc(float *dst, const void *M, const float *v, int out_dim, int in_dim,
                                   int ggml_type, int act_mode) {
    WeightInfo wi;
    if (!dst || !v || !holo_registry_find(M, &wi)) {
        holo_set_status(HOLO_E_ARG, "cuda_matvec_noalloc: M is not a tiled weight from cuda_upload_quant");
        return HOLO_E_ARG;
    }
    if (wi.type != ggml_type || wi.rows != out_dim || wi.cols != in_dim) {
        holo_set_status(HOLO_E_ARG, "cuda_matvec_noalloc: type or shape differs from the uploaded weight");
        return HOLO_E_ARG;
    }
    if (act_mode != HOLO_ACT_Q8 && act_mode != HOLO_ACT_F32) {
        holo_set_status(HOLO_E_ARG, "cuda_matvec_noalloc: unknown activation mode");
        return HOLO_E_ARG;
    }
    const int nrb = wi.rows_padded / TILE_ROWS;
    if (nrb > NA_MAX_ROWBLOCKS) {
        holo_set_status(HOLO_E_UNSUPPORTED, "cuda_matvec_noalloc: more than 262144 output rows (static scratch limit)");
        return HOLO_E_UNSUPPORTED;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        holo_set_status(HOLO_E_ARG, "cuda_matvec_noalloc: no current device");
        return HOLO_E_ARG;
    }
    cudaStream_t st = holo_stream_if_ready();
    NaDevice *N = na_device(dev, st);
    if (!N) return HOLO_E_ARG;
    if (cudaMemsetAsync(N->counters, 0, sizeof(int) * (size_t)nrb, st) != cudaSuccess) {
        holo_check_launch("cuda_matvec_noalloc: counter clear");
        return cuda_last_status();
    }
    MvScratch S;
    S.partials = N->partials;
    S.counters = N->counters;
    S.status = N->status;
    S.sms = N->sms;
    S.max_ctas = NA_MAX_CTAS;
    S.max_rowblocks = NA_MAX_ROWBLOCKS;
    MvLaunch L;
    L.x = v;
    L.y = dst;
    L.act = act_mode;
    L.epi = MV_EPI_STORE;
    L.pdl = false;
    if (!holo_matvec_launch_with(M, wi, L, st, S)) return cuda_last_status() ? cuda_last_status() : HOLO_E_ARG;
    return HOLO_OK;
}

extern "C" void *cuda_matvec_noalloc_status_word(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    NaDevice *N = na_device(dev, holo_stream_if_ready());
    return N ? (void *)N->status : nullptr;
}
