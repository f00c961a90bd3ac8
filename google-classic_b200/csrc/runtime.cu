// runtime.cu -- per-device state, memory, streams, status and the registry of
// repacked weights.  Replaces the global state and memory helpers of the
// reference op library (src/ai/cuda_ops.cu:83-233).
#include "holo_common.cuh"

#include <mutex>
#include <unordered_map>
#include <string>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace {

constexpr int kMaxDevices = 16;
HoloDevice g_dev[kMaxDevices];
std::mutex g_dev_mu;
thread_local cudaStream_t t_stream_override = nullptr;

std::mutex g_status_mu;
int g_status = 0;
std::string g_status_what;

std::mutex g_reg_mu;
std::unordered_map<const void *, WeightInfo> g_registry;

int g_act_mode = -1;
int g_q4k_layout = -1;
int g_pdl = -1;

int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) d = 0;
    return d;
}

bool init_device(HoloDevice &D, int id) {
    D.id = id;
    if (cudaSetDevice(id) != cudaSuccess) return false;
    if (cudaGetDeviceProperties(&D.prop, id) != cudaSuccess) return false;
    D.sms = D.prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&D.stream, cudaStreamNonBlocking) != cudaSuccess) return false;
    if (cudaStreamCreateWithFlags(&D.copy_stream, cudaStreamNonBlocking) != cudaSuccess) return false;
    if (cudaMalloc(&D.mv_partials, sizeof(float) * MV_MAX_CTAS * 2 * 32) != cudaSuccess) return false;
    if (cudaMalloc(&D.mv_counters, sizeof(int) * MV_MAX_ROWBLOCKS) != cudaSuccess) return false;
    if (cudaMalloc(&D.mvb_counters, sizeof(int) * MVB_MAX_GROUPS) != cudaSuccess) return false;
    if (cudaMalloc(&D.status, sizeof(int) * 4) != cudaSuccess) return false;
    if (cudaMalloc(&D.reduce_buf, 65536) != cudaSuccess) return false;
    if (cudaMallocHost(&D.pinned, 65536) != cudaSuccess) return false;
    cudaMemset(D.mv_counters, 0, sizeof(int) * MV_MAX_ROWBLOCKS);
    cudaMemset(D.mvb_counters, 0, sizeof(int) * MVB_MAX_GROUPS);
    cudaMemset(D.status, 0, sizeof(int) * 4);
    if (cudaDeviceSynchronize() != cudaSuccess) return false;
    D.ready = true;
    return true;
}

}  // namespace

HoloDevice *holo_dev() {
    int id = current_device();
    if (id < 0 || id >= kMaxDevices) return nullptr;
    HoloDevice &D = g_dev[id];
    if (!D.ready) {
        std::lock_guard<std::mutex> lk(g_dev_mu);
        if (!D.ready && !init_device(D, id)) {
            holo_set_status(HOLO_E_NOMEM, "device initialisation failed");
            return nullptr;
        }
    }
    return &D;
}

void *holo_tmp(size_t bytes) {
    HoloDevice *D = holo_dev();
    if (!D) return nullptr;
    if (D->tmp_bytes < bytes) {
        cudaStreamSynchronize(D->stream);
        if (D->tmp) cudaFree(D->tmp);
        D->tmp = nullptr;
        D->tmp_bytes = 0;
        size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
        if (cudaMalloc(&D->tmp, want) != cudaSuccess) {
            cudaGetLastError();
            holo_set_status(HOLO_E_NOMEM, "scratch allocation");
            return nullptr;
        }
        D->tmp_bytes = want;
    }
    return D->tmp;
}

cudaStream_t holo_stream() {
    if (t_stream_override) return t_stream_override;
    HoloDevice *D = holo_dev();
    return D ? D->stream : nullptr;
}

cudaStream_t holo_stream_if_ready() {
    if (t_stream_override) return t_stream_override;
    int id = current_device();
    if (id >= 0 && id < kMaxDevices && g_dev[id].ready) return g_dev[id].stream;
    return nullptr;
}

void holo_set_status(int code, const char *what) {
    std::lock_guard<std::mutex> lk(g_status_mu);
    if (g_status == 0 && code != 0) {
        g_status = code;
        g_status_what = what ? what : "";
        if (getenv("HOLO_VERBOSE")) fprintf(stderr, "holo: status %d (%s)\n", code, g_status_what.c_str());
    }
}

bool holo_check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        holo_set_status((int)e, what);
        return false;
    }
    return true;
}

bool holo_registry_find(const void *ptr, WeightInfo *out) {
    std::lock_guard<std::mutex> lk(g_reg_mu);
    auto it = g_registry.find(ptr);
    if (it == g_registry.end()) return false;
    if (out) *out = it->second;
    return true;
}
void holo_registry_add(const void *ptr, const WeightInfo &info) {
    std::lock_guard<std::mutex> lk(g_reg_mu);
    g_registry[ptr] = info;
}
bool holo_registry_remove(const void *ptr) {
    std::lock_guard<std::mutex> lk(g_reg_mu);
    return g_registry.erase(ptr) > 0;
}

int holo_act_mode() {
    if (g_act_mode < 0) {
        const char *e = getenv("HOLO_ACT");
        g_act_mode = (e && (strcmp(e, "f32") == 0 || strcmp(e, "F32") == 0)) ? HOLO_ACT_F32 : HOLO_ACT_Q8;
    }
    return g_act_mode;
}
int holo_pdl() {
    if (g_pdl < 0) {
        const char *e = getenv("HOLO_PDL");
        g_pdl = (e && e[0] == '1') ? 1 : 0;
    }
    return g_pdl;
}
int holo_q4k_layout() {
    if (g_q4k_layout < 0) {
        const char *e = getenv("HOLO_Q4K_LAYOUT");
        g_q4k_layout = (e && strcmp(e, "ggml") == 0) ? HOLO_Q4K_GGML : HOLO_Q4K_REF;
    }
    return g_q4k_layout;
}

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

int cuda_last_status(void) {
    HoloDevice *D = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) == cudaSuccess && n > 0) {
        int id = current_device();
        if (id >= 0 && id < kMaxDevices && g_dev[id].ready) D = &g_dev[id];
    }
    if (D) {
        int dev_status = 0;
        cudaError_t e = cudaStreamSynchronize(D->stream);
        if (e != cudaSuccess) holo_set_status((int)e, "stream synchronise");
        if (cudaMemcpy(&dev_status, D->status, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess &&
            dev_status != 0)
            holo_set_status(dev_status, "kernel bounded wait timed out");
    }
    if (n > 0) {
        int na_status = holo_noalloc_collect_status(current_device(), false);
        if (na_status != 0) holo_set_status(na_status, "cuda_matvec_noalloc: kernel bounded wait timed out");
    }
    std::lock_guard<std::mutex> lk(g_status_mu);
    return g_status;
}
const char *cuda_last_status_string(void) {
    std::lock_guard<std::mutex> lk(g_status_mu);
    return g_status_what.c_str();
}
void cuda_clear_status(void) {
    {
        std::lock_guard<std::mutex> lk(g_status_mu);
        g_status = 0;
        g_status_what.clear();
    }
    int id = current_device();
    if (id >= 0 && id < kMaxDevices && g_dev[id].ready) {
        // a launch that gave up (bounded wait) may leave split-K counters raised
        cudaStreamSynchronize(g_dev[id].stream);
        cudaMemset(g_dev[id].status, 0, sizeof(int));
        cudaMemset(g_dev[id].mv_counters, 0, sizeof(int) * MV_MAX_ROWBLOCKS);
        cudaMemset(g_dev[id].mvb_counters, 0, sizeof(int) * MVB_MAX_GROUPS);
        cudaDeviceSynchronize();
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) == cudaSuccess && n > 0) holo_noalloc_collect_status(id, true);
    cudaGetLastError();
}

void cuda_set_pdl(int on) { g_pdl = on ? 1 : 0; }
int cuda_get_pdl(void) { return holo_pdl(); }
void cuda_set_act_mode(int mode) { g_act_mode = (mode == HOLO_ACT_F32) ? HOLO_ACT_F32 : HOLO_ACT_Q8; }
int cuda_get_act_mode(void) { return holo_act_mode(); }
void cuda_set_q4k_layout(int layout) { g_q4k_layout = (layout == HOLO_Q4K_GGML) ? HOLO_Q4K_GGML : HOLO_Q4K_REF; }
int cuda_get_q4k_layout(void) { return holo_q4k_layout(); }

void *cuda_get_stream(void) { return (void *)holo_stream(); }

int cuda_capture_begin(void) {
    cudaStream_t st = holo_stream();
    if (!st) return -1;
    cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) { holo_set_status((int)e, "cuda_capture_begin"); return -1; }
    return 0;
}

void *cuda_capture_end(void) {
    cudaStream_t st = holo_stream();
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (e != cudaSuccess || !g) { holo_set_status((int)e, "cuda_capture_end"); return nullptr; }
    cudaGraphExec_t ex = nullptr;
    e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) { holo_set_status((int)e, "cuda_capture_end: instantiate"); return nullptr; }
    return (void *)ex;
}

void cuda_graph_launch(void *graph) {
    if (!graph) { holo_set_status(HOLO_E_ARG, "cuda_graph_launch: NULL graph"); return; }
    HOLO_CUDA_TRY(cudaGraphLaunch((cudaGraphExec_t)graph, holo_stream()), "cuda_graph_launch");
}

void cuda_graph_free(void *graph) {
    if (graph) cudaGraphExecDestroy((cudaGraphExec_t)graph);
}
void cuda_set_stream(void *stream) { t_stream_override = (cudaStream_t)stream; }

int cuda_init_rank(int local_rank, int world_size) {
    (void)world_size;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        fprintf(stderr, "CUDA: No CUDA devices found\n");
        return -1;
    }
    if (local_rank < 0 || local_rank >= n) {
        holo_set_status(HOLO_E_ARG, "cuda_init_rank: no such device");
        return -1;
    }
    if (cudaSetDevice(local_rank) != cudaSuccess) return -1;
    return holo_dev() ? 0 : -1;
}

int cuda_init(void) { return cuda_init_rank(0, 1); }

void cuda_cleanup(void) {
    int id = current_device();
    if (id < 0 || id >= kMaxDevices) return;
    HoloDevice &D = g_dev[id];
    if (!D.ready) return;
    cudaDeviceSynchronize();
    cudaStreamDestroy(D.stream);
    cudaStreamDestroy(D.copy_stream);
    cudaFree(D.mv_partials);
    cudaFree(D.mv_counters);
    cudaFree(D.mvb_counters);
    cudaFree(D.status);
    cudaFree(D.reduce_buf);
    cudaFreeHost(D.pinned);
    if (D.tmp) cudaFree(D.tmp);
    D = HoloDevice();
    std::lock_guard<std::mutex> lk(g_reg_mu);
    g_registry.clear();
}

bool cuda_available(void) {
    int id = current_device();
    return id >= 0 && id < kMaxDevices && g_dev[id].ready;
}

void cuda_print_info(void) {
    if (!cuda_available()) { printf("CUDA: Not initialized\n"); return; }
    HoloDevice *D = holo_dev();
    printf("CUDA Device: %s\n", D->prop.name);
    printf("  Compute capability: %d.%d\n", D->prop.major, D->prop.minor);
    printf("  Total memory: %.2f GB\n", D->prop.totalGlobalMem / (1024.0 * 1024.0 * 1024.0));
    printf("  SM count: %d\n", D->prop.multiProcessorCount);
    printf("  Max threads/block: %d\n", D->prop.maxThreadsPerBlock);
    printf("  Warp size: %d\n", D->prop.warpSize);
}

int cuda_get_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

size_t cuda_get_free_memory(void) {
    size_t f = 0, t = 0;
    if (cudaMemGetInfo(&f, &t) != cudaSuccess) return 0;
    return f;
}

const char *cuda_get_device_name(void) {
    if (!cuda_available()) return "No device";
    return holo_dev()->prop.name;
}

int cuda_sm_count(void) {
    HoloDevice *D = holo_dev();
    return D ? D->sms : 0;
}

void *cuda_malloc(size_t size) {
    if (!holo_dev()) return nullptr;
    void *p = nullptr;
    if (cudaMalloc(&p, size) != cudaSuccess) {
        cudaGetLastError();
        holo_set_status(HOLO_E_NOMEM, "cuda_malloc");
        return nullptr;
    }
    return p;
}

void cuda_free(void *ptr) {
    if (!ptr) return;
    holo_registry_remove(ptr);
    // work still queued on the library stream may read ptr
    cudaStreamSynchronize(holo_stream());
    HOLO_CUDA_TRY(cudaFree(ptr), "cuda_free");
}

void cuda_memcpy_h2d(void *dst, const void *src, size_t size) {
    cudaStream_t st = holo_stream();
    HOLO_CUDA_TRY(cudaMemcpyAsync(dst, src, size, cudaMemcpyHostToDevice, st), "cuda_memcpy_h2d");
    HOLO_CUDA_TRY(cudaStreamSynchronize(st), "cuda_memcpy_h2d");
}

void cuda_memcpy_d2h(void *dst, const void *src, size_t size) {
    cudaStream_t st = holo_stream();
    HOLO_CUDA_TRY(cudaMemcpyAsync(dst, src, size, cudaMemcpyDeviceToHost, st), "cuda_memcpy_d2h");
    HOLO_CUDA_TRY(cudaStreamSynchronize(st), "cuda_memcpy_d2h");
}

void cuda_memcpy_h2d_stream(void *dst, const void *src, size_t size) {
    HOLO_CUDA_TRY(cudaMemcpyAsync(dst, src, size, cudaMemcpyHostToDevice, holo_stream()), "cuda_memcpy_h2d_stream");
}

void cuda_memcpy_d2h_stream(void *dst, const void *src, size_t size) {
    HOLO_CUDA_TRY(cudaMemcpyAsync(dst, src, size, cudaMemcpyDeviceToHost, holo_stream()), "cuda_memcpy_d2h_stream");
}

void cuda_memcpy_d2d(void *dst, const void *src, size_t size) {
    // stream-ordered: later kernels on the library stream see the copy
    HOLO_CUDA_TRY(cudaMemcpyAsync(dst, src, size, cudaMemcpyDeviceToDevice, holo_stream()), "cuda_memcpy_d2d");
}

void cuda_memcpy_d2d_async(void *dst, const void *src, size_t size) {
    HoloDevice *D = holo_dev();
    if (!D) return;
    HOLO_CUDA_TRY(cudaMemcpyAsync(dst, src, size, cudaMemcpyDeviceToDevice, D->copy_stream), "cuda_memcpy_d2d_async");
}

void cuda_memcpy_d2h_async(void *dst, const void *src, size_t size) {
    HoloDevice *D = holo_dev();
    if (!D) return;
    HOLO_CUDA_TRY(cudaMemcpyAsync(dst, src, size, cudaMemcpyDeviceToHost, D->copy_stream), "cuda_memcpy_d2h_async");
}

void cuda_memset(void *ptr, int value, size_t size) {
    HOLO_CUDA_TRY(cudaMemsetAsync(ptr, value, size, holo_stream()), "cuda_memset");
}

void cuda_sync(void) {
    HOLO_CUDA_TRY(cudaStreamSynchronize(holo_stream()), "cuda_sync");
    HOLO_CUDA_TRY(cudaDeviceSynchronize(), "cuda_sync");
}

void cuda_sync_copy(void) {
    HoloDevice *D = holo_dev();
    if (D) HOLO_CUDA_TRY(cudaStreamSynchronize(D->copy_stream), "cuda_sync_copy");
}

}  // extern "C"
