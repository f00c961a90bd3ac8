// holo_common.cuh -- shared definitions of the B200 decode-path library.
//
// Block formats are GGUF's (src/ai/quant.h:43-120 of the reference engine);
// everything else here is this library's own: the per-device runtime state,
// the repacked ("tiled") weight layout, and the sm_100a PTX helpers for
// mbarriers and bulk (TMA) copies.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include "cuda_ops.h"
#include "holo_b200.h"

// library-internal spelling of success (the public header says HOLO_STATUS_OK)
#define HOLO_OK HOLO_STATUS_OK

// ---------------------------------------------------------------------------
// ggml type ids (src/ai/quant.h:20-33)
// ---------------------------------------------------------------------------
enum : int {
    GT_F32 = 0, GT_F16 = 1, GT_Q4_0 = 2, GT_Q8_0 = 8, GT_Q4_K = 12, GT_Q6_K = 14,
};

// ---------------------------------------------------------------------------
// Tiled weight layout (format version 3: units)
//
// Rows are grouped in row-blocks of 32 (padded with zero rows).  A row-block's
// K extent is cut into units of a fixed number of values (Q4_K: one 256-value
// super-block; Q4_0: eight 32-blocks; Q8_0: four 32-blocks), and units are
// stored back to back in (row-block, unit) order: unit u = rb*units_per_row + s
// starts at u * UNIT_BYTES.  Inside a unit, data is transposed so that lane r
// of a warp reads row r with unit stride between lanes:
//   head  [row][HEAD_BYTES]   Q4_K: the 16-byte super-block head (fp16 d, fp16
//                             dmin, 12 bytes of 6-bit scales/mins, quant.c
//                             packing, src/ai/quant.c:277-311);
//                             Q4_0: eight fp16 block scales; Q8_0: four
//   plane [p][row][16 B]      p = 0..7: Q4_K sub-block p / Q4_0 block p, 32
//                             nibbles (low nibble of byte l = position l, high
//                             = l+16); Q8_0 half p&1 of block p>>1, 16 int8
// A row whose block count is not a multiple of the unit's is padded with zero
// blocks (d = 0); Q4_K rows are whole units by definition.
// ---------------------------------------------------------------------------
constexpr int TILE_ROWS = 32;
constexpr int UNIT_PLANES = 8;

template <int T> struct UnitGeom;
template <> struct UnitGeom<GT_Q8_0> {
    static constexpr int BLK_ELEMS = 32, BLK_BYTES = 34, VALS = 128, BLKS32 = 4, HEAD_BYTES = 8;
    static constexpr int UNIT_BYTES = TILE_ROWS * HEAD_BYTES + UNIT_PLANES * TILE_ROWS * 16;   // 4352
};
template <> struct UnitGeom<GT_Q4_0> {
    static constexpr int BLK_ELEMS = 32, BLK_BYTES = 18, VALS = 256, BLKS32 = 8, HEAD_BYTES = 16;
    static constexpr int UNIT_BYTES = TILE_ROWS * HEAD_BYTES + UNIT_PLANES * TILE_ROWS * 16;   // 4608
};
template <> struct UnitGeom<GT_Q4_K> {
    static constexpr int BLK_ELEMS = 256, BLK_BYTES = 144, VALS = 256, BLKS32 = 8, HEAD_BYTES = 16;
    static constexpr int UNIT_BYTES = TILE_ROWS * HEAD_BYTES + UNIT_PLANES * TILE_ROWS * 16;   // 4608
};
// Q6_K: a unit is one 128-value half of a super-block (src/ai/quant.c:251-268
// walks the halves: 64 bytes of low codes, 32 of high bits, 8 scales each).
// head: fp16 d, the half's 8 int8 scales, 6 zero bytes; planes 0-3: ql[0..63]
// of the half (16 bytes each), planes 4-5: qh[0..31]; 6 planes a unit.
template <> struct UnitGeom<GT_Q6_K> {
    static constexpr int BLK_ELEMS = 256, BLK_BYTES = 210, VALS = 128, BLKS32 = 4, HEAD_BYTES = 16, PLANES = 6;
    static constexpr int UNIT_BYTES = TILE_ROWS * HEAD_BYTES + PLANES * TILE_ROWS * 16;   // 3584
};
// F16: 64 values a row a unit, plane p = values 8p..8p+7 (no head)
template <> struct UnitGeom<GT_F16> {
    static constexpr int BLK_ELEMS = 1, BLK_BYTES = 2, VALS = 64, BLKS32 = 2, HEAD_BYTES = 0;
    static constexpr int UNIT_BYTES = UNIT_PLANES * TILE_ROWS * 16;   // 4096
};

template <int T> __host__ __device__ constexpr size_t unit_head_off(int r) {
    return (size_t)r * UnitGeom<T>::HEAD_BYTES;
}
template <int T> __host__ __device__ constexpr size_t unit_plane_off(int p, int r) {
    return (size_t)TILE_ROWS * UnitGeom<T>::HEAD_BYTES + ((size_t)p * TILE_ROWS + r) * 16;
}

// units per row and bytes of the tiled copy (0: type without a tiled layout)
static inline int units_per_row(int type, int cols) {
    switch (type) {
    case GT_Q8_0: return (cols + UnitGeom<GT_Q8_0>::VALS - 1) / UnitGeom<GT_Q8_0>::VALS;
    case GT_Q4_0: return (cols + UnitGeom<GT_Q4_0>::VALS - 1) / UnitGeom<GT_Q4_0>::VALS;
    case GT_Q4_K: return cols / UnitGeom<GT_Q4_K>::VALS;
    case GT_Q6_K: return cols / UnitGeom<GT_Q6_K>::VALS;
    case GT_F16: return cols / UnitGeom<GT_F16>::VALS;
    default: return 0;
    }
}
static inline int unit_bytes(int type) {
    switch (type) {
    case GT_Q8_0: return UnitGeom<GT_Q8_0>::UNIT_BYTES;
    case GT_Q4_0: return UnitGeom<GT_Q4_0>::UNIT_BYTES;
    case GT_Q4_K: return UnitGeom<GT_Q4_K>::UNIT_BYTES;
    case GT_Q6_K: return UnitGeom<GT_Q6_K>::UNIT_BYTES;
    case GT_F16: return UnitGeom<GT_F16>::UNIT_BYTES;
    default: return 0;
    }
}

static inline int64_t gguf_row_bytes(int type, int64_t cols) {
    switch (type) {
    case GT_F32:  return cols * 4;
    case GT_F16:  return cols * 2;
    case GT_Q8_0: return (cols / 32) * 34;
    case GT_Q4_0: return (cols / 32) * 18;
    case GT_Q4_K: return (cols / 256) * 144;
    case GT_Q6_K: return (cols / 256) * 210;
    default: return -1;
    }
}
static inline int gguf_block_elems(int type) {
    switch (type) {
    case GT_Q8_0: case GT_Q4_0: return 32;
    case GT_Q4_K: case GT_Q6_K: return 256;
    default: return 1;
    }
}

// ---------------------------------------------------------------------------
// Host runtime (runtime.cu)
// ---------------------------------------------------------------------------
struct HoloDevice {
    bool ready = false;
    int id = 0;
    int sms = 0;
    cudaStream_t stream = nullptr;       // the ABI's implicit compute stream
    cudaStream_t copy_stream = nullptr;  // cuda_memcpy_*_async
    cudaDeviceProp prop{};
    // split-K fix-up scratch of the tiled matvec (zeroed once; self-cleaning)
    float *mv_partials = nullptr;        // [MV_MAX_CTAS][2][32]
    int *mv_counters = nullptr;          // [MV_MAX_ROWBLOCKS]
    int *mvb_counters = nullptr;         // [MVB_MAX_GROUPS] of the few-row matmul (zeroed once; self-cleaning)
    int *status = nullptr;               // device-side error word (bounded waits)
    // small persistent buffers for reductions that return to the host
    void *reduce_buf = nullptr;          // 64 KB
    void *pinned = nullptr;              // 64 KB pinned host buffer
    void *tmp = nullptr;                 // growable scratch of the ABI helpers
    size_t tmp_bytes = 0;
};
constexpr int MV_MAX_CTAS = 1024;
constexpr int MV_MAX_ROWBLOCKS = 1 << 16;
constexpr int MVB_MAX_GROUPS = 1 << 14;   // row groups (8 row-blocks) of one few-row matmul
constexpr int MVB_MAX_M = 16;             // activation rows the few-row matmul takes

HoloDevice *holo_dev();                  // current device's state, initialised on demand
cudaStream_t holo_stream();
// the stream calls use without initialising anything: the thread's override,
// else the device's library stream if it exists, else the legacy stream (0)
cudaStream_t holo_stream_if_ready();
void holo_set_status(int code, const char *what);   // sticky host-side status
// noalloc.cu: the static scratch's bounded-wait word on device `dev` (0 when
// never set up), reset afterwards when `clear`
int holo_noalloc_collect_status(int dev, bool clear);
bool holo_check_launch(const char *what);           // cudaGetLastError -> status
// Scratch of at least `bytes` on the current device for ABI helpers whose
// reference signature has no workspace argument (grows; synchronises then).
void *holo_tmp(size_t bytes);

// ops.cu: every row of a raw GGUF embedding table (Q8_0, Q4_0, Q4_K, Q6_K)
// dequantized into dst [rows][dim] as the reference's get_embedding decodes it
bool holo_embedding_table_f32(float *dst, const void *table, int type, int rows, int dim, bool ggml_q4k,
                              cudaStream_t st);

// prompt_attn.cu: causal prompt attention on the tensor cores (fp16 cache,
// head_dim 128); see the file for the layout of the arguments
bool holo_prompt_attn_tc(float *att, const float *qkv, const __half *kc, const __half *vc, const int *pos_p, int M,
                         int nseq, int n_heads, int group, int kv_dim, size_t qkv_bs, size_t att_bs, size_t kv_bs,
                         float sqrt_hd, int *status, cudaStream_t st);

// Registry of repacked weights: device pointer -> geometry.
struct WeightInfo {
    int type = 0;
    int rows = 0, cols = 0;
    int rows_padded = 0;
    int units = 0;          // units per row of the tiled layout
    int q4k_layout = 0;     // layout of the source blocks before normalisation
    size_t bytes = 0;
};
bool holo_registry_find(const void *ptr, WeightInfo *out);
// repack.cu: shape check, geometry, and repack of raw device blocks into a
// caller-provided buffer of cuda_quant_tiled_bytes() bytes (no allocation)
bool holo_quant_shape_ok(int ggml_type, int rows, int cols);
WeightInfo holo_weight_info(int ggml_type, int rows, int cols, int q4k_layout);
// Y[M][N] = X[M][K] . W^T on the tensor cores for a tiled weight (prefill.cu);
// scratch NULL: the library's shared scratch, else the caller's (at least
// holo_matmul_batched_scratch bytes).  plan_rows > 0: split K as for a weight
// of that many rows (a row shard passes the whole matrix's, so each row's sum
// is cut at the same K points as on one GPU); 0: the weight's own rows.
// norm_w: X is the un-normalized activation and each row is RMS-normalized
// with these weights on the way in (bit-identical to bt_rmsnorm_kernel
// followed by the matmul; M > MVB_MAX_M only).  resid: the product is also
// added into resid[M][N] (the residual stream), fused into the K-split
// reduction when there is one -- bit-identical to an add after; Y is then
// scratch (M > MVB_MAX_M only).
bool holo_matmul_batched(float *Y, const void *W, const WeightInfo &wi, const float *X, int M, cudaStream_t st,
                         void *scratch, size_t scratch_bytes, int plan_rows = 0, const float *norm_w = nullptr,
                         float norm_eps = 0.0f, float *resid = nullptr);
size_t holo_matmul_batched_scratch(const WeightInfo &wi, int M, int plan_rows = 0);
// the batched matmul's weights: rows a multiple of this (one MMA tile)
constexpr int PF_ROWS_ALIGN = 128;
// Y[M][N] = X[M][K] . W^T for M <= MVB_MAX_M on the CUDA cores (matvec_batch.cu):
// each weight unit read once and dotted with every Q8-quantized row;
// scratch: at least holo_matmul_few_scratch bytes (split-K partials)
bool holo_matmul_few(float *Y, const void *W, const WeightInfo &wi, const float *X, int M, cudaStream_t st,
                     void *scratch, size_t scratch_bytes);
size_t holo_matmul_few_scratch(const WeightInfo &wi, int M);
bool holo_repack_to(void *dst, const void *dev_blocks, int ggml_type, int rows, int cols, int q4k_layout,
                    cudaStream_t st);
void holo_registry_add(const void *ptr, const WeightInfo &info);
bool holo_registry_remove(const void *ptr);

int holo_act_mode();        // HOLO_ACT_F32 / HOLO_ACT_Q8 (env HOLO_ACT, cuda_set_act_mode)
int holo_q4k_layout();      // HOLO_Q4K_REF / HOLO_Q4K_GGML (env HOLO_Q4K_LAYOUT)
int holo_pdl();             // programmatic dependent launch of tiled matvecs (env HOLO_PDL)

// matvec dispatch (matvec.cu / matvec_raw.cu)
void holo_matvec_tiled(float *dst, const void *M, const WeightInfo &wi, const float *v,
                       int out_dim, int in_dim, int act_mode, const float *residual,
                       cudaStream_t st);
void holo_matvec_raw(float *dst, const void *M, int type, const float *v,
                     int out_dim, int in_dim, int act_mode, int q4k_layout, cudaStream_t st,
                     const float *residual);

#define HOLO_CUDA_TRY(call, what)                                                     \
    do {                                                                              \
        cudaError_t e_ = (call);                                                      \
        if (e_ != cudaSuccess) { holo_set_status((int)e_, what); }                    \
    } while (0)

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
#ifdef __CUDACC__

// Bounded waits: give up after this many nanoseconds of %globaltimer.
constexpr unsigned long long HOLO_WAIT_LIMIT_NS = 1000000000ull;   // 1 s

__device__ __forceinline__ unsigned long long holo_globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" :: "r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }"
                 :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Wait for phase `parity` of `bar` to complete, for at most HOLO_WAIT_LIMIT_NS.
// On time-out, records `code` in *status and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *status, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    unsigned long long t0 = holo_globaltimer();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 255u && holo_globaltimer() - t0 > HOLO_WAIT_LIMIT_NS) {
            if (status) atomicExch(status, code);
            return false;
        }
    }
}

// 1-D bulk copy global -> shared, completion counted on `bar` (no multicast).
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes,
                                         uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        :: "r"(smem_addr(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// named barrier among a subset of warps
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint4 lds128(const void *p) {
    return *reinterpret_cast<const uint4 *>(p);
}

// exact small-integer <-> float through the 2^23 mantissa (|v| < 2^22)
__device__ __forceinline__ float int_to_float_exact(int v) {
    return __int_as_float(v + 0x4B400000) - 12582912.0f;
}
// byte k of w (0..255) as an exact float
__device__ __forceinline__ float ubyte_to_float(uint32_t w, int k) {
    return __int_as_float(__byte_perm(w, 0x4B000000u, 0x7440u + k)) - 8388608.0f;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half((unsigned short)h16));
}

#endif  // __CUDACC__
