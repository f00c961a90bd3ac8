// matvec_multi.cu -- cuda_matvec_batch: several independent quantized matvecs
// (y_i = W_i . x_i, tiled weights of one type) in one persistent launch.
//
// A chain of single matvec launches pays, per matrix, the wait for the
// previous launch to finish, the activation copy and quantization, and the
// split-K fix-up, all on the critical path (about half of a 25 MB matvec's
// time on a B200).  Independent matvecs need none of that ordering: their
// units (32 rows x one K chunk, the layout of holo_common.cuh) form one
// sequence, problem after problem, that the CTAs split evenly (stream-K over
// all of them).  A CTA walks the problems its range touches; for each it
// stages that problem's x, quantizes it (the single kernel's prologue,
// mv_unit.cuh) and folds its units with the single kernel's unit dot, so
// every output row is computed with the same per-unit arithmetic.  Row-blocks
// cut between CTAs are finished by the last CTA to contribute (acq_rel
// counter, partials summed in CTA order: deterministic), as in matvec.cu.
// Only the first and the last row-block of a CTA's range can be cut.
//
// The weights are constant, so each warp keeps MV_L2_AHEAD units prefetched
// into L2 across problem boundaries; the next problem's activation is
// prefetched into L2 while the current one is folded.
#include "holo_common.cuh"
#include "mv_device.cuh"
#include "mv_unit.cuh"
#include "matvec.cuh"

#include <algorithm>
#include <vector>

namespace {

using namespace holo_mv;

constexpr int MM_WARPS = 8;
constexpr int MM_THREADS = MM_WARPS * 32;
constexpr int MM_DEPTH = 2;        // units in registers per warp
constexpr int MM_L2_AHEAD = 3;     // units per warp prefetched into L2 ahead of use (3-4 best measured)
constexpr int MM_MAX = 32;         // problems per launch
constexpr size_t MM_SMEM_LIMIT = 227 * 1024;

struct MmProblem {
    const uint8_t *W;
    const float *x;
    float *y;
    int rows, in_dim;
    int units;         // units per row
    int nblk32p;       // 32-blocks per row of the tiled layout
    unsigned u0;       // first unit of the problem in the launch's sequence
    unsigned rb0;      // first row-block (counter index) of the problem
};

struct MmParams {
    int n;
    unsigned total_units;
    int nctas;
    int max_nblk32p;
    int max_local_rb;
    float *partials;   // [nctas][2][32]
    int *counters;     // [sum of row-blocks], zero between launches
    int *status;
    MmProblem prob[MM_MAX];
};

__device__ __forceinline__ int mm_owner(unsigned t, unsigned T, unsigned C) { return (int)(((t + 1ull) * C - 1) / T); }
__device__ __forceinline__ unsigned mm_begin(unsigned c, unsigned T, unsigned C) {
    return (unsigned)((unsigned long long)T * c / C);
}

// the problem holding global unit u
__device__ __forceinline__ int mm_problem_of(const MmParams &p, unsigned u) {
    int i = 0;
    while (i + 1 < p.n && p.prob[i + 1].u0 <= u) ++i;
    return i;
}

// global row-block of global unit u
__device__ __forceinline__ unsigned mm_rb_of(const MmParams &p, unsigned u) {
    const MmProblem &q = p.prob[mm_problem_of(p, u)];
    return q.rb0 + (u - q.u0) / (unsigned)q.units;
}

// Row-block (global index grb, local index lrb of problem q) summed over this
// CTA's units: store it, or finish it with the other CTAs that hold part of it.
__device__ __forceinline__ void mm_complete(const MmParams &p, const MmProblem &q, int lrb, unsigned grb,
                                            unsigned U0, unsigned U1, int lane, float v) {
    const unsigned T = p.total_units, C = p.nctas;
    const unsigned tb = q.u0 + (unsigned)lrb * q.units, te = tb + q.units - 1;
    float out = v;
    if (tb < U0 || te >= U1) {
        const int c_first = mm_owner(tb, T, C), c_last = mm_owner(te, T, C);
        const int slot = tb <= U0 ? 0 : 1;   // the range's first row-block, or its last
        p.partials[((size_t)blockIdx.x * 2 + slot) * 32 + lane] = v;
        __syncwarp();
        int prev = 0;
        if (lane == 0)
            asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(prev) : "l"(&p.counters[grb]) : "memory");
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev != c_last - c_first) return;
        __syncwarp();
        out = 0.0f;
        for (int c = c_first; c <= c_last; ++c) {
            const int sl = mm_rb_of(p, mm_begin(c, T, C)) == grb ? 0 : 1;
            out += __ldcg(&p.partials[((size_t)c * 2 + sl) * 32 + lane]);
        }
        if (lane == 0) p.counters[grb] = 0;
    }
    const int row = lrb * TILE_ROWS + lane;
    if (row < q.rows) q.y[row] = out;
}

template <int TYPE, int ACT>
__global__ void __launch_bounds__(MM_THREADS, 2) mv_multi_kernel(const __grid_constant__ MmParams p) {
    constexpr int BLKS32 = UnitGeom<TYPE>::BLKS32;
    constexpr size_t UB = UnitGeom<TYPE>::UNIT_BYTES;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    // red [max_local_rb][warps][32] | aq [max_nblk32p*32] | ads [max_nblk32p] f32x2 |
    // stage (x, f32) [max_nblk32p*32] | xsum [max_nblk32p] | misc
    float *red = reinterpret_cast<float *>(smem);
    size_t o = (size_t)p.max_local_rb * MM_WARPS * 32 * 4;
    uint8_t *aq = smem + o;
    float2 *ads = reinterpret_cast<float2 *>(smem + o + (size_t)p.max_nblk32p * 32);
    o += (size_t)p.max_nblk32p * 40;
    float *xst = reinterpret_cast<float *>(smem + o);
    float *xsum = xst + (size_t)p.max_nblk32p * 32;
    o += (size_t)p.max_nblk32p * 132;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + o);
    float *wsum = reinterpret_cast<float *>(smem + o + 64);

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const unsigned T = p.total_units, C = p.nctas;
    const unsigned U0 = mm_begin(blockIdx.x, T, C), U1 = mm_begin(blockIdx.x + 1, T, C);
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }
    // the weights are constant: the first units of every warp go to L2 before
    // waiting for the kernel this one follows
    if (lane == 0) {
        for (int k = 0; k < MM_L2_AHEAD; ++k) {
            const unsigned u = U0 + warp + k * MM_WARPS;
            if (u < U1) {
                const MmProblem &q = p.prob[mm_problem_of(p, u)];
                prefetch_l2_bulk(q.W + (size_t)(u - q.u0) * UB, (uint32_t)UB);
            }
        }
    }
    __syncthreads();
    asm volatile("griddepcontrol.wait;" ::: "memory");

    unsigned par = 0;
    unsigned seg = U0;
    int pi = mm_problem_of(p, U0);
    while (seg < U1) {
        const MmProblem &q = p.prob[pi];
        const unsigned qend = q.u0 + (unsigned)q.units * (unsigned)((q.rows + TILE_ROWS - 1) / TILE_ROWS);
        const unsigned s0 = seg, s1 = min(U1, qend);
        // the next problem's activation to L2 while this one is folded
        if (tid == 32 && s1 < U1 && pi + 1 < p.n) prefetch_l2_bulk(p.prob[pi + 1].x, (uint32_t)p.prob[pi + 1].in_dim * 4u);
        // ---- prologue: x of problem q in shared memory, quantized ----
        const bool bulk = ((uintptr_t)q.x % 16) == 0;
        const uint32_t xbytes = (uint32_t)q.in_dim * 4u;
        if (bulk) {
            if (tid == 0) {
                fence_proxy_async_smem();   // the previous problem's reads of xst come first
                mbar_arrive_expect_tx(bar, xbytes);
                bulk_copy_g2s(xst, q.x, xbytes, bar);
            }
        } else {
            for (int i = tid; i < q.in_dim; i += MM_THREADS) xst[i] = __ldg(q.x + i);
        }
        Frag ring[MM_DEPTH];
#pragma unroll
        for (int k = 0; k < MM_DEPTH; ++k) {
            const unsigned u = s0 + warp + k * MM_WARPS;
            if (u < s1) load_unit<TYPE>(ring[k], q.W + (size_t)(u - q.u0) * UB, lane);
        }
        for (int i = q.in_dim + tid; i < q.nblk32p * 32; i += MM_THREADS) xst[i] = 0.0f;
        const int lrb_first = (int)((s0 - q.u0) / q.units);
        const int n_local = (int)((s1 - 1 - q.u0) / q.units) - lrb_first + 1;
        for (int i = tid; i < n_local * MM_WARPS * 32; i += MM_THREADS) red[i] = 0.0f;
        bool ok = true;
        if (bulk) {
            ok = mbar_wait_bounded(bar, par, p.status, HOLO_E_TIMEOUT);
            par ^= 1u;
        }
        if (!__syncthreads_and(ok)) return;
        act_prologue<ACT, false, MM_THREADS>(xst, nullptr, aq, ads, xsum, wsum, q.in_dim, q.nblk32p, 0.0f);

        // ---- units [s0, s1): warp w takes s0 + w, s0 + w + warps, ... ----
        const unsigned lu = s0 - q.u0 + warp;          // problem-local unit
        int rb = (int)(lu / q.units), s = (int)(lu - (unsigned)rb * q.units);
        const int dq = MM_WARPS / q.units, dr = MM_WARPS - dq * q.units;
        int cur = rb;
        float acc = 0.0f;
        for (unsigned ub = s0 + warp; ub < s1; ub += MM_DEPTH * MM_WARPS) {
#pragma unroll
            for (int k = 0; k < MM_DEPTH; ++k) {
                const unsigned u = ub + k * MM_WARPS;
                if (u >= s1) break;
                if (rb != cur) {
                    red[((cur - lrb_first) * MM_WARPS + warp) * 32 + lane] = acc;
                    acc = 0.0f;
                    cur = rb;
                }
                unit_dot<TYPE, ACT>(acc, ring[k], s * BLKS32, aq, ads, xst, xsum);
                const unsigned un = u + MM_DEPTH * MM_WARPS;
                if (un < s1) load_unit<TYPE>(ring[k], q.W + (size_t)(un - q.u0) * UB, lane);
                // L2 prefetch ahead, across the problem boundary
                const unsigned up = u + MM_L2_AHEAD * MM_WARPS;
                if (lane == 0 && up < U1) {
                    const MmProblem &r = up < qend ? q : p.prob[mm_problem_of(p, up)];
                    prefetch_l2_bulk(r.W + (size_t)(up - r.u0) * UB, (uint32_t)UB);
                }
                s += dr;
                rb += dq;
                if (s >= q.units) { s -= q.units; ++rb; }
            }
        }
        if (s0 + warp < s1) red[((cur - lrb_first) * MM_WARPS + warp) * 32 + lane] = acc;
        __syncthreads();
        for (int l = warp; l < n_local; l += MM_WARPS) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < MM_WARPS; ++w) v += red[(l * MM_WARPS + w) * 32 + lane];
            mm_complete(p, q, lrb_first + l, q.rb0 + lrb_first + l, U0, U1, lane, v);
        }
        __syncthreads();   // shared memory is the next problem's
        seg = s1;
        ++pi;
    }
}

size_t mm_smem(int max_local_rb, int max_nblk32p) {
    return (size_t)max_local_rb * MM_WARPS * 32 * 4 + (size_t)max_nblk32p * 40 + (size_t)max_nblk32p * 132 + 128;
}

template <int TYPE, int ACT>
bool mm_launch(MmParams &p, int sms, cudaStream_t st, bool pdl) {
    auto kern = mv_multi_kernel<TYPE, ACT>;
    static bool configured[16] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 16 && !configured[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MM_SMEM_LIMIT) != cudaSuccess) {
            holo_check_launch("cuda_matvec_batch: kernel attributes");
            return false;
        }
        configured[dev] = true;
    }
    // two CTAs an SM: 16 warps with their loads in flight (the loop is
    // latency-bound at one; 5.4 against 4.8 TB/s on the bench sweep)
    p.nctas = (int)std::min<unsigned>(p.total_units, 2u * (unsigned)sms);
    // row-blocks a CTA's range can touch: its units over the shortest row-block, plus the two cut ones
    int min_units = 1 << 30;
    for (int i = 0; i < p.n; ++i) min_units = std::min(min_units, p.prob[i].units);
    const unsigned per = (p.total_units + p.nctas - 1) / p.nctas;
    p.max_local_rb = (int)std::min<unsigned>(per / min_units + 2, per + 1);
    const size_t smem = mm_smem(p.max_local_rb, p.max_nblk32p);
    if (smem > MM_SMEM_LIMIT) {
        holo_set_status(HOLO_E_UNSUPPORTED, "cuda_matvec_batch: in_dim too large for shared memory");
        return false;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.nctas);
    cfg.blockDim = dim3(MM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kern, p);
    return holo_check_launch("cuda_matvec_batch launch");
}

template <int TYPE>
bool mm_dispatch(MmParams &p, int act, int sms, cudaStream_t st, bool pdl) {
    return act == HOLO_ACT_Q8 ? mm_launch<TYPE, HOLO_ACT_Q8>(p, sms, st, pdl)
                              : mm_launch<TYPE, HOLO_ACT_F32>(p, sms, st, pdl);
}

// one launch over problems idx[0..n) (one weight type, n <= MM_MAX)
bool mm_group(const int *idx, int n, float *const *dst, const void *const *M, const float *const *v,
              const WeightInfo *wi, int act, HoloDevice *D, cudaStream_t st, bool pdl) {
    MmParams p{};
    p.n = n;
    p.partials = D->mv_partials;
    p.counters = D->mv_counters;
    p.status = D->status;
    unsigned u = 0, rb = 0;
    for (int k = 0; k < n; ++k) {
        const int i = idx[k];
        MmProblem &q = p.prob[k];
        q.W = (const uint8_t *)M[i];
        q.x = v[i];
        q.y = dst[i];
        q.rows = wi[i].rows;
        q.in_dim = wi[i].cols;
        q.units = wi[i].units;
        const int nrb = wi[i].rows_padded / TILE_ROWS;
        q.nblk32p = q.units * (wi[i].type == GT_Q6_K ? UnitGeom<GT_Q6_K>::BLKS32
                                 : wi[i].type == GT_Q8_0 ? UnitGeom<GT_Q8_0>::BLKS32
                                 : wi[i].type == GT_F16 ? UnitGeom<GT_F16>::BLKS32 : UnitGeom<GT_Q4_K>::BLKS32);
        q.u0 = u;
        q.rb0 = rb;
        p.max_nblk32p = std::max(p.max_nblk32p, q.nblk32p);
        if ((unsigned long long)u + (unsigned long long)nrb * q.units >= (1ull << 31)) {
            holo_set_status(HOLO_E_UNSUPPORTED, "cuda_matvec_batch: too many units");
            return false;
        }
        u += (unsigned)nrb * q.units;
        rb += (unsigned)nrb;
    }
    if (rb > (unsigned)MV_MAX_ROWBLOCKS) {
        holo_set_status(HOLO_E_UNSUPPORTED, "cuda_matvec_batch: too many output rows in one call");
        return false;
    }
    p.total_units = u;
    if ((unsigned long long)u * (unsigned long long)D->sms >= (1ull << 32)) {
        holo_set_status(HOLO_E_UNSUPPORTED, "cuda_matvec_batch: too many units");
        return false;
    }
    switch (wi[idx[0]].type) {
    case GT_Q8_0: return mm_dispatch<GT_Q8_0>(p, act, D->sms, st, pdl);
    case GT_Q4_0: return mm_dispatch<GT_Q4_0>(p, act, D->sms, st, pdl);
    case GT_Q4_K: return mm_dispatch<GT_Q4_K>(p, act, D->sms, st, pdl);
    case GT_Q6_K: return mm_dispatch<GT_Q6_K>(p, act, D->sms, st, pdl);
    case GT_F16: return mm_launch<GT_F16, HOLO_ACT_F32>(p, D->sms, st, pdl);
    default:
        holo_set_status(HOLO_E_ARG, "cuda_matvec_batch: type has no tiled kernel");
        return false;
    }
}

}  // namespace

extern "C" int cuda_matvec_batch(int n, float *const *dst, const void *const *M, const float *const *v,
                                 int act_mode) {
    if (n < 0 || (n > 0 && (!dst || !M || !v)) || (act_mode != HOLO_ACT_Q8 && act_mode != HOLO_ACT_F32)) {
        holo_set_status(HOLO_E_ARG, "cuda_matvec_batch: bad arguments");
        return HOLO_E_ARG;
    }
    if (n == 0) return HOLO_OK;
    HoloDevice *D = holo_dev();
    if (!D) return cuda_last_status();
    std::vector<WeightInfo> wi(n);
    for (int i = 0; i < n; ++i) {
        if (!dst[i] || !v[i] || !holo_registry_find(M[i], &wi[i])) {
            holo_set_status(HOLO_E_ARG, "cuda_matvec_batch: every M must be a tiled weight from cuda_upload_quant");
            return HOLO_E_ARG;
        }
    }
    cudaStream_t st = holo_stream();
    const bool pdl = holo_pdl() != 0;
    // one launch per weight type (problems in call order), MM_MAX problems a launch
    std::vector<int> done(n, 0);
    for (int i = 0; i < n; ++i) {
        if (done[i]) continue;
        int idx[MM_MAX], k = 0;
        for (int j = i; j < n && k < MM_MAX; ++j)
            if (!done[j] && wi[j].type == wi[i].type) {
                idx[k++] = j;
                done[j] = 1;
            }
        if (!mm_group(idx, k, dst, M, v, wi.data(), act_mode, D, st, pdl))
            return cuda_last_status() ? cuda_last_status() : HOLO_E_ARG;
    }
    return HOLO_OK;
}
