// matvec.cu -- tiled batch-1 quantized matvec for sm_100a.
//
// Replaces the reference's matvec kernels (src/ai/cuda_ops.cu:446-508,
// 618-676, 694-732, 859-1060), which read 34/18/144-byte blocks with byte
// loads, one block or warp per row.
//
// Design (one 256-thread CTA per SM, room for a second one):
//   * the weights are in the unit layout (holo_common.cuh): warp w of a CTA
//     takes every NWARP-th unit of the CTA's contiguous unit range, and lane r
//     holds row r of the unit -- eight coalesced 16-byte loads per lane per
//     unit, so the per-unit index work is amortised over 144 bytes a row;
//   * before the PDL wait, the CTA prefetches its first units into L2 with
//     bulk prefetches (nothing returns to the SM) -- the next kernel's CTAs
//     are resident while this one runs, so HBM streams the next matrix while
//     the current one finishes; after the wait, x (and the RMSNorm weights)
//     arrive in shared memory through one bulk copy each, and each warp keeps
//     MV_DEPTH units loading into registers and MV_L2_AHEAD units in L2;
//   * prologue: optional RMSNorm of x (the reference's rms_norm,
//     src/ai/tensor.c:242-255), then HOLO_ACT_Q8 quantizes x per 32-block
//     (one thread per block) or HOLO_ACT_F32 takes fp32 block sums;
//   * per-warp partials of each row-block meet in shared memory; a row-block
//     cut between CTAs is finished deterministically by the last CTA to
//     contribute (acq_rel atomic counter, partials summed in CTA order);
//   * epilogues: store, residual add (src/ai/llm.c:1217, 1245), or the SwiGLU
//     gate (silu(g)*u, llm.c:1231-1236) over row pairs interleaved by 16.
// The kernel has no waits on other CTAs: the fix-up is last-arriver, not spin;
// its one wait (the activation copy) is bounded.
#include "holo_common.cuh"
#include "mv_device.cuh"
#include "mv_unit.cuh"
#include "matvec.cuh"

#include <cstdio>

namespace {

using namespace holo_mv;

constexpr int NWARP = 8;                  // warps per CTA
constexpr int NTHREADS = NWARP * 32;
constexpr int MIN_CTAS_PER_SM = 2;        // room for the next kernel's CTA (PDL overlap)
constexpr int MV_DEPTH = 2;               // units of loads kept in flight per warp (ring)
constexpr int MV_L2_AHEAD = 5;            // units per warp prefetched into L2 ahead of use
constexpr size_t SMEM_LIMIT = 227 * 1024;

struct MvParams {
    const uint8_t *W;
    const float *x;
    float *y;
    const float *residual;
    const float *norm_w;
    float eps;
    int out_dim, in_dim;
    int nblk32;          // in_dim / 32
    int nblk32p;         // 32-blocks per row of the tiled layout (padded to whole units)
    int units;           // units per row
    int nrb, total_units, nctas;
    int max_local_rb;    // row-blocks one CTA can touch (size of the reduction buffer)
    int bulk;            // x (and norm_w) 16-byte aligned: staged by one bulk copy each
    float *partials;
    int *counters;
    int *status;         // device status word (bounded waits)
};

// Shared-memory map of one CTA (byte offsets), the same on host and device:
//   red   [max_local_rb][NWARP][32] f32   per-warp row-block partials
//   act   ACT_Q8: q8 [nblk32p*32] i8, (d, d*asum) [nblk32p] f32x2
//   stage x as copied in, padded with zeros to nblk32p*32 values
//         (ACT_F32: this is the activation itself, followed by xsum [nblk32p])
//   nw    RMSNorm weights (NORM only)
//   misc  mbarrier, per-warp sums of squares
struct MvSmem {
    size_t red, act, stage, nw, misc, total;
};
__host__ __device__ __forceinline__ MvSmem mv_smem_layout(int act, bool norm, int max_local_rb, int nblk32p) {
    MvSmem L;
    size_t o = 0;
    L.red = o;
    o += (size_t)max_local_rb * NWARP * 32 * sizeof(float);
    L.act = o;
    if (act == HOLO_ACT_Q8) {
        o += (size_t)nblk32p * 40;
        L.stage = o;
        o += (size_t)nblk32p * 128;
    } else {
        L.stage = o;
        o += (size_t)nblk32p * 132;
    }
    L.nw = o;
    if (norm) o += (size_t)nblk32p * 128;
    L.misc = o;
    o += 128;
    L.total = o;
    return L;
}

// Even split of T units over C CTAs (T*C < 2^32 is checked on the host).
__device__ __forceinline__ int tile_owner(unsigned t, unsigned T, unsigned C) {
    return (int)(((t + 1) * C - 1) / T);
}
__device__ __forceinline__ int tile_begin(unsigned c, unsigned T, unsigned C) {
    return (int)(T * c / C);
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Final value of the 32 rows of row-block rb (v held by lane r = row r),
// executed by all lanes of one warp.
template <int EPI>
__device__ __forceinline__ void finish_rowblock(const MvParams &p, int rb, int lane, float v) {
    if constexpr (EPI == MV_EPI_SILU_MUL) {
        const float u = __shfl_down_sync(0xffffffffu, v, 16);
        const int r = rb * 16 + lane;
        if (lane < 16 && r < (p.out_dim >> 1)) p.y[r] = (v / (1.0f + expf(-v))) * u;
    } else {
        const int row = rb * TILE_ROWS + lane;
        if (row < p.out_dim) {
            if constexpr (EPI == MV_EPI_ADD) v += p.residual[row];
            p.y[row] = v;
        }
    }
}

// Row-block rb's sum over this CTA's units is v (lane r = row r): store it,
// or -- when other CTAs hold part of the row-block -- publish it and let the
// last contributor sum all parts in CTA order (stream-K fix-up).
template <int EPI>
__device__ __forceinline__ void complete_rowblock(const MvParams &p, int rb, int rb_first, int t0, int t1,
                                                  unsigned T, unsigned C, int lane, float v) {
    const unsigned tb = (unsigned)rb * p.units, te = tb + p.units - 1;
    if ((int)tb >= t0 && (int)te < t1) {
        finish_rowblock<EPI>(p, rb, lane, v);
        return;
    }
    const int c_first = tile_owner(tb, T, C), c_last = tile_owner(te, T, C);
    const int slot = (rb == rb_first) ? 0 : 1;
    p.partials[((size_t)blockIdx.x * 2 + slot) * 32 + lane] = v;
    __syncwarp();
    int prev = 0;
    if (lane == 0)
        asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(prev) : "l"(&p.counters[rb]) : "memory");
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev == c_last - c_first) {
        __syncwarp();   // lane 0's acquire orders the reads below
        float tot = 0.0f;
        for (int c = c_first; c <= c_last; ++c) {
            const int sl = (rb == tile_begin(c, T, C) / p.units) ? 0 : 1;
            tot += __ldcg(&p.partials[((size_t)c * 2 + sl) * 32 + lane]);
        }
        finish_rowblock<EPI>(p, rb, lane, tot);
        if (lane == 0) p.counters[rb] = 0;
    }
}

template <int TYPE, int ACT, int EPI, bool NORM>
__global__ void __launch_bounds__(NTHREADS, MIN_CTAS_PER_SM) mv_tiled_kernel(const MvParams p) {
    constexpr int BLKS32 = UnitGeom<TYPE>::BLKS32;
    constexpr size_t UB = UnitGeom<TYPE>::UNIT_BYTES;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const MvSmem SL = mv_smem_layout(ACT, NORM, p.max_local_rb, p.nblk32p);
    float *red = reinterpret_cast<float *>(smem + SL.red);
    uint8_t *aq = smem + SL.act;
    float2 *ads = reinterpret_cast<float2 *>(smem + SL.act + (size_t)p.nblk32p * 32);
    float *xst = reinterpret_cast<float *>(smem + SL.stage);
    float *xs = xst;                                            // ACT_F32 activation
    float *xsum = xst + (size_t)p.nblk32p * 32;
    float *nw = reinterpret_cast<float *>(smem + SL.nw);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + SL.misc);
    float *wsum = reinterpret_cast<float *>(smem + SL.misc + 64);

    pdl_trigger();
    const unsigned T = p.total_units, C = p.nctas;
    const int u0 = tile_begin(blockIdx.x, T, C), u1 = tile_begin(blockIdx.x + 1, T, C);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }

    // Warp w takes units u0+w, u0+w+NWARP, ... (the CTA's warps read NWARP
    // consecutive units at a time).  Weights are constant, so before waiting
    // for the kernel this one depends on, the first MV_L2_AHEAD units of every
    // warp are prefetched into L2: HBM streams them while the previous kernel
    // finishes, and nothing returns to this SM yet, so the activation copy
    // below is not queued behind them.  In the loop, each warp keeps
    // MV_L2_AHEAD units prefetched and MV_DEPTH units loading into registers.
    // The activation (and norm weights, residual) go first: it is on the
    // critical path after the wait, and a line the previous kernel is still
    // writing is simply updated in L2.
    if (threadIdx.x == 32 && p.bulk) {
        prefetch_l2_bulk(p.x, (uint32_t)p.in_dim * 4u);
        if constexpr (NORM) prefetch_l2_bulk(p.norm_w, (uint32_t)p.in_dim * 4u);
    }
    if (lane == 0) {
#pragma unroll
        for (int k = 0; k < MV_L2_AHEAD; ++k) {
            const int uu = u0 + warp + k * NWARP;
            if (uu < u1) prefetch_l2_bulk(p.W + (size_t)uu * UB, (uint32_t)UB);
        }
    }
    __syncthreads();   // barrier initialised

    // ------------------------------ prologue ---------------------------------
    // x (and the norm weights) land in shared memory through one bulk copy each
    // -- one round trip, however long the vector -- then 8 threads per 32-value
    // block normalise and quantize from there.
    pdl_wait();   // x and residual come from earlier kernels
    const int ctid = threadIdx.x;
    const uint32_t xbytes = (uint32_t)p.in_dim * 4u;
    if (p.bulk) {
        if (ctid == 0) {
            mbar_arrive_expect_tx(bar, NORM ? 2u * xbytes : xbytes);
            bulk_copy_g2s(xst, p.x, xbytes, bar);
            if constexpr (NORM) bulk_copy_g2s(nw, p.norm_w, xbytes, bar);
        }
    } else {
        for (int i = ctid; i < p.in_dim; i += NTHREADS) {
            xst[i] = __ldg(p.x + i);
            if constexpr (NORM) nw[i] = __ldg(p.norm_w + i);
        }
    }
    Frag ring[MV_DEPTH];
#pragma unroll
    for (int k = 0; k < MV_DEPTH; ++k) {
        const int uu = u0 + warp + k * NWARP;
        if (uu < u1) load_unit<TYPE>(ring[k], p.W + (size_t)uu * UB, lane);
    }
    for (int i = p.in_dim + ctid; i < p.nblk32p * 32; i += NTHREADS) {
        xst[i] = 0.0f;
        if constexpr (NORM) nw[i] = 0.0f;
    }
    const int rb_first = u0 / p.units;
    const int n_local = (u1 - 1) / p.units - rb_first + 1;
    for (int i = ctid; i < n_local * NWARP * 32; i += NTHREADS) red[i] = 0.0f;
    bool ok = true;
    if (p.bulk) ok = mbar_wait_bounded(bar, 0, p.status, HOLO_E_TIMEOUT);
    if (!__syncthreads_and(ok)) return;

    act_prologue<ACT, NORM, NTHREADS>(xst, nw, aq, ads, xsum, wsum, p.in_dim, p.nblk32p, p.eps);

    // ------------------------------- main loop --------------------------------
    // The warp's running sum of one row-block is parked in red[row-block][warp]
    // when the warp moves on to the next row-block (no barrier); one barrier at
    // the end, then the row-blocks are reduced over the warps in warp order.
    int rb = (u0 + warp) / p.units, s = u0 + warp - rb * p.units;   // unit (rb, s)
    const int dq = NWARP / p.units, dr = NWARP - dq * p.units;      // step of NWARP units
    int cur_rb = rb;
    float acc = 0.0f;
    for (int ub = u0 + warp; ub < u1; ub += MV_DEPTH * NWARP) {
#pragma unroll
        for (int k = 0; k < MV_DEPTH; ++k) {
            const int u = ub + k * NWARP;
            if (u >= u1) break;
            if (rb != cur_rb) {
                red[((cur_rb - rb_first) * NWARP + warp) * 32 + lane] = acc;
                acc = 0.0f;
                cur_rb = rb;
            }
            unit_dot<TYPE, ACT>(acc, ring[k], s * BLKS32, aq, ads, xs, xsum);
            const int un = u + MV_DEPTH * NWARP;
            if (un < u1) load_unit<TYPE>(ring[k], p.W + (size_t)un * UB, lane);
            const int up = u + MV_L2_AHEAD * NWARP;
            if (lane == 0 && up < u1) prefetch_l2_bulk(p.W + (size_t)up * UB, (uint32_t)UB);
            s += dr;
            rb += dq;
            if (s >= p.units) { s -= p.units; ++rb; }
        }
    }
    if (u0 + warp < u1) red[((cur_rb - rb_first) * NWARP + warp) * 32 + lane] = acc;
    __syncthreads();
    for (int l = warp; l < n_local; l += NWARP) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < NWARP; w++) v += red[(l * NWARP + w) * 32 + lane];
        complete_rowblock<EPI>(p, rb_first + l, rb_first, u0, u1, T, C, lane, v);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// kernel attributes (dynamic shared memory limit, carveout), once per device
template <int TYPE, int ACT, int EPI, bool NORM>
bool configure_tiled() {
    auto kern = mv_tiled_kernel<TYPE, ACT, EPI, NORM>;
    static bool configured[16] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 16 || configured[dev]) return true;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_LIMIT) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess) {
        holo_check_launch("tiled matvec: kernel attributes");
        return false;
    }
    configured[dev] = true;
    return true;
}

// max_ctas == 0: set-up only (holo_matvec_prepare)
template <int TYPE, int ACT, int EPI, bool NORM>
bool launch_tiled(const MvParams &base, int sms, int max_ctas, bool pdl, cudaStream_t st) {
    if (!configure_tiled<TYPE, ACT, EPI, NORM>()) return false;
    if (max_ctas == 0) return true;
    MvParams p = base;
    if ((unsigned long long)p.total_units * (unsigned long long)max_ctas >= (1ull << 32)) {
        holo_set_status(HOLO_E_UNSUPPORTED, "tiled matvec: too many units");
        return false;
    }
    // One CTA per SM; more (in further waves) only when a CTA's share of the
    // row-blocks would not fit its reduction buffer.
    size_t smem = 0;
    p.nctas = min(p.total_units, min(sms, max_ctas));
    for (;;) {
        const int per_cta = (p.total_units + p.nctas - 1) / p.nctas;
        p.max_local_rb = (p.units + per_cta - 2) / p.units + 1;
        smem = mv_smem_layout(ACT, NORM, p.max_local_rb, p.nblk32p).total;
        if (smem <= SMEM_LIMIT) break;
        if (p.nctas >= min(p.total_units, max_ctas) || mv_smem_layout(ACT, NORM, 2, p.nblk32p).total > SMEM_LIMIT) {
            holo_set_status(HOLO_E_UNSUPPORTED, "tiled matvec: in_dim too large for shared memory");
            return false;
        }
        p.nctas = min(min(p.total_units, max_ctas), p.nctas + sms);
    }
    auto kern = mv_tiled_kernel<TYPE, ACT, EPI, NORM>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.nctas);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return holo_check_launch("tiled matvec launch");
    return holo_check_launch("tiled matvec launch");
}

template <int TYPE, int ACT>
bool dispatch_epi(const MvParams &p, int epi, bool norm, int sms, int mc, bool pdl, cudaStream_t st) {
    switch (epi) {
    case MV_EPI_ADD:
        return norm ? launch_tiled<TYPE, ACT, MV_EPI_ADD, true>(p, sms, mc, pdl, st)
                    : launch_tiled<TYPE, ACT, MV_EPI_ADD, false>(p, sms, mc, pdl, st);
    case MV_EPI_SILU_MUL:
        return norm ? launch_tiled<TYPE, ACT, MV_EPI_SILU_MUL, true>(p, sms, mc, pdl, st)
                    : launch_tiled<TYPE, ACT, MV_EPI_SILU_MUL, false>(p, sms, mc, pdl, st);
    default:
        return norm ? launch_tiled<TYPE, ACT, MV_EPI_STORE, true>(p, sms, mc, pdl, st)
                    : launch_tiled<TYPE, ACT, MV_EPI_STORE, false>(p, sms, mc, pdl, st);
    }
}

template <int TYPE>
bool dispatch_act(const MvParams &p, int act, int epi, bool norm, int sms, int mc, bool pdl, cudaStream_t st) {
    if (act == HOLO_ACT_Q8) return dispatch_epi<TYPE, HOLO_ACT_Q8>(p, epi, norm, sms, mc, pdl, st);
    return dispatch_epi<TYPE, HOLO_ACT_F32>(p, epi, norm, sms, mc, pdl, st);
}

}  // namespace

bool holo_matvec_launch(const void *M, const WeightInfo &wi, const MvLaunch &L, cudaStream_t st) {
    HoloDevice *D = holo_dev();
    if (!D) return false;
    MvScratch S;
    S.partials = L.partials ? L.partials : D->mv_partials;
    S.counters = L.counters ? L.counters : D->mv_counters;
    S.status = D->status;
    S.sms = D->sms;
    S.max_ctas = MV_MAX_CTAS;
    S.max_rowblocks = MV_MAX_ROWBLOCKS;
    return holo_matvec_launch_with(M, wi, L, st, S);
}

bool holo_matvec_prepare(const WeightInfo &wi, const MvLaunch &L) {
    MvScratch S;   // max_ctas == 0: set-up only, nothing is launched
    S.sms = 1;
    S.max_rowblocks = MV_MAX_ROWBLOCKS;
    return holo_matvec_launch_with(nullptr, wi, L, nullptr, S);
}

bool holo_matvec_launch_with(const void *M, const WeightInfo &wi, const MvLaunch &L, cudaStream_t st,
                             const MvScratch &S) {
    MvParams p{};
    p.W = (const uint8_t *)M;
    p.x = L.x;
    p.y = L.y;
    p.residual = L.residual;
    p.norm_w = L.norm_w;
    p.eps = L.eps;
    p.out_dim = wi.rows;
    p.in_dim = wi.cols;
    p.nblk32 = wi.cols / 32;
    p.units = wi.units;
    p.nrb = wi.rows_padded / TILE_ROWS;
    p.total_units = p.nrb * p.units;
    p.partials = S.partials;
    p.counters = S.counters;
    p.status = S.status;
    p.bulk = ((uintptr_t)L.x % 16 == 0) && ((uintptr_t)L.norm_w % 16 == 0);
    if (p.nrb > S.max_rowblocks) {
        holo_set_status(HOLO_E_UNSUPPORTED, "matvec: too many rows");
        return false;
    }
    if (L.epi == MV_EPI_SILU_MUL && (wi.rows % 32) != 0) {
        holo_set_status(HOLO_E_ARG, "matvec: the gated epilogue needs paired rows (multiple of 32)");
        return false;
    }
    const bool norm = L.norm_w != nullptr;
    switch (wi.type) {
    case GT_Q8_0:
        p.nblk32p = p.units * UnitGeom<GT_Q8_0>::BLKS32;
        return dispatch_act<GT_Q8_0>(p, L.act, L.epi, norm, S.sms, S.max_ctas, L.pdl, st);
    case GT_Q4_0:
        p.nblk32p = p.units * UnitGeom<GT_Q4_0>::BLKS32;
        return dispatch_act<GT_Q4_0>(p, L.act, L.epi, norm, S.sms, S.max_ctas, L.pdl, st);
    case GT_Q4_K:
        p.nblk32p = p.units * UnitGeom<GT_Q4_K>::BLKS32;
        return dispatch_act<GT_Q4_K>(p, L.act, L.epi, norm, S.sms, S.max_ctas, L.pdl, st);
    case GT_Q6_K:
        p.nblk32p = p.units * UnitGeom<GT_Q6_K>::BLKS32;
        return dispatch_act<GT_Q6_K>(p, L.act, L.epi, norm, S.sms, S.max_ctas, L.pdl, st);
    case GT_F16:   // fp32 activations whatever the mode (x as staged)
        p.nblk32p = p.units * UnitGeom<GT_F16>::BLKS32;
        return dispatch_act<GT_F16>(p, HOLO_ACT_F32, L.epi, norm, S.sms, S.max_ctas, L.pdl, st);
    default:
        holo_set_status(HOLO_E_ARG, "matvec: type has no tiled kernel");
        return false;
    }
}

void holo_matvec_tiled(float *dst, const void *M, const WeightInfo &wi, const float *v, int out_dim, int in_dim,
                       int act_mode, const float *residual, cudaStream_t st) {
    if (wi.rows != out_dim || wi.cols != in_dim) {
        holo_set_status(HOLO_E_ARG, "matvec: shape differs from the uploaded weight");
        return;
    }
    MvLaunch L;
    L.x = v;
    L.y = dst;
    L.residual = residual;
    L.act = act_mode;
    L.epi = residual ? MV_EPI_ADD : MV_EPI_STORE;
    L.pdl = holo_pdl() != 0;
    holo_matvec_launch(M, wi, L, st);
}
