// matvec_batch.cu -- quantized matmul for a few activation rows (M <= 16),
// the projections of batched decode (batch 8).
//
// At small M a tensor-core tile is mostly padding and its issue rate, not
// HBM, bounds the matmul; here every weight unit is read from HBM once and
// dotted with all M activation rows on the CUDA cores, with the batch-1 Q8
// matvec's arithmetic per row (holo_mv::unit_dot: dp4a integer block dots,
// the activation quantized per 32 values as quantize_vals_q8 does).
//
// Design:
//   * grid = (row groups of MVB_WARPS row-blocks) x (K slices); warp w of a
//     CTA owns row-block rb = group*MVB_WARPS + w (lane r = row r) and walks
//     the slice's units of that row-block, which are contiguous in the unit
//     layout: one unit in registers, each of its planes replaced by the next
//     unit's as soon as it is consumed, MVB_L2_AHEAD more prefetched into L2;
//   * prologue: the CTA quantizes its K slice of every activation row into
//     shared memory (one thread per 32-value block), after issuing its first
//     weight loads;
//   * each unit fragment is dotted with every row (acc[m] for row m); the
//     nibble masks of a plane are computed once for all rows;
//   * one K slice: results stored directly.  Several: per-slice partials, and
//     the last CTA of a row group to finish (acq_rel counter) sums them in
//     slice order -- deterministic, no second kernel.
#include "holo_common.cuh"
#include "mv_device.cuh"
#include "mv_unit.cuh"

#include <algorithm>

namespace {

using namespace holo_mv;

constexpr int MVB_WARPS = 8;
constexpr int MVB_THREADS = MVB_WARPS * 32;
constexpr int MVB_L2_AHEAD = 4;           // units a warp keeps prefetched into L2
constexpr size_t MVB_SMEM_TARGET = 100 * 1024;   // two CTAs an SM

struct MvbParams {
    const uint8_t *W;
    const float *X;
    float *Y;
    float *part;        // [S][M][N] split-K partials (S > 1)
    int *counters;      // [groups], zero between launches
    int M, N, K;
    int units;          // units a row
    int nrb, groups;    // row-blocks, row groups
    int S, us;          // K slices, units a slice
};

// One unit fragment (lane = row) against NB activation rows.  Shared memory
// holds the rows interleaved by 32-block: block b of row m has its codes at
// aq + (b*NB + m)*32 and its scale pair at ads[b*NB + m] (mvb_kernel's
// prologue).  b0 = the unit's first 32-block within the slice.  The masked
// code words of a block are formed once for all rows.  As each plane (and the
// head) is consumed, the same part of the next unit (`next`, unless NULL) is
// loaded into its registers: one fragment of registers, each load issued a
// unit of work ahead of its use.  Per row, the sums are the batch-1 Q8
// matvec's integer block dots (dot16 = 16 * sum nib*q, high nibbles used in
// place), scaled in fp32:
//   Q4_K  acc += (sc/16 * d_a) * dot16 - mn * (d_a*asum)   (sc/16 exact);
//   Q4_0  acc += (dw * d_a/16) * (dot16 - 128*asum), the code offset 8 taken
//         out in integers (|dot16 - 128*asum| < 2^20: exact);
//   Q8_0  acc += (dw * d_a) * dot.
template <int TYPE, int NB>
__device__ __forceinline__ void unit_dot_rows(float (&acc)[NB], Frag &f, int b0, const uint8_t *__restrict__ aq,
                                              const float2 *__restrict__ ads, const uint8_t *__restrict__ next,
                                              int lane) {
    constexpr uint32_t HI4 = 0xF0F0F0F0u;
    const uint8_t *nrow = next + (size_t)TILE_ROWS * UnitGeom<TYPE>::HEAD_BYTES + lane * 16;
    const uint4 h = f.h;
    if (next) {
        if constexpr (TYPE == GT_Q8_0) {
            const uint2 hn = ldg_stream2(next + lane * 8);
            f.h = make_uint4(hn.x, hn.y, 0u, 0u);
        } else {
            f.h = ldg_stream(next + lane * 16);
        }
    }
    if constexpr (TYPE == GT_Q4_K) {
        const float d = half_bits_to_float(h.x & 0xffffu) * 0.0625f;
        const float dmin = half_bits_to_float(h.x >> 16);
        const uint32_t sc_lo = h.y & 0x3F3F3F3Fu, m_lo = h.z & 0x3F3F3F3Fu;
        const uint32_t sc_hi = ((h.w & LO4) << 2) | ((h.y >> 6) & 0x03030303u);
        const uint32_t m_hi = (((h.w >> 4) & LO4) << 2) | ((h.z >> 6) & 0x03030303u);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float sc = d * ubyte_to_float(j < 4 ? sc_lo : sc_hi, j & 3);
            const float nmn = -(dmin * ubyte_to_float(j < 4 ? m_lo : m_hi, j & 3));
            const uint4 q = f.q[j];
            const uint4 lo = make_uint4(q.x & LO4, q.y & LO4, q.z & LO4, q.w & LO4);
            const uint4 hi = make_uint4(q.x & HI4, q.y & HI4, q.z & HI4, q.w & HI4);
            if (next) f.q[j] = ldg_stream(nrow + j * TILE_ROWS * 16);
            const uint8_t *ab = aq + (size_t)(b0 + j) * NB * 32;
            const float2 *db = ads + (size_t)(b0 + j) * NB;
#pragma unroll
            for (int m = 0; m < NB; ++m) {
                const uint4 a0 = lds128(ab + m * 32), a1 = lds128(ab + m * 32 + 16);
                const float2 ds = db[m];
                int sl = 0, sh = 0;
                sl = __dp4a((int)lo.x, (int)a0.x, sl); sh = dp4a_us(hi.x, a1.x, sh);
                sl = __dp4a((int)lo.y, (int)a0.y, sl); sh = dp4a_us(hi.y, a1.y, sh);
                sl = __dp4a((int)lo.z, (int)a0.z, sl); sh = dp4a_us(hi.z, a1.z, sh);
                sl = __dp4a((int)lo.w, (int)a0.w, sl); sh = dp4a_us(hi.w, a1.w, sh);
                acc[m] = fmaf(sc * ds.x, int_to_float_exact((sl << 4) + sh), acc[m]);
                acc[m] = fmaf(nmn, ds.y, acc[m]);
            }
        }
    } else if constexpr (TYPE == GT_Q4_0) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float dw = head_half(h, j);
            const uint4 q = f.q[j];
            const uint4 lo = make_uint4(q.x & LO4, q.y & LO4, q.z & LO4, q.w & LO4);
            const uint4 hi = make_uint4(q.x & HI4, q.y & HI4, q.z & HI4, q.w & HI4);
            if (next) f.q[j] = ldg_stream(nrow + j * TILE_ROWS * 16);
            const uint8_t *ab = aq + (size_t)(b0 + j) * NB * 32;
            const float2 *db = ads + (size_t)(b0 + j) * NB;
#pragma unroll
            for (int m = 0; m < NB; ++m) {
                const uint4 a0 = lds128(ab + m * 32), a1 = lds128(ab + m * 32 + 16);
                const float2 ds = db[m];   // (d_a/16, bits of 2^23 + 2^22 - 128*asum)
                int sl = 0, sh = 0;
                sl = __dp4a((int)lo.x, (int)a0.x, sl); sh = dp4a_us(hi.x, a1.x, sh);
                sl = __dp4a((int)lo.y, (int)a0.y, sl); sh = dp4a_us(hi.y, a1.y, sh);
                sl = __dp4a((int)lo.z, (int)a0.z, sl); sh = dp4a_us(hi.z, a1.z, sh);
                sl = __dp4a((int)lo.w, (int)a0.w, sl); sh = dp4a_us(hi.w, a1.w, sh);
                const float t = __int_as_float((sl << 4) + sh + __float_as_int(ds.y)) - 12582912.0f;
                acc[m] = fmaf(dw * ds.x, t, acc[m]);
            }
        }
    } else {  // Q8_0: block j = planes 2j, 2j+1
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float dw = head_half(h, j);
            const uint4 q0 = f.q[2 * j], q1 = f.q[2 * j + 1];
            if (next) {
                f.q[2 * j] = ldg_stream(nrow + (2 * j) * TILE_ROWS * 16);
                f.q[2 * j + 1] = ldg_stream(nrow + (2 * j + 1) * TILE_ROWS * 16);
            }
            const uint8_t *ab = aq + (size_t)(b0 + j) * NB * 32;
            const float2 *db = ads + (size_t)(b0 + j) * NB;
#pragma unroll
            for (int m = 0; m < NB; ++m) {
                const uint4 a0 = lds128(ab + m * 32), a1 = lds128(ab + m * 32 + 16);
                const int sd = dot_i8x32_q8(q0, q1, a0, a1);
                acc[m] = fmaf(dw * db[m].x, int_to_float_exact(sd), acc[m]);
            }
        }
    }
}

template <int TYPE, int NB>
__global__ void __launch_bounds__(MVB_THREADS, 2) mvb_kernel(const MvbParams p) {
    constexpr int BLKS32 = UnitGeom<TYPE>::BLKS32;
    constexpr size_t UB = UnitGeom<TYPE>::UNIT_BYTES;
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = blockIdx.x, sl = blockIdx.y;
    const int s0 = sl * p.us, s1 = min(p.units, s0 + p.us);
    const int ns = s1 - s0, nb = ns * BLKS32;   // units and 32-blocks of the slice
    uint8_t *aq = smem;                                                       // [nb][NB][32] int8
    float2 *ads = reinterpret_cast<float2 *>(smem + (size_t)NB * nb * 32);   // [nb][NB] scale pairs
    const int rb = grp * MVB_WARPS + warp;
    const bool live = rb < p.nrb;
    const uint8_t *wrow = p.W + ((size_t)rb * p.units + s0) * UB;

    // the warp's first unit into registers, the next ones into L2, before
    // the prologue
    Frag f;
    if (live && ns > 0) {
        load_unit<TYPE>(f, wrow, lane);
        if (lane == 0)
            for (int k = 1; k <= MVB_L2_AHEAD && k < ns; ++k) prefetch_l2_bulk(wrow + (size_t)k * UB, (uint32_t)UB);
    }

    // prologue: the slice of every activation row, quantized per 32 values
    for (int t = threadIdx.x; t < NB * nb; t += MVB_THREADS) {
        const int m = t / nb, b = t - m * nb;
        uint32_t w[8];
        float d = 0.0f;
        int asum = 0;
        if (m < p.M) {
            quantize_block_q8(p.X + (size_t)m * p.K + (size_t)(s0 * BLKS32 + b) * 32, w, d, asum);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = 0u;
        }
        uint4 *dst = reinterpret_cast<uint4 *>(aq + ((size_t)b * NB + m) * 32);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        if constexpr (TYPE == GT_Q4_0)
            ads[(size_t)b * NB + m] = make_float2(d * 0.0625f, __int_as_float(0x4B400000 - 128 * asum));
        else
            ads[(size_t)b * NB + m] = make_float2(d, d * (float)asum);
    }
    __syncthreads();

    float acc[NB];
#pragma unroll
    for (int m = 0; m < NB; ++m) acc[m] = 0.0f;
    if (live) {
        for (int u = 0; u < ns; ++u) {
            const int up = u + 1 + MVB_L2_AHEAD;
            if (lane == 0 && up < ns) prefetch_l2_bulk(wrow + (size_t)up * UB, (uint32_t)UB);
            unit_dot_rows<TYPE, NB>(acc, f, u * BLKS32, aq, ads, u + 1 < ns ? wrow + (size_t)(u + 1) * UB : nullptr,
                                    lane);
        }
    }

    const int row = rb * TILE_ROWS + lane;
    if (p.S == 1) {
        if (live && row < p.N)
#pragma unroll
            for (int m = 0; m < NB; ++m)
                if (m < p.M) p.Y[(size_t)m * p.N + row] = acc[m];
        return;
    }
    if (live && row < p.N)
#pragma unroll
        for (int m = 0; m < NB; ++m)
            if (m < p.M) p.part[((size_t)sl * p.M + m) * p.N + row] = acc[m];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int prev;
        asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(prev) : "l"(p.counters + grp) : "memory");
        s_last = prev == p.S - 1;
    }
    __syncthreads();
    if (!s_last) return;
    // the last slice of the group: sum the partials in slice order
    const int r0 = grp * MVB_WARPS * TILE_ROWS;
    const int nr = min(MVB_WARPS * TILE_ROWS, p.N - r0);
    for (int t = threadIdx.x; t < p.M * nr; t += MVB_THREADS) {
        const int m = t / nr, r = r0 + (t - m * nr);
        float v = 0.0f;
        for (int k = 0; k < p.S; ++k) v += __ldcg(p.part + ((size_t)k * p.M + m) * p.N + r);
        p.Y[(size_t)m * p.N + r] = v;
    }
    if (threadIdx.x == 0) p.counters[grp] = 0;
}

// launch plan: K in MVB_SLICES slices (fewer when the rows are short, more
// when a slice's activations would exceed the shared-memory target).  Swept
// on the 7B and 70B projections at 8 rows (1 to 32 units a slice): eight
// slices were within a few percent of the best count for every shape, and
// up to 30 % faster than one slice -- the per-warp chain of dependent unit
// loads, not the partials, sets the time.
constexpr int MVB_SLICES = 8;

struct MvbPlan {
    int groups, S, us;
    size_t smem, part_bytes;
};

MvbPlan mvb_plan(const WeightInfo &wi, int M, int sms) {
    (void)sms;
    const int nb_unit = wi.type == GT_Q8_0 ? UnitGeom<GT_Q8_0>::BLKS32 : UnitGeom<GT_Q4_0>::BLKS32;
    const int NB = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16;
    MvbPlan pl{};
    const int nrb = wi.rows_padded / TILE_ROWS;
    pl.groups = (nrb + MVB_WARPS - 1) / MVB_WARPS;
    pl.us = (wi.units + MVB_SLICES - 1) / MVB_SLICES;
    while (pl.us > 1 && (size_t)NB * pl.us * nb_unit * 40 > MVB_SMEM_TARGET) --pl.us;
    pl.S = (wi.units + pl.us - 1) / pl.us;
    pl.smem = (size_t)NB * pl.us * nb_unit * 40;
    pl.part_bytes = pl.S > 1 ? sizeof(float) * (size_t)pl.S * M * wi.rows : 0;
    return pl;
}

template <int TYPE, int NB>
bool launch_mvb(const MvbParams &p, size_t smem, cudaStream_t st) {
    auto kern = mvb_kernel<TYPE, NB>;
    static bool configured[16] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 16 && !configured[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
            return holo_check_launch("few-row matmul: kernel attributes");
        configured[dev] = true;
    }
    kern<<<dim3(p.groups, p.S), MVB_THREADS, smem, st>>>(p);
    return holo_check_launch("few-row matmul launch");
}

template <int TYPE>
bool dispatch_nb(const MvbParams &p, size_t smem, cudaStream_t st) {
    if (p.M <= 1) return launch_mvb<TYPE, 1>(p, smem, st);
    if (p.M <= 2) return launch_mvb<TYPE, 2>(p, smem, st);
    if (p.M <= 4) return launch_mvb<TYPE, 4>(p, smem, st);
    if (p.M <= 8) return launch_mvb<TYPE, 8>(p, smem, st);
    return launch_mvb<TYPE, 16>(p, smem, st);
}

}  // namespace

size_t holo_matmul_few_scratch(const WeightInfo &wi, int M) {
    HoloDevice *D = holo_dev();
    return mvb_plan(wi, M, D ? D->sms : 148).part_bytes;
}

bool holo_matmul_few(float *Y, const void *W, const WeightInfo &wi, const float *X, int M, cudaStream_t st,
                     void *scratch, size_t scratch_bytes) {
    HoloDevice *D = holo_dev();
    if (!D) return false;
    const int vals = wi.type == GT_Q8_0 ? 128 : 256;
    if (!Y || !W || !X || M <= 0 || M > MVB_MAX_M || wi.cols % vals || (uintptr_t)X % 16 ||
        (wi.type != GT_Q4_K && wi.type != GT_Q4_0 && wi.type != GT_Q8_0)) {
        holo_set_status(HOLO_E_ARG, "few-row matmul: needs 1..16 rows, a tiled Q8_0/Q4_0/Q4_K weight of whole "
                                    "units, 16-byte aligned X");
        return false;
    }
    const MvbPlan pl = mvb_plan(wi, M, D->sms);
    if (pl.groups > MVB_MAX_GROUPS) {
        holo_set_status(HOLO_E_UNSUPPORTED, "few-row matmul: too many rows");
        return false;
    }
    float *part = nullptr;
    if (pl.part_bytes) {
        if (scratch) {
            if (scratch_bytes < pl.part_bytes) {
                holo_set_status(HOLO_E_ARG, "few-row matmul: scratch too small");
                return false;
            }
            part = static_cast<float *>(scratch);
        } else {
            part = static_cast<float *>(holo_tmp(pl.part_bytes));
            if (!part) return false;
        }
    }
    MvbParams p{};
    p.W = static_cast<const uint8_t *>(W);
    p.X = X;
    p.Y = Y;
    p.part = part;
    p.counters = D->mvb_counters;
    p.M = M;
    p.N = wi.rows;
    p.K = wi.cols;
    p.units = wi.units;
    p.nrb = wi.rows_padded / TILE_ROWS;
    p.groups = pl.groups;
    p.S = pl.S;
    p.us = pl.us;
    switch (wi.type) {
    case GT_Q8_0: return dispatch_nb<GT_Q8_0>(p, pl.smem, st);
    case GT_Q4_0: return dispatch_nb<GT_Q4_0>(p, pl.smem, st);
    default: return dispatch_nb<GT_Q4_K>(p, pl.smem, st);
    }
}
