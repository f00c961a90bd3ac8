// matvec.cu -- tiled batch-1 quantized matvec for sm_100a.
//
// Replaces the reference's matvec kernels (src/ai/cuda_ops.cu:446-508,
// 618-676, 694-732, 859-1060), which read 34/18/144-byte blocks with byte
// loads, one block or warp per row.
//
// Design (persistent, two CTAs per SM when shared memory allows, 9 warps each):
//   * warp 8 is the producer: one lane streams the CTA's tiles (~18 KB) from
//     HBM into a ring of shared-memory stages with 1-D bulk copies
//     (cp.async.bulk, L2 evict-first), completion counted on an mbarrier per
//     stage; weights are constant, so it starts before the PDL wait;
//   * warps 0..7 consume: lane r owns row r of the 32-row tile, warp w owns
//     1/8 of the tile's K extent, so the shared-memory reads of a warp are 32
//     consecutive 16-byte pieces (conflict-free) and activation reads are
//     broadcasts; per-row partials meet in shared memory at the end of each
//     row-block;
//   * the CTAs split the (row-block, K-chunk) tile sequence evenly (stream-K);
//     a row-block cut between CTAs is finished deterministically by the last
//     CTA to contribute (acq_rel atomic counter, partials summed in CTA order);
//   * prologue (consumers, after the PDL wait): optional RMSNorm of x (the
//     reference's rms_norm, src/ai/tensor.c:242-255), then HOLO_ACT_Q8
//     quantizes per 32-block into shared memory (dp4a dots) or HOLO_ACT_F32
//     stages fp32 x in shared memory (fp32 FMA dots);
//   * epilogues: store, residual add (src/ai/llm.c:1217, 1245), or the SwiGLU
//     gate (silu(g)*u, llm.c:1231-1236) over row pairs interleaved by 16.
// Every wait is bounded (1 s); a time-out sets the device status word.
#include "holo_common.cuh"
#include "mv_device.cuh"
#include "matvec.cuh"

#include <cstdio>

namespace {

constexpr int NCWARP = 8;                 // consumer warps
constexpr int NTHREADS = (NCWARP + 1) * 32;
constexpr int BAR_CONSUMERS = 1;          // named barrier id of the consumer warps

struct MvParams {
    const uint8_t *W;
    const float *x;
    float *y;
    const float *residual;
    const float *norm_w;
    float eps;
    int out_dim, in_dim;
    int nblk32;          // in_dim / 32
    int blks_per_row;    // GGUF blocks per row (Q4_K: super-blocks)
    int nkc, nrb, total_tiles, nctas, stages;
    size_t row_bytes;
    float *partials;
    int *counters;
    int *status;
};

__device__ __forceinline__ int tile_owner(long long t, long long T, long long C) {
    return (int)(((t + 1) * C - 1) / T);
}
__device__ __forceinline__ int tile_begin(long long c, long long T, long long C) {
    return (int)(T * c / C);
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// per-tile consumer arithmetic: this lane's (row's) partial over the warp's
// share of the tile
// ---------------------------------------------------------------------------
template <int TYPE, int ACT>
__device__ __forceinline__ float consume_tile(const uint8_t *__restrict__ tile, int kc, int nb, int warp, int lane,
                                              const uint8_t *__restrict__ aq, const float2 *__restrict__ ads,
                                              const float *__restrict__ xs, const float *__restrict__ xsum) {
    float acc = 0.0f;
    if constexpr (TYPE == GT_Q4_K) {
        const int sb = warp >> 1, half = warp & 1;
        if (sb < nb) {
            const uint8_t *sbp = tile + (size_t)(sb * TILE_ROWS + lane) * 144;
            const uint4 h = lds128(sbp);
            const float d = half_bits_to_float(h.x & 0xffffu), dmin = half_bits_to_float(h.x >> 16);
            uint32_t scw, mw;
            if (half == 0) {
                scw = h.y & 0x3F3F3F3Fu;
                mw = h.z & 0x3F3F3F3Fu;
            } else {
                scw = ((h.w & LO4) << 2) | ((h.y >> 6) & 0x03030303u);
                mw = (((h.w >> 4) & LO4) << 2) | ((h.z >> 6) & 0x03030303u);
            }
            const int blk0 = (kc * TileGeom<GT_Q4_K>::BLKS_PER_TILE + sb) * 8 + half * 4;
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const uint4 q = lds128(sbp + 16 + 16 * (half * 4 + jj));
                const int blk = blk0 + jj;
                const float sc = d * ubyte_to_float(scw, jj), mn = dmin * ubyte_to_float(mw, jj);
                if constexpr (ACT == HOLO_ACT_Q8) {
                    const uint4 a0 = lds128(aq + (size_t)blk * 32), a1 = lds128(aq + (size_t)blk * 32 + 16);
                    const float2 ds = ads[blk];
                    const float f16 = int_to_float_exact(dot_nib16_q8_x16(q, a0, a1));
                    acc = fmaf(sc * 0.0625f, ds.x * f16, acc);
                    acc = fmaf(-mn, ds.y, acc);
                } else {
                    acc = fmaf(sc, dot_nib16_f32<true>(q, xs + (size_t)blk * 32), acc);
                    acc = fmaf(-mn, xsum[blk], acc);
                }
            }
        }
    } else if constexpr (TYPE == GT_Q4_0) {
        constexpr int BPW = TileGeom<GT_Q4_0>::BLKS_PER_WARP;
        const uint8_t *dbase = tile + (size_t)nb * 512;
#pragma unroll
        for (int i = 0; i < BPW; i++) {
            const int b = warp * BPW + i;
            if (b >= nb) break;
            const uint4 q = lds128(tile + (size_t)(b * TILE_ROWS + lane) * 16);
            const float dw = half_bits_to_float(*reinterpret_cast<const uint16_t *>(dbase + (b * TILE_ROWS + lane) * 2));
            const int gb = kc * TileGeom<GT_Q4_0>::BLKS_PER_TILE + b;
            if constexpr (ACT == HOLO_ACT_Q8) {
                const uint4 a0 = lds128(aq + (size_t)gb * 32), a1 = lds128(aq + (size_t)gb * 32 + 16);
                const float2 ds = ads[gb];
                const float f16 = int_to_float_exact(dot_nib16_q8_x16(q, a0, a1));
                acc = fmaf(dw, fmaf(ds.x * 0.0625f, f16, -8.0f * ds.y), acc);
            } else {
                acc = fmaf(dw, dot_nib16_f32<true>(q, xs + (size_t)gb * 32) - 8.0f * xsum[gb], acc);
            }
        }
    } else {  // Q8_0
        constexpr int BPW = TileGeom<GT_Q8_0>::BLKS_PER_WARP;
        const uint8_t *dbase = tile + (size_t)nb * 1024;
#pragma unroll
        for (int i = 0; i < BPW; i++) {
            const int b = warp * BPW + i;
            if (b >= nb) break;
            const uint4 q0 = lds128(tile + (size_t)((b * 2 + 0) * TILE_ROWS + lane) * 16);
            const uint4 q1 = lds128(tile + (size_t)((b * 2 + 1) * TILE_ROWS + lane) * 16);
            const float dw = half_bits_to_float(*reinterpret_cast<const uint16_t *>(dbase + (b * TILE_ROWS + lane) * 2));
            const int gb = kc * TileGeom<GT_Q8_0>::BLKS_PER_TILE + b;
            if constexpr (ACT == HOLO_ACT_Q8) {
                const uint4 a0 = lds128(aq + (size_t)gb * 32), a1 = lds128(aq + (size_t)gb * 32 + 16);
                acc = fmaf(dw * ads[gb].x, int_to_float_exact(dot_i8x32_q8(q0, q1, a0, a1)), acc);
            } else {
                acc = fmaf(dw, dot_i8x32_f32<true>(q0, q1, xs + (size_t)gb * 32), acc);
            }
        }
    }
    return acc;
}

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

template <int TYPE, int ACT, int EPI, bool NORM>
__global__ void __launch_bounds__(NTHREADS, 2) mv_tiled_kernel(const MvParams p) {
    using G = TileGeom<TYPE>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.stages;
    uint8_t *stages = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * G::TILE_FULL);
    uint64_t *empty = full + S;
    float *red = reinterpret_cast<float *>(empty + S);               // [NCWARP][32]
    uint8_t *act = reinterpret_cast<uint8_t *>(red + NCWARP * 32);     // 16-B aligned
    // ACT_Q8: q8[in_dim] | (d, d*asum)[nblk32];  ACT_F32: xs[in_dim] | xsum[nblk32]
    uint8_t *aq = act;
    float2 *ads = reinterpret_cast<float2 *>(act + p.in_dim);
    float *xs = reinterpret_cast<float *>(act);
    float *xsum = xs + p.in_dim;

    pdl_trigger();
    const long long T = p.total_tiles, C = p.nctas;
    const int t0 = tile_begin(blockIdx.x, T, C), t1 = tile_begin(blockIdx.x + 1, T, C);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], NCWARP); }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == NCWARP) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            int issued = 0;
            for (int t = t0; t < t1; ++t, ++issued) {
                const int s = issued % S;
                if (issued >= S && !mbar_wait_bounded(&empty[s], ((issued / S) - 1) & 1, p.status, HOLO_E_TIMEOUT))
                    break;
                const int rb = t / p.nkc, kc = t % p.nkc;
                const int nb = min(G::BLKS_PER_TILE, p.blks_per_row - kc * G::BLKS_PER_TILE);
                const uint32_t bytes = (uint32_t)(TILE_ROWS * nb * G::BLK_BYTES);
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(stages + (size_t)s * G::TILE_FULL, p.W + tile_base(rb, kc, p.row_bytes, G::TILE_FULL),
                         bytes, &full[s], pol);
            }
            // never leave with copies in flight
            for (int k = max(0, issued - S); k < issued; ++k)
                mbar_wait_bounded(&full[k % S], (k / S) & 1, p.status, HOLO_E_TIMEOUT);
        }
        return;
    }

    // -------------------------------- consumers --------------------------------
    pdl_wait();   // x, norm weights and residual come from earlier kernels
    const int ctid = threadIdx.x;   // 0..255
    float scale = 1.0f;
    if constexpr (NORM) {
        float ss = 0.0f;
        for (int i = ctid * 4; i < p.in_dim; i += NCWARP * 32 * 4) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(p.x + i));
            ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[warp * 32] = ss;
        named_bar_sync(BAR_CONSUMERS, NCWARP * 32);
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < NCWARP; w++) tot += red[w * 32];
        scale = 1.0f / sqrtf(tot / (float)p.in_dim + p.eps);
    }
    for (int b = ctid; b < p.nblk32; b += NCWARP * 32) {
        float v[32];
        const float4 *x4 = reinterpret_cast<const float4 *>(p.x + (size_t)b * 32);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float4 t = __ldg(x4 + i);
            v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
        }
        if constexpr (NORM) {
            const float4 *w4 = reinterpret_cast<const float4 *>(p.norm_w + (size_t)b * 32);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                float4 t = __ldg(w4 + i);
                v[4 * i] = (v[4 * i] * scale) * t.x;
                v[4 * i + 1] = (v[4 * i + 1] * scale) * t.y;
                v[4 * i + 2] = (v[4 * i + 2] * scale) * t.z;
                v[4 * i + 3] = (v[4 * i + 3] * scale) * t.w;
            }
        }
        if constexpr (ACT == HOLO_ACT_Q8) {
            uint32_t w[8];
            float d;
            int asum;
            quantize_vals_q8(v, w, d, asum);
            uint4 *dst = reinterpret_cast<uint4 *>(aq + (size_t)b * 32);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
            ads[b] = make_float2(d, d * (float)asum);
        } else {
            float4 *dst = reinterpret_cast<float4 *>(xs + (size_t)b * 32);
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                s += (v[4 * i] + v[4 * i + 1]) + (v[4 * i + 2] + v[4 * i + 3]);
            }
            xsum[b] = s;
        }
    }
    named_bar_sync(BAR_CONSUMERS, NCWARP * 32);

    float acc = 0.0f;
    bool dead = false;
    const int rb_first = t0 / p.nkc;
    for (int t = t0, i = 0; t < t1; ++t, ++i) {
        const int s = i % S;
        const int rb = t / p.nkc, kc = t % p.nkc;
        const int nb = min(G::BLKS_PER_TILE, p.blks_per_row - kc * G::BLKS_PER_TILE);
        if (!dead) {
            if (mbar_wait_bounded(&full[s], (i / S) & 1, p.status, HOLO_E_TIMEOUT)) {
                acc += consume_tile<TYPE, ACT>(stages + (size_t)s * G::TILE_FULL, kc, nb, warp, lane, aq, ads, xs, xsum);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            } else {
                dead = true;
            }
        }
        if (kc == p.nkc - 1 || t == t1 - 1) {
            // end of this CTA's share of row-block rb: combine the warps
            red[warp * 32 + lane] = acc;
            named_bar_sync(BAR_CONSUMERS, NCWARP * 32);
            if (warp == 0 && !dead) {
                float v = 0.0f;
#pragma unroll
                for (int w = 0; w < NCWARP; w++) v += red[w * 32 + lane];
                const long long tb = (long long)rb * p.nkc, te = tb + p.nkc - 1;
                if (tb >= t0 && te < t1) {
                    finish_rowblock<EPI>(p, rb, lane, v);
                } else {
                    // stream-K fix-up: publish my partial (release), count the
                    // contributors; the last one sums all partials in CTA order
                    const int c_first = tile_owner(tb, T, C), c_last = tile_owner(te, T, C);
                    const int slot = (rb == rb_first) ? 0 : 1;
                    p.partials[((size_t)blockIdx.x * 2 + slot) * 32 + lane] = v;
                    __syncwarp();
                    int prev = 0;
                    if (lane == 0)
                        asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(prev) : "l"(&p.counters[rb]) : "memory");
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    if (prev == c_last - c_first) {
                        __threadfence();
                        float tot = 0.0f;
                        for (int c = c_first; c <= c_last; ++c) {
                            const int sl = (rb == tile_begin(c, T, C) / p.nkc) ? 0 : 1;
                            tot += __ldcg(&p.partials[((size_t)c * 2 + sl) * 32 + lane]);
                        }
                        finish_rowblock<EPI>(p, rb, lane, tot);
                        if (lane == 0) p.counters[rb] = 0;
                    }
                }
            }
            named_bar_sync(BAR_CONSUMERS, NCWARP * 32);
            acc = 0.0f;
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int TYPE, int ACT, int EPI, bool NORM>
bool launch_tiled(const MvParams &base, int sms, bool pdl, cudaStream_t st) {
    using G = TileGeom<TYPE>;
    MvParams p = base;
    size_t act_bytes = (ACT == HOLO_ACT_Q8) ? (size_t)p.in_dim + 8 * (size_t)p.nblk32
                                             : 4 * (size_t)p.in_dim + 4 * (size_t)p.nblk32;
    act_bytes = (act_bytes + 15) & ~(size_t)15;
    const size_t fixed = NCWARP * 32 * 4 + act_bytes;
    const size_t per_stage = G::TILE_FULL + 16;
    // two CTAs per SM when at least 3 stages fit in half of the SM's shared
    // memory, else one CTA with up to 8 stages
    const size_t half_budget = 113 * 1024, full_budget = 227 * 1024;
    int per_sm = 2, stages = (int)((half_budget - fixed) / per_stage);
    if (fixed >= half_budget || stages < 3) {
        per_sm = 1;
        stages = fixed >= full_budget ? 0 : (int)((full_budget - fixed) / per_stage);
    }
    stages = min(stages, 8);
    if (stages < 2) {
        holo_set_status(HOLO_E_UNSUPPORTED, "tiled matvec: in_dim too large for shared memory");
        return false;
    }
    p.stages = stages;
    const size_t smem = (size_t)stages * per_stage + fixed;
    auto kern = mv_tiled_kernel<TYPE, ACT, EPI, NORM>;
    static bool configured[16] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 16 && !configured[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)full_budget) != cudaSuccess) {
            holo_check_launch("tiled matvec: smem attribute");
            return false;
        }
        configured[dev] = true;
    }
    p.nctas = min(p.total_tiles, min(per_sm * sms, MV_MAX_CTAS));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.nctas);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return holo_check_launch("tiled matvec launch");
    return holo_check_launch("tiled matvec launch");
}

template <int TYPE, int ACT>
bool dispatch_epi(const MvParams &p, int epi, bool norm, int sms, bool pdl, cudaStream_t st) {
    switch (epi) {
    case MV_EPI_ADD:
        return norm ? launch_tiled<TYPE, ACT, MV_EPI_ADD, true>(p, sms, pdl, st)
                    : launch_tiled<TYPE, ACT, MV_EPI_ADD, false>(p, sms, pdl, st);
    case MV_EPI_SILU_MUL:
        return norm ? launch_tiled<TYPE, ACT, MV_EPI_SILU_MUL, true>(p, sms, pdl, st)
                    : launch_tiled<TYPE, ACT, MV_EPI_SILU_MUL, false>(p, sms, pdl, st);
    default:
        return norm ? launch_tiled<TYPE, ACT, MV_EPI_STORE, true>(p, sms, pdl, st)
                    : launch_tiled<TYPE, ACT, MV_EPI_STORE, false>(p, sms, pdl, st);
    }
}

template <int TYPE>
bool dispatch_act(const MvParams &p, int act, int epi, bool norm, int sms, bool pdl, cudaStream_t st) {
    if (act == HOLO_ACT_Q8) return dispatch_epi<TYPE, HOLO_ACT_Q8>(p, epi, norm, sms, pdl, st);
    return dispatch_epi<TYPE, HOLO_ACT_F32>(p, epi, norm, sms, pdl, st);
}

}  // namespace

bool holo_matvec_launch(const void *M, const WeightInfo &wi, const MvLaunch &L, cudaStream_t st) {
    HoloDevice *D = holo_dev();
    if (!D) return false;
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
    p.row_bytes = (size_t)gguf_row_bytes(wi.type, wi.cols);
    p.nrb = wi.rows_padded / TILE_ROWS;
    p.partials = L.partials ? L.partials : D->mv_partials;
    p.counters = L.counters ? L.counters : D->mv_counters;
    p.status = D->status;
    if (p.nrb > MV_MAX_ROWBLOCKS) {
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
        p.blks_per_row = wi.cols / 32;
        p.nkc = (p.blks_per_row + TileGeom<GT_Q8_0>::BLKS_PER_TILE - 1) / TileGeom<GT_Q8_0>::BLKS_PER_TILE;
        p.total_tiles = p.nrb * p.nkc;
        return dispatch_act<GT_Q8_0>(p, L.act, L.epi, norm, D->sms, L.pdl, st);
    case GT_Q4_0:
        p.blks_per_row = wi.cols / 32;
        p.nkc = (p.blks_per_row + TileGeom<GT_Q4_0>::BLKS_PER_TILE - 1) / TileGeom<GT_Q4_0>::BLKS_PER_TILE;
        p.total_tiles = p.nrb * p.nkc;
        return dispatch_act<GT_Q4_0>(p, L.act, L.epi, norm, D->sms, L.pdl, st);
    case GT_Q4_K:
        p.blks_per_row = wi.cols / 256;
        p.nkc = (p.blks_per_row + TileGeom<GT_Q4_K>::BLKS_PER_TILE - 1) / TileGeom<GT_Q4_K>::BLKS_PER_TILE;
        p.total_tiles = p.nrb * p.nkc;
        return dispatch_act<GT_Q4_K>(p, L.act, L.epi, norm, D->sms, L.pdl, st);
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
