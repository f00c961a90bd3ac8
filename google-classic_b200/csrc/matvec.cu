// matvec.cu -- tiled batch-1 quantized matvec for sm_100a.
//
// Replaces the reference's matvec kernels (src/ai/cuda_ops.cu:446-508,
// 618-676, 694-732, 859-1060), which read 34/18/144-byte blocks with byte
// loads, one block or warp per row.
//
// Design (one persistent CTA per SM, 9 warps):
//   * warp 8 is the producer: one lane streams the CTA's tiles from HBM into
//     a ring of shared-memory stages with 1-D bulk copies (cp.async.bulk,
//     L2 evict-first), completion counted on an mbarrier per stage;
//   * warps 0..7 consume: lane r owns row r of the 32-row tile, warp w owns
//     1/8 of the tile's K extent, so the shared-memory reads of a warp are
//     32 consecutive 16-byte pieces (conflict-free) and the activation reads
//     are broadcasts; per-row partials are combined across warps through
//     shared memory at the end of each row-block;
//   * the CTAs split the (row-block, K-chunk) tile sequence evenly (stream-K);
//     a row-block cut between CTAs is finished deterministically by the last
//     CTA to contribute (atomic counter, partials summed in CTA order);
//   * activations: HOLO_ACT_Q8 quantizes x per 32-block into shared memory in
//     the prologue (while the first bulk copies are in flight) and uses dp4a
//     integer dots; HOLO_ACT_F32 reads x through L1 and uses fp32 FMA.
// Every wait is bounded (1 s); a time-out sets the device status word.
#include "holo_common.cuh"
#include "mv_device.cuh"

#include <cstdio>

namespace {

constexpr int NCWARP = 8;                 // consumer warps
constexpr int NTHREADS = (NCWARP + 1) * 32;
constexpr int BAR_CONSUMERS = 1;          // named barrier id of the consumer warps

enum { EPI_STORE = 0, EPI_ADD = 1 };

struct MvParams {
    const uint8_t *W;
    const float *x;
    float *y;
    const float *residual;
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

// ---------------------------------------------------------------------------
// per-tile consumer arithmetic: returns this lane's (row's) partial over the
// warp's K slice of the tile
// ---------------------------------------------------------------------------
template <int TYPE, int ACT>
__device__ __forceinline__ float consume_tile(const uint8_t *__restrict__ tile, int kc, int nb,
                                              int warp, int lane, const MvParams &p,
                                              const uint8_t *__restrict__ aq, const float *__restrict__ ad,
                                              const int *__restrict__ as, const float *__restrict__ xsum) {
    float acc = 0.0f;
    if constexpr (TYPE == GT_Q4_K) {
        if (warp < nb) {
            const uint8_t *sbp = tile + (size_t)(warp * TILE_ROWS + lane) * 144;
            Q4KHead h = q4k_head(lds128(sbp));
            int sbg = kc * TileGeom<GT_Q4_K>::BLKS_PER_TILE + warp;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                uint4 q = lds128(sbp + 16 + 16 * j);
                int blk = sbg * 8 + j;
                float scf = q4k_scale(h, j), mf = q4k_min(h, j);
                if constexpr (ACT == HOLO_ACT_Q8) {
                    uint4 a0 = lds128(aq + (size_t)blk * 32), a1 = lds128(aq + (size_t)blk * 32 + 16);
                    int s = dot_nib16_q8(q, a0, a1);
                    acc += ad[blk] * ((h.d * scf) * int_to_float_exact(s) - (h.dmin * mf) * int_to_float_exact(as[blk]));
                } else {
                    float nx = dot_nib16_f32(q, p.x + (size_t)blk * 32);
                    acc += (h.d * scf) * nx - (h.dmin * mf) * xsum[blk];
                }
            }
        }
    } else if constexpr (TYPE == GT_Q4_0) {
        constexpr int BPW = TileGeom<GT_Q4_0>::BLKS_PER_WARP;
        const uint8_t *dbase = tile + (size_t)nb * 512;
#pragma unroll 4
        for (int i = 0; i < BPW; i++) {
            int b = warp * BPW + i;
            if (b >= nb) break;
            uint4 q = lds128(tile + (size_t)(b * TILE_ROWS + lane) * 16);
            float dw = half_bits_to_float(*reinterpret_cast<const uint16_t *>(dbase + (b * TILE_ROWS + lane) * 2));
            int gb = kc * TileGeom<GT_Q4_0>::BLKS_PER_TILE + b;
            if constexpr (ACT == HOLO_ACT_Q8) {
                uint4 a0 = lds128(aq + (size_t)gb * 32), a1 = lds128(aq + (size_t)gb * 32 + 16);
                int s = dot_nib16_q8(q, a0, a1) - 8 * as[gb];
                acc += (dw * ad[gb]) * int_to_float_exact(s);
            } else {
                float nx = dot_nib16_f32(q, p.x + (size_t)gb * 32);
                acc += dw * (nx - 8.0f * xsum[gb]);
            }
        }
    } else {  // Q8_0
        constexpr int BPW = TileGeom<GT_Q8_0>::BLKS_PER_WARP;
        const uint8_t *dbase = tile + (size_t)nb * 1024;
#pragma unroll
        for (int i = 0; i < BPW; i++) {
            int b = warp * BPW + i;
            if (b >= nb) break;
            uint4 q0 = lds128(tile + (size_t)((b * 2 + 0) * TILE_ROWS + lane) * 16);
            uint4 q1 = lds128(tile + (size_t)((b * 2 + 1) * TILE_ROWS + lane) * 16);
            float dw = half_bits_to_float(*reinterpret_cast<const uint16_t *>(dbase + (b * TILE_ROWS + lane) * 2));
            int gb = kc * TileGeom<GT_Q8_0>::BLKS_PER_TILE + b;
            if constexpr (ACT == HOLO_ACT_Q8) {
                uint4 a0 = lds128(aq + (size_t)gb * 32), a1 = lds128(aq + (size_t)gb * 32 + 16);
                int s = dot_i8x32_q8(q0, q1, a0, a1);
                acc += (dw * ad[gb]) * int_to_float_exact(s);
            } else {
                acc += dw * dot_i8x32_f32(q0, q1, p.x + (size_t)gb * 32);
            }
        }
    }
    return acc;
}

template <int EPI>
__device__ __forceinline__ void store_row(const MvParams &p, int row, float v) {
    if (row < p.out_dim) {
        if constexpr (EPI == EPI_ADD) v += p.residual[row];
        p.y[row] = v;
    }
}

template <int TYPE, int ACT, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1) mv_tiled_kernel(const MvParams p) {
    using G = TileGeom<TYPE>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.stages;
    uint8_t *stages = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * G::TILE_FULL);
    uint64_t *empty = full + S;
    float *red = reinterpret_cast<float *>(empty + S);             // [NCWARP][32]
    uint8_t *act = reinterpret_cast<uint8_t *>(red + NCWARP * 32);   // 16-B aligned
    // ACT_Q8: q8[in_dim] | d[nblk32] | asum[nblk32];  ACT_F32: xsum[nblk32]
    uint8_t *aq = act;
    float *ad = reinterpret_cast<float *>(act + p.in_dim);
    int *as = reinterpret_cast<int *>(ad + p.nblk32);
    float *xsum = reinterpret_cast<float *>(act);

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
            // never leave with copies in flight: wait (bounded) for the last
            // copy issued into each stage
            for (int k = max(0, issued - S); k < issued; ++k)
                mbar_wait_bounded(&full[k % S], (k / S) & 1, p.status, HOLO_E_TIMEOUT);
        }
        return;
    }

    // -------------------------------- consumers --------------------------------
    const int ctid = threadIdx.x;   // 0..255
    if constexpr (ACT == HOLO_ACT_Q8) {
        for (int b = ctid; b < p.nblk32; b += NCWARP * 32) {
            uint32_t w[8];
            float d;
            int asum;
            quantize_block_q8(p.x + (size_t)b * 32, w, d, asum);
            uint4 *dst = reinterpret_cast<uint4 *>(aq + (size_t)b * 32);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
            ad[b] = d;
            as[b] = asum;
        }
    } else {
        for (int b = ctid; b < p.nblk32; b += NCWARP * 32) {
            const float4 *x4 = reinterpret_cast<const float4 *>(p.x + (size_t)b * 32);
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                float4 t = __ldg(x4 + i);
                s += (t.x + t.y) + (t.z + t.w);
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
                acc += consume_tile<TYPE, ACT>(stages + (size_t)s * G::TILE_FULL, kc, nb, warp, lane, p,
                                               aq, ad, as, xsum);
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
                const int row = rb * TILE_ROWS + lane;
                if (tb >= t0 && te < t1) {
                    store_row<EPI>(p, row, v);
                } else {
                    // stream-K fix-up (deterministic): write my partial, count
                    // contributors; the last one sums all partials in CTA order
                    const int c_first = tile_owner(tb, T, C), c_last = tile_owner(te, T, C);
                    const int slot = (rb == rb_first) ? 0 : 1;
                    p.partials[((size_t)blockIdx.x * 2 + slot) * 32 + lane] = v;
                    __threadfence();
                    __syncwarp();
                    int prev = 0;
                    if (lane == 0) prev = atomicAdd(&p.counters[rb], 1);
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    if (prev == c_last - c_first) {
                        __threadfence();
                        float tot = 0.0f;
                        for (int c = c_first; c <= c_last; ++c) {
                            const int sl = (rb == tile_begin(c, T, C) / p.nkc) ? 0 : 1;
                            tot += __ldcg(&p.partials[((size_t)c * 2 + sl) * 32 + lane]);
                        }
                        store_row<EPI>(p, row, tot);
                        if (lane == 0) p.counters[rb] = 0;
                    }
                }
            }
            named_bar_sync(BAR_CONSUMERS, NCWARP * 32);
            acc = 0.0f;
        }
    }
}

template <int TYPE, int ACT, int EPI>
bool launch_tiled(const MvParams &base, int sms, cudaStream_t st) {
    using G = TileGeom<TYPE>;
    MvParams p = base;
    size_t act_bytes = (ACT == HOLO_ACT_Q8) ? (size_t)p.in_dim + 8 * (size_t)p.nblk32 : 4 * (size_t)p.nblk32;
    act_bytes = (act_bytes + 15) & ~(size_t)15;
    const size_t fixed = NCWARP * 32 * 4 + act_bytes;
    const size_t limit = 227 * 1024;
    int stages = 4;
    while (stages >= 2 && (size_t)stages * (G::TILE_FULL + 16) + fixed > limit) stages--;
    if (stages < 2) {
        holo_set_status(HOLO_E_UNSUPPORTED, "tiled matvec: in_dim too large for shared memory");
        return false;
    }
    p.stages = stages;
    size_t smem = (size_t)stages * (G::TILE_FULL + 16) + fixed;
    auto kern = mv_tiled_kernel<TYPE, ACT, EPI>;
    static int configured_dev[16] = {0};
    static size_t configured_bytes[16] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 16 && configured_bytes[dev] < smem) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)limit) != cudaSuccess) {
            holo_check_launch("tiled matvec: smem attribute");
            return false;
        }
        configured_bytes[dev] = limit;
        configured_dev[dev] = 1;
    }
    p.nctas = min(p.total_tiles, min(sms, MV_MAX_CTAS));
    kern<<<p.nctas, NTHREADS, smem, st>>>(p);
    return holo_check_launch("tiled matvec launch");
}

template <int TYPE>
bool dispatch_act(const MvParams &p, int act, bool add, int sms, cudaStream_t st) {
    if (act == HOLO_ACT_Q8)
        return add ? launch_tiled<TYPE, HOLO_ACT_Q8, EPI_ADD>(p, sms, st) : launch_tiled<TYPE, HOLO_ACT_Q8, EPI_STORE>(p, sms, st);
    return add ? launch_tiled<TYPE, HOLO_ACT_F32, EPI_ADD>(p, sms, st) : launch_tiled<TYPE, HOLO_ACT_F32, EPI_STORE>(p, sms, st);
}

}  // namespace

void holo_matvec_tiled(float *dst, const void *M, const WeightInfo &wi, const float *v,
                       int out_dim, int in_dim, int act_mode, const float *residual, cudaStream_t st) {
    HoloDevice *D = holo_dev();
    if (!D) return;
    if (wi.rows != out_dim || wi.cols != in_dim) {
        holo_set_status(HOLO_E_ARG, "matvec: shape differs from the uploaded weight");
        return;
    }
    MvParams p{};
    p.W = (const uint8_t *)M;
    p.x = v;
    p.y = dst;
    p.residual = residual;
    p.out_dim = out_dim;
    p.in_dim = in_dim;
    p.nblk32 = in_dim / 32;
    p.row_bytes = (size_t)gguf_row_bytes(wi.type, in_dim);
    p.nrb = wi.rows_padded / TILE_ROWS;
    p.partials = D->mv_partials;
    p.counters = D->mv_counters;
    p.status = D->status;
    if (p.nrb > MV_MAX_ROWBLOCKS) {
        holo_set_status(HOLO_E_UNSUPPORTED, "matvec: too many rows");
        return;
    }
    bool add = residual != nullptr;
    switch (wi.type) {
    case GT_Q8_0:
        p.blks_per_row = in_dim / 32;
        p.nkc = (p.blks_per_row + TileGeom<GT_Q8_0>::BLKS_PER_TILE - 1) / TileGeom<GT_Q8_0>::BLKS_PER_TILE;
        p.total_tiles = p.nrb * p.nkc;
        dispatch_act<GT_Q8_0>(p, act_mode, add, D->sms, st);
        break;
    case GT_Q4_0:
        p.blks_per_row = in_dim / 32;
        p.nkc = (p.blks_per_row + TileGeom<GT_Q4_0>::BLKS_PER_TILE - 1) / TileGeom<GT_Q4_0>::BLKS_PER_TILE;
        p.total_tiles = p.nrb * p.nkc;
        dispatch_act<GT_Q4_0>(p, act_mode, add, D->sms, st);
        break;
    case GT_Q4_K:
        p.blks_per_row = in_dim / 256;
        p.nkc = (p.blks_per_row + TileGeom<GT_Q4_K>::BLKS_PER_TILE - 1) / TileGeom<GT_Q4_K>::BLKS_PER_TILE;
        p.total_tiles = p.nrb * p.nkc;
        dispatch_act<GT_Q4_K>(p, act_mode, add, D->sms, st);
        break;
    default:
        holo_set_status(HOLO_E_ARG, "matvec: type has no tiled kernel");
    }
}
