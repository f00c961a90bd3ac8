// prefill.cu -- batched quantized matmul for prompt processing on the 5th-gen
// tensor cores: Y[M][N] = X[M][K] . W^T, W an N x K tiled Q4_K weight
// (cuda_upload_quant), X fp32, M tokens.
//
// The reference has no batched path: its prefill runs llm_forward one token at
// a time (src/ai/llm.c:1049, llm_cuda.c:574), i.e. M matvecs (cuda_ops.cu
// kernels 976-1060 for Q4_K).  Here the weight tile is dequantized once and
// multiplied against all M activation rows with tcgen05.mma:
//
//   * activations: each row quantized to Q8 per 32-block exactly as the
//     matvec does (d = amax/127, q = rint(x/d)), then the dequantized value
//     d*q rounded to fp16, written pre-swizzled in the tensor core's 128-byte
//     K-major layout (pf_act_kernel) so one 1-D bulk copy stages a tile;
//   * weights: 16 warps dequantize Q4_K (quant.c: y = (d*sc)*q - dmin*m, here
//     with d*sc and dmin*m rounded to fp16 and one fp16 fma per pair of
//     values) straight into the same swizzled layout in shared memory;
//   * one warp bulk-copies the activation tiles, another the raw weights;
//   * one thread issues tcgen05.mma.kind::f16 (fp32 accumulation in TMEM,
//     128 weight rows x TN tokens per CTA), tcgen05.commit frees each stage;
//   * the 16 warps read the accumulators back with tcgen05.ld.
// A CTA owns 128 weight rows, TN <= 256 tokens and a range of K; several K
// ranges (few weight tiles, e.g. 4096 x 14336) are summed by pf_reduce_kernel
// in a fixed order.  Every wait is bounded (HOLO_E_TIMEOUT).
#include "holo_common.cuh"
#include "mv_unit.cuh"
#include "tc_util.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>

namespace {

using namespace holo_mv;

constexpr int PF_BM = 128;                         // weight rows per CTA (MMA M)
static_assert(PF_BM == PF_ROWS_ALIGN, "row tile");
constexpr int PF_BK = 128;                         // K per stage: two 128-byte atoms of fp16
constexpr int PF_MAX_AST = 4;                      // dequantized weight stages, at most
constexpr int PF_A_COLS = PF_BK / 2;               // TMEM columns of one stage in TMEM (fp16 pairs)
constexpr int PF_DQ_WARPS = 16;                    // dequantize, then read the accumulators
constexpr int PF_B_WARP = PF_DQ_WARPS, PF_RAW_WARP = PF_DQ_WARPS + 1, PF_MMA_WARP = PF_DQ_WARPS + 2;
constexpr int PF_THREADS = (PF_DQ_WARPS + 3) * 32; // + activation copies + weight copies + MMA
constexpr int PF_A_BYTES = PF_BM * 256;            // one stage of weights: 32 KB (two atom columns)
constexpr int PF_RAW_BYTES = 4 * 4608;             // raw units of 128 rows (4 row-blocks), at most
constexpr int PF_MAX_RAW = 2;
constexpr int PF_MAX_BST = 4;

// raw super-blocks staged ahead in shared memory, and activation-tile stages:
// the activation tiles get their own, deeper ring (a tile is requested as soon
// as its slot is free, so its copy latency is hidden behind several stages)
// (AT: the dequantized weights go to TMEM, which frees the shared memory
// their stages took for deeper activation and raw-weight rings)
// (measured: deeper raw-weight rings -- 6 / 4 / 3 slots -- gained nothing at
// TN = 64 and lost 8 % at TN = 256, where the activation ring needs the room)
__host__ __device__ constexpr int pf_raw_slots(int tn, bool at) { return tn == 64 || (at && tn == 128) ? PF_MAX_RAW : 1; }
__host__ __device__ constexpr int pf_b_stages(int tn, bool at) {
    return tn == 64 ? 4 : tn == 128 ? (at ? 4 : 3) : (at ? 3 : 2);
}
// dequantized weight stages: the dequantizing warps run this many chunks
// ahead of the MMAs that free them
__host__ __device__ constexpr int pf_a_stages(int tn, bool at) { return at ? 4 : tn == 256 ? 2 : 3; }
// TMEM columns: the TN accumulator columns, then (AT) the weight stages
__host__ __device__ constexpr uint32_t pf_tmem_cols(int tn, bool at) { return at ? 512u : (uint32_t)tn; }
static_assert(256 + 4 * PF_A_COLS <= 512, "accumulator + weight stages fit TMEM");

struct PfBars {
    uint64_t full_a[PF_MAX_AST];  // the dequantizing warps arrived
    uint64_t empty[PF_MAX_AST];   // the weight stage's MMAs completed
    uint64_t full_b[PF_MAX_BST];  // activation tile landed
    uint64_t empty_b[PF_MAX_BST]; // the activation stage's MMAs completed
    uint64_t rfull[PF_MAX_RAW];   // raw super-block landed
    uint64_t rempty[PF_MAX_RAW];  // the dequantizing warps have read the raw super-block
    uint64_t done;                // the last MMA completed
    uint32_t tmem;                // accumulator base (TMEM address)
};

// ---- tcgen05 primitives: tc_util.cuh --------------------------------------
using namespace holo_tc;

// instruction descriptor: fp16 x fp16 -> fp32, both K-major, M = 128, N = tn
__host__ __device__ constexpr uint32_t pf_idesc(int tn) { return tc_idesc_f16(PF_BM, tn); }

// ---- activations: Q8 per 32-block, dequantized to fp16, tiled + swizzled ---
// xt = [K / 128 chunks][2 atom columns of 64 values][Mpad rows][128 bytes]:
// for a chunk and an atom column the rows are contiguous (and 128-byte
// swizzled in 8-row atoms), so any 8-aligned run of tokens is one 1-D bulk
// copy; rows past M are zero.  Four threads per (row, 32-block), 8 consecutive values each: two 16-byte
// loads, the block maximum over the four lanes, one 16-byte store (8 values
// are one 16-byte chunk of the swizzled layout).  Mpad * K / 8 threads, a
// multiple of 32, so every warp is whole.
__global__ void pf_act_kernel(__half *__restrict__ xt, const float *__restrict__ x, int M, int Mpad, int K,
                              int tn) {
    const int nb = K / 32;
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long g = t >> 2;   // (row, block)
    if (g >= (long long)Mpad * nb) return;
    const int m = (int)(g / nb), b = (int)(g % nb), sub = (int)(t & 3);
    float v[8];
    if (m < M) {
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)m * K + (size_t)b * 32 + 8 * sub);
        const float4 a = __ldg(src), c = __ldg(src + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.0f;
    }
    // quantize_act_q8's arithmetic: d = amax / 127, id = 1 / d, q = rint(v * id)
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    __align__(16) __half h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float q = fminf(fmaxf(rintf(__fmul_rn(v[j], id)), -127.0f), 127.0f);
        h[j] = __float2half_rn(__fmul_rn(d, q));
    }
    const int k = b * 32 + 8 * sub, kc = k / PF_BK, kk = k % PF_BK;
    uint8_t *col = reinterpret_cast<uint8_t *>(xt) + ((size_t)kc * 2 + (kk >> 6)) * (size_t)Mpad * 128;
    *reinterpret_cast<uint4 *>(col + sw128_off(m, kk & 63)) = *reinterpret_cast<const uint4 *>(h);
    (void)tn;
}

// Sum over the block, in the order of the batched RMSNorm's block_sum
// (sampler.cuh): a butterfly within each warp, then warp 0 over the warps.
__device__ __forceinline__ float pf_block_sum(float v, float *sv) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sv[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (int)(blockDim.x >> 5) ? sv[lane] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) sv[0] = v;
    }
    __syncthreads();
    v = sv[0];
    __syncthreads();
    return v;
}

// RMSNorm fused into pf_act_kernel (the projections that follow a norm):
// block m (1024 threads) = activation row m: sum of squares and scale exactly
// as bt_rmsnorm_kernel (rms_norm, tensor.c:242-255), x * scale * w, then the
// Q8 quantization and the swizzled 16-byte stores of pf_act_kernel; rows
// past M are zero.  Every lane of a warp runs each round (the 4-lane
// shuffles), idle lanes compute on zeros and store nothing.
__global__ void __launch_bounds__(1024) pf_act_norm_kernel(__half *__restrict__ xt, const float *__restrict__ x,
                                                           const float *__restrict__ w, float eps, int M, int Mpad,
                                                           int K) {
    __shared__ float sv[32];
    const int m = blockIdx.x, ng = K / 8;
    float scale = 0.0f;
    if (m < M) {
        const float *xr = x + (size_t)m * K;
        float ss = 0.0f;
        for (int i = threadIdx.x; i < K; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
        ss = pf_block_sum(ss, sv);
        scale = 1.0f / sqrtf(ss / (float)K + eps);
    }
    for (int g0 = 0; g0 < ng; g0 += blockDim.x) {
        const int g = g0 + threadIdx.x;   // 8-value group; a 32-block is 4 consecutive lanes
        const bool live = g < ng;
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.0f;
        if (live && m < M) {
            const float *xr = x + (size_t)m * K + 8 * g;
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = xr[j] * scale * w[8 * g + j];
        }
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        __align__(16) __half h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float q = fminf(fmaxf(rintf(__fmul_rn(v[j], id)), -127.0f), 127.0f);
            h[j] = __float2half_rn(__fmul_rn(d, q));
        }
        if (live) {
            const int k = 8 * g, kc = k / PF_BK, kk = k % PF_BK;
            uint8_t *col = reinterpret_cast<uint8_t *>(xt) + ((size_t)kc * 2 + (kk >> 6)) * (size_t)Mpad * 128;
            *reinterpret_cast<uint4 *>(col + sw128_off(m, kk & 63)) = *reinterpret_cast<const uint4 *>(h);
        }
    }
}

// ---- weight dequantization (one thread: one row, 32 positions of a chunk) ---
// The raw unit of the thread's row-block in shared memory -> the registers a
// unit needs: the row's head and two 16-byte planes.
template <int TYPE>
__device__ __forceinline__ void dq_load(const uint8_t *unit, int lr, int q, uint4 &h, uint4 &p0, uint4 &p1) {
    if constexpr (TYPE == GT_Q8_0) {
        // one 128-value chunk a unit; block q = planes 2q (positions 0..15), 2q+1
        const uint2 hh = *reinterpret_cast<const uint2 *>(unit + unit_head_off<GT_Q8_0>(lr));
        h = make_uint4(hh.x, hh.y, 0u, 0u);
        p0 = lds128(unit + unit_plane_off<GT_Q8_0>(2 * q, lr));
        p1 = lds128(unit + unit_plane_off<GT_Q8_0>(2 * q + 1, lr));
    } else {
        // two chunks a unit; chunk c2 holds sub-blocks 4 c2 .. 4 c2 + 3
        h = lds128(unit + unit_head_off<TYPE>(lr));
        p0 = lds128(unit + unit_plane_off<TYPE>(q, lr));
        p1 = lds128(unit + unit_plane_off<TYPE>(4 + q, lr));
    }
}

// the 32 values (fp16, 4 x 16 bytes: positions 8 cc .. 8 cc + 7) of block
// 4 c2 + q of the unit: Q4_K (d*sc)*q - dmin*m (quant.c:290-297 scale
// unpack; sc, m rounded to fp16, one fp16 fma), Q4_0 d*(q - 8), Q8_0 d*q
// (one rounding each).  Nibble pairs: bytes (2e, 2e+1) of a word moved to
// the two halves by a permute, 0x6400 | n read as fp16 is 1024 + n.
template <int TYPE>
__device__ __forceinline__ void dq_block(const uint4 &h, const uint4 &p0, const uint4 &p1, int c2, int q,
                                         uint4 (&outv)[4]) {
    __half2 mul2, add2, off2;
    uint4 qw = c2 ? p1 : p0;
    if constexpr (TYPE == GT_Q4_K) {
        const float d = half_bits_to_float(h.x & 0xffffu), dmin = half_bits_to_float(h.x >> 16);
        const uint32_t scw = c2 ? (((h.w & LO4) << 2) | ((h.y >> 6) & 0x03030303u)) : (h.y & 0x3F3F3F3Fu);
        const uint32_t mw = c2 ? ((((h.w >> 4) & LO4) << 2) | ((h.z >> 6) & 0x03030303u)) : (h.z & 0x3F3F3F3Fu);
        mul2 = __float2half2_rn(__fmul_rn(d, ubyte_to_float(scw, q)));
        add2 = __float2half2_rn(-__fmul_rn(dmin, ubyte_to_float(mw, q)));
        off2 = __float2half2_rn(1024.0f);
    } else if constexpr (TYPE == GT_Q4_0) {
        mul2 = __float2half2_rn(head_half(h, 4 * c2 + q));   // an fp16 scale: exact
        add2 = __float2half2_rn(0.0f);
        off2 = __float2half2_rn(1032.0f);   // 1024 + the Q4_0 offset 8
    } else {
        mul2 = __float2half2_rn(head_half(h, q));   // an fp16 scale: exact
        add2 = __float2half2_rn(0.0f);
        off2 = __float2half2_rn(1152.0f);   // 1024 + 128: the sign bit is flipped below
        (void)qw;
    }
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
        uint32_t w0, w1;
        if constexpr (TYPE == GT_Q8_0) {
            const uint4 pl = (cc & 2) ? p1 : p0;   // positions 0..15 | 16..31
            w0 = (cc & 1) ? pl.z : pl.x;
            w1 = (cc & 1) ? pl.w : pl.y;
        } else {
            w0 = (cc & 1) ? qw.z : qw.x;
            w1 = (cc & 1) ? qw.w : qw.y;
        }
        uint32_t packed[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            uint32_t tt = __byte_perm(e < 2 ? w0 : w1, 0u, (e & 1) ? 0x4342u : 0x4140u);
            uint32_t hb;
            if constexpr (TYPE == GT_Q8_0) {
                hb = (tt ^ 0x00800080u) | 0x64006400u;   // int8 + 128 in the low byte of each half
            } else {
                if (cc & 2) tt >>= 4;
                hb = (tt & 0x000F000Fu) | 0x64006400u;
            }
            const __half2 qh = __hsub2(*reinterpret_cast<const __half2 *>(&hb), off2);
            const __half2 hv = TYPE == GT_Q4_K ? __hfma2(qh, mul2, add2) : __hmul2(qh, mul2);
            packed[e] = *reinterpret_cast<const uint32_t *>(&hv);
        }
        outv[cc] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
}

// ---- the matmul ----------------------------------------------------------------
// out[ks][M][N] (ks = blockIdx.z, K chunks [kc0, kc1)); W tiled TYPE with
// `units` units a row.  AT: the dequantizing warps store the weight tile into
// TMEM (tcgen05.st; row r = lane r, columns TN + 64 s ..) and the MMAs read A
// from there, so the only operand the tensor core reads from shared memory is
// the activation tile: a stage in shared memory costs the tile's write, its
// read by the MMAs and the staging of the activations -- the shared-memory
// bandwidth that bounded the first version.
template <int TYPE, int TN, bool AT>
__global__ void __launch_bounds__(PF_THREADS, 1)
pf_mma_kernel(float *__restrict__ out, const uint8_t *__restrict__ W, const uint8_t *__restrict__ xt, int M, int Mpad,
              int N, int K, int units, int kc_per_split, int *status) {
    extern __shared__ uint8_t pf_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)pf_smem_raw + 1023) & ~(uintptr_t)1023);
    constexpr int PF_STAGES = pf_a_stages(TN, AT), SB = pf_b_stages(TN, AT), R = pf_raw_slots(TN, AT);
    constexpr uint32_t TCOLS = pf_tmem_cols(TN, AT);
    uint8_t *sa = smem;                                   // !AT: [stages][2 atom columns][128 rows][128 B]
    uint8_t *sb = smem + (AT ? 0 : PF_STAGES * PF_A_BYTES);   // [SB][2 atom columns][TN rows][128 B]
    uint8_t *sr = sb + SB * TN * 256;                     // [R][4 row-blocks][UB]
    constexpr int UB = UnitGeom<TYPE>::UNIT_BYTES, CPU = UnitGeom<TYPE>::VALS / PF_BK;   // chunks a unit
    PfBars &B = *reinterpret_cast<PfBars *>(sr + R * PF_RAW_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkc = K / PF_BK;
    const int n0 = blockIdx.x * PF_BM, mt = blockIdx.y, ks = blockIdx.z;
    const int kc0 = ks * kc_per_split, kc1 = min(nkc, kc0 + kc_per_split);
    const int nch = kc1 - kc0;   // >= 1 by construction

    if (threadIdx.x == 0) {
        for (int s = 0; s < PF_STAGES; ++s) {
            mbar_init(&B.full_a[s], PF_DQ_WARPS);
            mbar_init(&B.empty[s], 1);
        }
        for (int s = 0; s < PF_MAX_BST; ++s) {
            mbar_init(&B.full_b[s], 1);
            mbar_init(&B.empty_b[s], 1);
        }
        for (int k = 0; k < PF_MAX_RAW; ++k) {
            mbar_init(&B.rfull[k], 1);
            mbar_init(&B.rempty[k], PF_DQ_WARPS);
        }
        mbar_init(&B.done, 1);
        fence_barrier_init();
    }
    if (warp == PF_MMA_WARP) tc_alloc(&B.tmem, TCOLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = B.tmem;

    if (warp < PF_DQ_WARPS) {
        // thread -> weight row r and block q of the 4 32-value blocks a
        // 128-value chunk holds (all 32 positions).  The raw units arrive in
        // shared memory R ahead (bulk copies).
        const int t = threadIdx.x, r = t & (PF_BM - 1), q = t >> 7, lr = r & 31;
        const int nun = nch / CPU;   // K ranges are whole units
        bool ok = true;
        for (int b = 0; b < nun && ok; ++b) {
            const int rs = b % R;
            ok = mbar_wait_bounded(&B.rfull[rs], (b / R) & 1, status, HOLO_E_TIMEOUT);
            ok = __all_sync(0xffffffffu, ok);   // the warp leaves together
                if (!ok) break;
            uint4 h, p0, p1;
            dq_load<TYPE>(sr + rs * PF_RAW_BYTES + (r >> 5) * UB, lr, q, h, p0, p1);
            __syncwarp();
            if (lane == 0) mbar_arrive(&B.rempty[rs]);   // the copy of unit b + R may land
#pragma unroll
            for (int c2 = 0; c2 < CPU; ++c2) {
                const int i = CPU * b + c2, s = i % PF_STAGES;
                uint4 outv[4];
                dq_block<TYPE>(h, p0, p1, c2, q, outv);
                if (i >= PF_STAGES)
                    ok = mbar_wait_bounded(&B.empty[s], ((i / PF_STAGES) + 1) & 1, status, HOLO_E_TIMEOUT);
                ok = __all_sync(0xffffffffu, ok);   // the warp leaves together
                if (!ok) break;
                if constexpr (AT) {
                    // the stage's previous MMAs completed (empty[s]); order this
                    // thread's TMEM stores after that wait
                    tc_fence_after();
                    // lane r, columns TN + 64 s + 16 q ..: positions 32 q .. 32 q + 31 in pairs
                    uint32_t v[16];
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        v[4 * cc] = outv[cc].x;
                        v[4 * cc + 1] = outv[cc].y;
                        v[4 * cc + 2] = outv[cc].z;
                        v[4 * cc + 3] = outv[cc].w;
                    }
                    tc_st16(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(TN + s * PF_A_COLS + 16 * q), v);
                    tc_fence_before();   // the MMA thread reads the stage after the barrier
                } else {
                    // column 32 q + position of the chunk: atom column q / 2
                    uint8_t *acol = sa + s * PF_A_BYTES + (q >> 1) * (PF_BM * 128);
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc)
                        *reinterpret_cast<uint4 *>(acol + sw128_off(r, 32 * (q & 1) + 8 * cc)) = outv[cc];
                    fence_proxy_async_smem();   // the tensor core reads these through the async proxy
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&B.full_a[s]);
            }
        }
        // accumulators -> out: warp w reads TMEM lanes 32 (w % 4).., a
        // quarter of the columns
        ok = __all_sync(0xffffffffu, ok && mbar_wait_bounded(&B.done, 0, status, HOLO_E_TIMEOUT));
        tc_fence_after();
        if (ok) {
            const int quarter = warp & 3, colq = warp >> 2;
            const int row = n0 + 32 * quarter + lane;
            float *o = out + (size_t)ks * M * N;
            for (int cb = colq * (TN / 4); cb < (colq + 1) * (TN / 4); cb += 16) {
                uint32_t v[16];
                tc_ld16(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)cb, v);
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) {
                    const int m = mt * TN + cb + jj;
                    if (m < M && row < N) o[(size_t)m * N + row] = __uint_as_float(v[jj]);
                }
            }
        }
    } else if (warp == PF_B_WARP) {
        // activation tiles, one bulk copy a stage, SB stages ahead
        if (lane == 0) {
            // rows [mt * TN, +TN) of both atom columns of chunk kc0 + i
            const uint8_t *xb = xt + (size_t)mt * TN * 128;
            int issued = 0;
            for (int i = 0; i < nch; ++i) {
                const int s = i % SB;
                if (i >= SB && !mbar_wait_bounded(&B.empty_b[s], ((i / SB) + 1) & 1, status, HOLO_E_TIMEOUT))
                    break;
                mbar_arrive_expect_tx(&B.full_b[s], (uint32_t)(TN * 256));
#pragma unroll
                for (int a = 0; a < 2; ++a)
                    bulk_copy_g2s(sb + (size_t)s * TN * 256 + (size_t)a * TN * 128,
                                  xb + ((size_t)(kc0 + i) * 2 + a) * (size_t)Mpad * 128, (uint32_t)(TN * 128),
                                  &B.full_b[s]);
                issued = i + 1;
            }
            // every copy has landed before the CTA ends (the MMA thread may
            // have stopped consuming on a time-out)
            for (int i = max(0, issued - SB); i < issued; ++i)
                mbar_wait_bounded(&B.full_b[i % SB], (i / SB) & 1, nullptr, 0);
        }
    } else if (warp == PF_RAW_WARP) {
        // raw weight units (4 row-blocks each), R ahead of the dequantizing warps
        if (lane == 0) {
            const int nun = nch / CPU, u0 = kc0 / CPU;
            const uint8_t *wrb = W + (size_t)(n0 >> 5) * units * UB;   // the CTA's first row-block
            // a last, partial tile holds fewer row-blocks: the missing ones are
            // not loaded, their rows of the product are not stored
            const int nq = min(4, (N + 31) / 32 - (n0 >> 5));
            int issued = 0;
            for (int b = 0; b < nun; ++b) {
                const int rs = b % R;
                if (b >= R && !mbar_wait_bounded(&B.rempty[rs], ((b / R) + 1) & 1, status, HOLO_E_TIMEOUT)) break;
                mbar_arrive_expect_tx(&B.rfull[rs], (uint32_t)(nq * UB));
                for (int q = 0; q < nq; ++q)
                    bulk_copy_g2s(sr + rs * PF_RAW_BYTES + q * UB, wrb + ((size_t)q * units + u0 + b) * UB,
                                  (uint32_t)UB, &B.rfull[rs]);
                issued = b + 1;
            }
            for (int b = max(0, issued - R); b < issued; ++b)
                mbar_wait_bounded(&B.rfull[b % R], (b / R) & 1, nullptr, 0);
        }
    } else {
        // MMA issue: 8 K-steps of 16 a stage (4 in each atom column)
        if (lane == 0) {
            constexpr uint32_t idesc = pf_idesc(TN);
            // descriptors of stage 0; a stage, atom column and K step move the
            // start address (the low field, in 16-byte units) by constants
            const uint64_t a0 = sw128_desc(sa), b0 = sw128_desc(sb);
            bool ok = true;
            for (int i = 0; i < nch && ok; ++i) {
                const int s = i % PF_STAGES, t = i % SB;
                ok = mbar_wait_bounded(&B.full_a[s], (i / PF_STAGES) & 1, status, HOLO_E_TIMEOUT) &&
                     mbar_wait_bounded(&B.full_b[t], (i / SB) & 1, status, HOLO_E_TIMEOUT);
                if (!ok) break;
                tc_fence_after();
                const uint64_t bd = b0 + (uint64_t)((t * TN * 256) >> 4);
                if constexpr (AT) {
                    // K step kk: 16 values = 8 columns of the stage
                    const uint32_t ta = tmem + (uint32_t)(TN + s * PF_A_COLS);
#pragma unroll
                    for (int kk = 0; kk < PF_BK / 16; ++kk)
                        tc_mma_ts(tmem, ta + (uint32_t)(8 * kk),
                                  bd + (uint64_t)(((kk >> 2) * (TN * 128) + (kk & 3) * 32) >> 4), idesc, (i | kk) != 0);
                } else {
                    const uint64_t ad = a0 + (uint64_t)((s * PF_A_BYTES) >> 4);
#pragma unroll
                    for (int kk = 0; kk < PF_BK / 16; ++kk)
                        tc_mma(tmem, ad + (uint64_t)(((kk >> 2) * (PF_BM * 128) + (kk & 3) * 32) >> 4),
                               bd + (uint64_t)(((kk >> 2) * (TN * 128) + (kk & 3) * 32) >> 4), idesc, (i | kk) != 0);
                }
                tc_commit(&B.empty[s]);
                tc_commit(&B.empty_b[t]);
            }
            // completes once every MMA issued above has (or at once if none was)
            tc_commit(&B.done);
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == PF_MMA_WARP) {
        tc_fence_after();
        tc_dealloc(tmem, TCOLS);
    }
}

// ---- the matmul on a persistent token-range schedule --------------------------
// The tile grid above runs (row tiles x token tiles x K splits) CTAs; when
// that is not a whole number of waves (224 tiles on 148 SMs at M = 512, 172
// at the W1/W3 projection of a 127-token prompt) the last wave leaves SMs
// idle.  Here the same work is cut along the tokens instead: the space of
// (K split, 128-row weight tile, 16-token group) is flattened and every CTA
// takes an equal contiguous share, in pieces of up to 256 tokens of one
// weight tile.  Each output element is still the full K range of its split
// accumulated in one TMEM accumulator, chunk by chunk in K order, so the
// result does not depend on the schedule.  Between pieces the accumulator is
// drained by the 16 warps (acc_free) before the MMA thread starts the next.
// Measured slower than the tile grid at every prefill shape (M = 512:
// 92 vs 63 us; M = 64: 58 vs 29 us; a 7B 127-token prompt: 7.25 vs 6.15 ms):
// every piece dequantizes its weight tile over the whole K range, and the
// pieces average far fewer tokens than a 256-token tile, so the extra
// dequantization outweighs the idle SMs of the last wave.  Kept selectable
// (HOLO_PREFILL_SCHED=seg) with its bit-identity test; a K-wise split of the
// last wave (partial accumulators, fixed-order sum) is the remaining option.
constexpr int SG_TN = 256;        // token capacity of a piece (accumulator columns)
constexpr int SG_STAGES = 4, SG_B = 2, SG_R = 1;   // 2 activation stages: see holo_matmul_batched

struct SegBars {
    uint64_t full_a[SG_STAGES], empty[SG_STAGES];
    uint64_t full_b[SG_B], empty_b[SG_B];
    uint64_t rfull[SG_R], rempty[SG_R];
    uint64_t done, acc_free;
    uint32_t tmem;
};

// the pieces of one CTA's share [f, f1) of the flattened group space
struct SegWalk {
    long long f, f1;
    int g16, nt;
    __device__ __forceinline__ bool next(int &ks, int &n0, int &t0, int &ng) {
        if (f >= f1) return false;
        const long long item = f / g16;
        const long long end = min(f1, (item + 1) * (long long)g16);
        ng = (int)min((long long)(SG_TN / 16), end - f);
        ks = (int)(item / nt);
        n0 = (int)(item % nt) * PF_BM;
        t0 = 16 * (int)(f % g16);
        f += ng;
        return true;
    }
};

template <int TYPE>
__global__ void __launch_bounds__(PF_THREADS, 1)
pf_seg_kernel(float *__restrict__ out, const uint8_t *__restrict__ W, const uint8_t *__restrict__ xt, int M, int Mpad,
              int N, int K, int units, int kc_per_split, int g16, long long total, int *status) {
    extern __shared__ uint8_t pf_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)pf_smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sb = smem;                                   // [SG_B][2 atom columns][SG_TN rows][128 B]
    uint8_t *sr = sb + SG_B * SG_TN * 256;                // [SG_R][4 row-blocks][UB]
    constexpr int UB = UnitGeom<TYPE>::UNIT_BYTES, CPU = UnitGeom<TYPE>::VALS / PF_BK;
    SegBars &B = *reinterpret_cast<SegBars *>(sr + SG_R * PF_RAW_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkc = K / PF_BK, nt = (N + PF_BM - 1) / PF_BM;
    const long long f0 = total * blockIdx.x / gridDim.x, f1 = total * (blockIdx.x + 1) / gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SG_STAGES; ++s) {
            mbar_init(&B.full_a[s], PF_DQ_WARPS);
            mbar_init(&B.empty[s], 1);
        }
        for (int s = 0; s < SG_B; ++s) {
            mbar_init(&B.full_b[s], 1);
            mbar_init(&B.empty_b[s], 1);
        }
        for (int k = 0; k < SG_R; ++k) {
            mbar_init(&B.rfull[k], 1);
            mbar_init(&B.rempty[k], PF_DQ_WARPS);
        }
        mbar_init(&B.done, 1);
        mbar_init(&B.acc_free, PF_DQ_WARPS);
        fence_barrier_init();
    }
    if (warp == PF_MMA_WARP) tc_alloc(&B.tmem, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = B.tmem;
    SegWalk walk{f0, f1, g16, nt};
    int ks, n0, t0, ng;

    if (warp < PF_DQ_WARPS) {
        // as pf_mma_kernel: thread -> weight row r, 32-value block q of a chunk
        const int t = threadIdx.x, r = t & (PF_BM - 1), q = t >> 7, lr = r & 31;
        bool ok = true;
        int bg = 0, ig = 0, piece = 0;   // raw units, chunks, pieces so far
        while (ok && walk.next(ks, n0, t0, ng)) {
            const int kc0 = ks * kc_per_split, nun = (min(nkc, kc0 + kc_per_split) - kc0) / CPU;
            for (int b = 0; b < nun && ok; ++b, ++bg) {
                const int rs = bg % SG_R;
                ok = mbar_wait_bounded(&B.rfull[rs], (bg / SG_R) & 1, status, HOLO_E_TIMEOUT);
                ok = __all_sync(0xffffffffu, ok);   // the warp leaves together
                if (!ok) break;
                uint4 h, p0, p1;
                dq_load<TYPE>(sr + rs * PF_RAW_BYTES + (r >> 5) * UB, lr, q, h, p0, p1);
                __syncwarp();
                if (lane == 0) mbar_arrive(&B.rempty[rs]);
#pragma unroll
                for (int c2 = 0; c2 < CPU; ++c2) {
                    const int s = ig % SG_STAGES;
                    uint4 outv[4];
                    dq_block<TYPE>(h, p0, p1, c2, q, outv);
                    if (ig >= SG_STAGES)
                        ok = mbar_wait_bounded(&B.empty[s], ((ig / SG_STAGES) + 1) & 1, status, HOLO_E_TIMEOUT);
                    ok = __all_sync(0xffffffffu, ok);   // the warp leaves together
                if (!ok) break;
                    tc_fence_after();   // after the empty[s] wait, before the stores (as pf_mma_kernel)
                    uint32_t v[16];
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        v[4 * cc] = outv[cc].x;
                        v[4 * cc + 1] = outv[cc].y;
                        v[4 * cc + 2] = outv[cc].z;
                        v[4 * cc + 3] = outv[cc].w;
                    }
                    tc_st16(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(SG_TN + s * PF_A_COLS + 16 * q), v);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&B.full_a[s]);
                    ++ig;
                }
            }
            // the piece's accumulators -> out: warp w reads TMEM lanes
            // 32 (w % 4).., every fourth 16-column block
            ok = __all_sync(0xffffffffu, ok && mbar_wait_bounded(&B.done, piece & 1, status, HOLO_E_TIMEOUT));
            tc_fence_after();
            if (ok) {
                const int quarter = warp & 3, colq = warp >> 2, n16 = 16 * ng;
                const int row = n0 + 32 * quarter + lane;
                float *o = out + (size_t)ks * M * N;
                for (int cb = 16 * colq; cb < n16; cb += 64) {
                    uint32_t v[16];
                    tc_ld16(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)cb, v);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int m = t0 + cb + jj;
                        if (m < M && row < N) o[(size_t)m * N + row] = __uint_as_float(v[jj]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&B.acc_free);   // the MMA thread may overwrite the accumulator
            ++piece;
        }
    } else if (warp == PF_B_WARP) {
        if (lane == 0) {
            int ig = 0;
            bool ok = true;
            while (ok && walk.next(ks, n0, t0, ng)) {
                const int kc0 = ks * kc_per_split, nch = min(nkc, kc0 + kc_per_split) - kc0;
                const uint32_t bytes = (uint32_t)(16 * ng * 128);
                for (int i = 0; i < nch; ++i, ++ig) {
                    const int s = ig % SG_B;
                    if (ig >= SG_B && !mbar_wait_bounded(&B.empty_b[s], ((ig / SG_B) + 1) & 1, status, HOLO_E_TIMEOUT)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&B.full_b[s], 2 * bytes);
#pragma unroll
                    for (int a = 0; a < 2; ++a)
                        bulk_copy_g2s(sb + (size_t)s * SG_TN * 256 + (size_t)a * SG_TN * 128,
                                      xt + (((size_t)(kc0 + i) * 2 + a) * (size_t)Mpad + t0) * 128, bytes, &B.full_b[s]);
                }
            }
            for (int j = max(0, ig - SG_B); j < ig; ++j) mbar_wait_bounded(&B.full_b[j % SG_B], (j / SG_B) & 1, nullptr, 0);
        }
    } else if (warp == PF_RAW_WARP) {
        if (lane == 0) {
            int bg = 0;
            bool ok = true;
            while (ok && walk.next(ks, n0, t0, ng)) {
                const int kc0 = ks * kc_per_split, nun = (min(nkc, kc0 + kc_per_split) - kc0) / CPU, u0 = kc0 / CPU;
                const uint8_t *wrb = W + (size_t)(n0 >> 5) * units * UB;
                const int nq = min(4, (N + 31) / 32 - (n0 >> 5));
                for (int b = 0; b < nun; ++b, ++bg) {
                    const int rs = bg % SG_R;
                    if (bg >= SG_R && !mbar_wait_bounded(&B.rempty[rs], ((bg / SG_R) + 1) & 1, status, HOLO_E_TIMEOUT)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&B.rfull[rs], (uint32_t)(nq * UB));
                    for (int qq = 0; qq < nq; ++qq)
                        bulk_copy_g2s(sr + rs * PF_RAW_BYTES + qq * UB, wrb + ((size_t)qq * units + u0 + b) * UB,
                                      (uint32_t)UB, &B.rfull[rs]);
                }
            }
            for (int b = max(0, bg - SG_R); b < bg; ++b) mbar_wait_bounded(&B.rfull[b % SG_R], (b / SG_R) & 1, nullptr, 0);
        }
    } else {
        if (lane == 0) {
            const uint64_t b0 = sw128_desc(sb);
            bool ok = true;
            int ig = 0, piece = 0;
            while (ok && walk.next(ks, n0, t0, ng)) {
                const int kc0 = ks * kc_per_split, nch = min(nkc, kc0 + kc_per_split) - kc0;
                const uint32_t idesc = tc_idesc_f16(PF_BM, 16 * ng);
                if (piece > 0) {
                    ok = mbar_wait_bounded(&B.acc_free, (piece - 1) & 1, status, HOLO_E_TIMEOUT);
                    tc_fence_after();
                }
                for (int i = 0; i < nch && ok; ++i, ++ig) {
                    const int s = ig % SG_STAGES, tb = ig % SG_B;
                    ok = mbar_wait_bounded(&B.full_a[s], (ig / SG_STAGES) & 1, status, HOLO_E_TIMEOUT) &&
                         mbar_wait_bounded(&B.full_b[tb], (ig / SG_B) & 1, status, HOLO_E_TIMEOUT);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t bd = b0 + (uint64_t)((tb * SG_TN * 256) >> 4);
                    const uint32_t ta = tmem + (uint32_t)(SG_TN + s * PF_A_COLS);
#pragma unroll
                    for (int kk = 0; kk < PF_BK / 16; ++kk)
                        tc_mma_ts(tmem, ta + (uint32_t)(8 * kk),
                                  bd + (uint64_t)(((kk >> 2) * (SG_TN * 128) + (kk & 3) * 32) >> 4), idesc, (i | kk) != 0);
                    tc_commit(&B.empty[s]);
                    tc_commit(&B.empty_b[tb]);
                }
                tc_commit(&B.done);   // the piece's MMAs (at once if none was issued)
                ++piece;
            }
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == PF_MMA_WARP) {
        tc_fence_after();
        tc_dealloc(tmem, 512);
    }
}

constexpr size_t SG_SMEM = 1024 + (size_t)SG_B * SG_TN * 256 + (size_t)SG_R * PF_RAW_BYTES + sizeof(SegBars);

template <int TYPE>
bool launch_seg(float *out, const uint8_t *W, const uint8_t *xt, int M, int Mpad, int N, int K, int units,
                int kc_per_split, int g16, long long total, int grid, int *status, cudaStream_t st) {
    static int configured = -1;
    const int dev = holo_dev() ? holo_dev()->id : -1;
    if (configured != dev) {
        if (cudaFuncSetAttribute(pf_seg_kernel<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SG_SMEM) !=
            cudaSuccess)
            return holo_check_launch("prefill: attributes");
        configured = dev;
    }
    pf_seg_kernel<TYPE><<<grid, PF_THREADS, SG_SMEM, st>>>(out, W, xt, M, Mpad, N, K, units, kc_per_split, g16, total,
                                                         status);
    return holo_check_launch("prefill matmul (token-range schedule)");
}

// y[m][n] = sum over ks of part[ks][m][n], in ks order; RESID: y[i] += that
// sum (a residual stream updated in place, the arithmetic of computing the
// sum into a buffer and adding it after)
template <bool RESID>
__global__ void pf_reduce_kernel(float *__restrict__ y, const float *__restrict__ part, long long mn, int splits) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < mn; i += (long long)gridDim.x * blockDim.x) {
        float s = part[i];
        for (int k = 1; k < splits; ++k) s += part[(size_t)k * mn + i];
        if (RESID) y[i] = y[i] + s;
        else y[i] = s;
    }
}

// y[i] += t[i] (the residual add after a matmul that was not K-split)
__global__ void pf_add_kernel(float *__restrict__ y, const float *__restrict__ t, long long mn) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < mn; i += (long long)gridDim.x * blockDim.x)
        y[i] += t[i];
}

size_t pf_smem(int tn, bool at) {
    return 1024 + (at ? 0 : (size_t)pf_a_stages(tn, at) * PF_A_BYTES) + (size_t)pf_b_stages(tn, at) * tn * 256 +
           (size_t)pf_raw_slots(tn, at) * PF_RAW_BYTES + sizeof(PfBars);
}

template <int TYPE, int TN, bool AT>
bool launch_mma(float *out, const uint8_t *W, const uint8_t *xt, int M, int Mpad, int N, int K, int units, int splits,
                int kc_per_split, int mtiles, int *status, cudaStream_t st) {
    const size_t smem = pf_smem(TN, AT);
    static int configured = -1;   // the device the attribute was set for
    const int dev = holo_dev() ? holo_dev()->id : -1;
    if (configured != dev) {
        if (cudaFuncSetAttribute(pf_mma_kernel<TYPE, TN, AT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return holo_check_launch("prefill: attributes");
        configured = dev;
    }
    pf_mma_kernel<TYPE, TN, AT><<<dim3((N + PF_BM - 1) / PF_BM, mtiles, splits), PF_THREADS, smem, st>>>(out, W, xt, M, Mpad, N, K, units,
                                                                                kc_per_split, status);
    return holo_check_launch("prefill matmul");
}

}  // namespace

namespace {

// dequantized weight tiles in TMEM (default) or in shared memory
// (HOLO_PREFILL_A=smem, the first version, kept for comparison)
bool pf_weights_in_tmem() {
    static const bool at = [] {
        const char *e = getenv("HOLO_PREFILL_A");
        return !(e && strcmp(e, "smem") == 0);
    }();
    return at;
}

// the schedule: the tile grid (default) or the token-range schedule
// (HOLO_PREFILL_SCHED=seg, kept for comparison: measured slower, see
// pf_seg_kernel)
bool pf_sched_seg() {
    static const bool v = [] {
        const char *e = getenv("HOLO_PREFILL_SCHED");
        return e && strcmp(e, "seg") == 0;
    }();
    return v;
}

// the launch plan of one batched matmul: token tile, K splits, scratch bytes,
// and the schedule (seg: token-range pieces on `grid` CTAs over `total`
// (split, row tile, 16-token group) units)
struct PfPlan {
    int tn, mtiles, Mpad, splits, kc_per_split;
    size_t xt_bytes, part_bytes;
    bool seg;
    int grid, g16;
    long long total;
};

PfPlan pf_plan(const WeightInfo &wi, int M, int sms, int plan_rows) {
    PfPlan p;
    const int N = wi.rows, K = wi.cols, vals = wi.type == GT_Q8_0 ? 128 : 256;
    const int NP = plan_rows > 0 ? plan_rows : N;   // rows the K split is planned for
    p.tn = M <= 64 ? 64 : M <= 128 ? 128 : 256;
    p.mtiles = (M + p.tn - 1) / p.tn;
    p.Mpad = p.mtiles * p.tn;
    const int nkc = K / PF_BK, cpu = vals / PF_BK;
    // K splits (whole units) so that the CTAs cover the SMs when the weight
    // has few row tiles
    const int base = (NP + PF_BM - 1) / PF_BM * p.mtiles;
    p.splits = std::max(1, std::min(nkc / 4, sms / base));
    p.kc_per_split = ((nkc + p.splits - 1) / p.splits + cpu - 1) / cpu * cpu;
    p.splits = (nkc + p.kc_per_split - 1) / p.kc_per_split;   // every split non-empty
    p.xt_bytes = ((size_t)p.Mpad * K * 2 + 255) & ~(size_t)255;
    p.part_bytes = p.splits > 1 ? (size_t)p.splits * M * N * 4 : 0;
    // the token-range schedule (numerics do not depend on it): the same
    // (split, row tile, 16-token group) work spread evenly over the SMs
    const int nt = (N + PF_BM - 1) / PF_BM;
    p.g16 = (M + 15) / 16;
    p.total = (long long)p.splits * nt * p.g16;
    p.grid = (int)std::min<long long>(sms, p.total);
    p.seg = pf_weights_in_tmem() && pf_sched_seg();
    return p;
}

}  // namespace

size_t holo_matmul_batched_scratch(const WeightInfo &wi, int M, int plan_rows) {
    if (M <= MVB_MAX_M) return holo_matmul_few_scratch(wi, M);
    HoloDevice *D = holo_dev();
    const PfPlan p = pf_plan(wi, M, D ? D->sms : 148, plan_rows);
    return p.xt_bytes + p.part_bytes;
}

// Y[M][N] = X[M][K] . W^T for a tiled weight described by wi, on stream st
// (the ABI entry below and the batched decode engine).  scratch: the caller's
// buffer of scratch_bytes (at least holo_matmul_batched_scratch), or NULL for
// the library's shared one.
bool holo_matmul_batched(float *Y, const void *W, const WeightInfo &wi, const float *X, int M, cudaStream_t st,
                         void *scratch, size_t scratch_bytes, int plan_rows, const float *norm_w, float norm_eps,
                         float *resid) {
    // a few rows: the CUDA-core kernel that reads each weight unit once for all
    // of them (matvec_batch.cu); a tensor-core tile would be mostly padding
    if (M > 0 && M <= MVB_MAX_M) {
        if (norm_w || resid) {
            holo_set_status(HOLO_E_ARG, "batched matmul: the fused RMSNorm / residual need more than 16 rows");
            return false;
        }
        return holo_matmul_few(Y, W, wi, X, M, st, scratch, scratch_bytes);
    }
    HoloDevice *D = holo_dev();
    if (!D) return false;
    const int N = wi.rows, K = wi.cols;
    const int vals = wi.type == GT_Q8_0 ? 128 : 256;
    if (!Y || !W || !X || M <= 0 || K % vals || (reinterpret_cast<uintptr_t>(X) & 15) ||
        (wi.type != GT_Q4_K && wi.type != GT_Q4_0 && wi.type != GT_Q8_0)) {
        holo_set_status(HOLO_E_ARG, "batched matmul: needs a tiled Q8_0/Q4_0/Q4_K weight (cuda_upload_quant), "
                                    "K a whole number of 128/256-value units, X 16-byte aligned");
        return false;
    }
    const PfPlan pl = pf_plan(wi, M, D->sms, plan_rows);
    const int tn = pl.tn, mtiles = pl.mtiles, Mpad = pl.Mpad, splits = pl.splits, kc_per_split = pl.kc_per_split;
    const size_t xt_bytes = pl.xt_bytes, part_bytes = pl.part_bytes;
    uint8_t *tmp;
    if (scratch) {
        if (scratch_bytes < xt_bytes + part_bytes) {
            holo_set_status(HOLO_E_ARG, "batched matmul: scratch too small");
            return false;
        }
        tmp = static_cast<uint8_t *>(scratch);
    } else {
        tmp = static_cast<uint8_t *>(holo_tmp(xt_bytes + part_bytes));
    }
    if (!tmp) return false;
    uint8_t *xt = tmp;
    float *part = splits > 1 ? reinterpret_cast<float *>(tmp + xt_bytes) : Y;
    if (norm_w) {
        pf_act_norm_kernel<<<Mpad, 1024, 0, st>>>(reinterpret_cast<__half *>(xt), X, norm_w, norm_eps, M, Mpad, K);
    } else {
        const long long act_threads = (long long)Mpad * (K / 32) * 4;
        pf_act_kernel<<<(unsigned)((act_threads + 255) / 256), 256, 0, st>>>(reinterpret_cast<__half *>(xt), X, M,
                                                                           Mpad, K, tn);
    }
    if (!holo_check_launch("batched matmul activations")) return false;
    const uint8_t *w = static_cast<const uint8_t *>(W);
    bool ok;
    // weights in TMEM for token tiles up to 128 (4 activation stages); a
    // 256-token tile keeps them in shared memory: with TMEM weights and its 3
    // activation stages of 64 KB the results varied from run to run (cause
    // not found; 2 stages, or the weights in shared memory, measured
    // bit-stable over 14 repeated 70B-shape prompt passes)
    const bool at = pf_weights_in_tmem() && tn <= 128;
#define PF_SEG(T) launch_seg<T>(part, w, xt, M, Mpad, N, K, wi.units, kc_per_split, pl.g16, pl.total, pl.grid, D->status, st)
#define PF_LAUNCH_AT(T, A)                                                                                           \
    (tn == 64    ? launch_mma<T, 64, A>(part, w, xt, M, Mpad, N, K, wi.units, splits, kc_per_split, mtiles, D->status, st)  \
     : tn == 128 ? launch_mma<T, 128, A>(part, w, xt, M, Mpad, N, K, wi.units, splits, kc_per_split, mtiles, D->status, st) \
                 : launch_mma<T, 256, A>(part, w, xt, M, Mpad, N, K, wi.units, splits, kc_per_split, mtiles, D->status, st))
#define PF_LAUNCH(T) (pl.seg ? PF_SEG(T) : at ? PF_LAUNCH_AT(T, true) : PF_LAUNCH_AT(T, false))
    switch (wi.type) {
    case GT_Q4_K: ok = PF_LAUNCH(GT_Q4_K); break;
    case GT_Q4_0: ok = PF_LAUNCH(GT_Q4_0); break;
    default: ok = PF_LAUNCH(GT_Q8_0); break;
    }
#undef PF_LAUNCH
#undef PF_LAUNCH_AT
#undef PF_SEG
    if (!ok) return false;
    const long long mn = (long long)M * N;
    const unsigned rgrid = (unsigned)std::min<long long>((mn + 255) / 256, 4 * D->sms);
    if (splits > 1) {
        if (resid) pf_reduce_kernel<true><<<rgrid, 256, 0, st>>>(resid, part, mn, splits);
        else pf_reduce_kernel<false><<<rgrid, 256, 0, st>>>(Y, part, mn, splits);
        if (!holo_check_launch("batched matmul reduce")) return false;
    } else if (resid) {
        pf_add_kernel<<<rgrid, 256, 0, st>>>(resid, Y, mn);
        if (!holo_check_launch("batched matmul residual")) return false;
    }
    return true;
}

extern "C" int cuda_matmul_quant_batched(float *Y, const void *W, const float *X, int M, int N, int K) {
    if (!holo_dev()) return cuda_last_status();
    WeightInfo wi;
    if (!W || !holo_registry_find(W, &wi) || wi.rows != N || wi.cols != K) {
        holo_set_status(HOLO_E_ARG, "cuda_matmul_quant_batched: W is not a tiled weight of N x K "
                                    "(cuda_upload_quant)");
        return HOLO_E_ARG;
    }
    return holo_matmul_batched(Y, W, wi, X, M, holo_stream(), nullptr, 0) ? HOLO_OK : cuda_last_status();
}
