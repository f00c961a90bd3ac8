// prompt_attn.cu -- causal attention of a prompt pass on the 5th-gen tensor
// cores (fp16 KV cache, head_dim 128).
//
// The reference forwards a prompt one position at a time (src/ai/llm.c:1049,
// llm_cuda.c:574); per position and head it takes score = q.k / sqrtf(hd)
// over the cached positions 0..pos, a softmax, and the sum of p * v
// (llm.c:1180-1210).  A prompt pass has the rows of many positions at once,
// so the scores of 128 query rows against 128 cached positions are one
// tcgen05.mma tile (M = 128 rows, N = 128 positions, K = head_dim 128: eight
// K = 16 instructions), and so is the weighted sum of V (M = 128 rows, N = 128
// dims, K = 128 positions).
//
// CTA = one query head x 128 query rows of one sequence (8 warps: query row
// r is TMEM lane r, read by two threads, one for each half of the columns).  Operands in shared memory, all
// K-major and 128-byte swizzled (two 64-column atom blocks of 16 KB each):
//   Q  [128 rows][hd]        the rotated queries, rounded to fp16
//   K  [128 positions][hd]   a tile of the cache (fp16 as stored)
//   Vt [hd][128 positions]   the same positions' values, transposed on the way in
//                            (4-byte position pairs, bank-conflict free)
//   P  [128 rows][128 positions]  the softmax weights, fp16
// TMEM: S (128 columns, fp32 scores) and O (128 columns, fp32 output).
// Two passes over the key tiles: the first takes each row's maximum and sum
// of exp(score - max) (online, in registers); the second recomputes the
// scores (or reuses them when there is one tile), writes P = exp(s - max) /
// sum and accumulates O += P.V -- no rescaling of O, so the result does not
// depend on the tile order.  Causal: row i (position pos0 + r0 + i) sees the
// positions <= its own; rows past the pass and positions past the block's
// last row are masked.  Every wait is bounded (HOLO_E_TIMEOUT).
#include "holo_common.cuh"
#include "mv_unit.cuh"
#include "tc_util.cuh"

#include <cfloat>

namespace {

using namespace holo_tc;
using holo_mv::fence_proxy_async_smem;

constexpr int AT_ROWS = 128;      // query rows a CTA (MMA M)
constexpr int AT_KT = 128;        // cached positions a tile (MMA N of the scores, K of P.V)
constexpr int AT_HD = 128;        // head dim
constexpr int AT_THREADS = 256;   // 8 warps: warps w and w + 4 read TMEM lanes 32 (w % 4).., one column half each
constexpr int AT_TILE = AT_ROWS * AT_HD * 2;   // 32 KB: one fp16 128 x 128 operand
constexpr uint32_t AT_TMEM_COLS = 256;          // S and O

struct AtBars {
    uint64_t mma;
    uint32_t tmem;
    float2 ml[AT_THREADS];        // pass-1 (max, sum) of each half row
};

// element (r, c) of a [128][128] fp16 operand: atom block c / 64, swizzled
__device__ __forceinline__ uint32_t at_off(int r, int c) {
    return (uint32_t)((c >> 6) * (AT_ROWS * 128)) + sw128_off(r, c & 63);
}

// the 8 K = 16 MMAs of one 128 x 128 x 128 tile, A and B K-major
__device__ __forceinline__ void at_mma_tile(uint32_t tmem_d, const uint8_t *a, const uint8_t *b, bool acc) {
    constexpr uint32_t idesc = tc_idesc_f16(AT_ROWS, AT_KT);
    const uint64_t ad = sw128_desc(a), bd = sw128_desc(b);
#pragma unroll
    for (int kk = 0; kk < AT_HD / 16; ++kk) {
        const uint64_t off = (uint64_t)(((kk >> 2) * (AT_ROWS * 128) + (kk & 3) * 32) >> 4);
        tc_mma(tmem_d, ad + off, bd + off, idesc, acc || kk > 0);
    }
}

// K tile t (positions [t*128, +128)) of the cache into sk: thread item i =
// (position i / 16, 16-byte chunk i % 16), 8 items a thread, loads first
__device__ __forceinline__ void at_stage_k(uint8_t *sk, const __half *__restrict__ kc, int kv_dim, int kvh, int t,
                                           int kv_end) {
    uint4 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int i = threadIdx.x + AT_THREADS * k, p = t * AT_KT + (i >> 4);
        v[k] = make_uint4(0u, 0u, 0u, 0u);
        if (p < kv_end) v[k] = __ldg(reinterpret_cast<const uint4 *>(kc + (size_t)p * kv_dim + (size_t)kvh * AT_HD) + (i & 15));
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int i = threadIdx.x + AT_THREADS * k;
        *reinterpret_cast<uint4 *>(sk + at_off(i >> 4, 8 * (i & 15))) = v[k];
    }
}

// V tile t transposed into sv (row = dim, column = position): thread item i =
// (position pair i % 64, 16-dim chunk i / 64), 2 items a thread; a warp's
// lanes hold 32 consecutive pairs, so each 4-byte store of a dim row covers
// all 32 banks
__device__ __forceinline__ void at_stage_vt(uint8_t *sv, const __half *__restrict__ vc, int kv_dim, int kvh, int t,
                                            int kv_end) {
    uint4 v[2][4];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int i = threadIdx.x + AT_THREADS * k, pp = i & 63, ch = i >> 6;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int p = t * AT_KT + 2 * pp + (e >> 1);
            v[k][e] = make_uint4(0u, 0u, 0u, 0u);
            if (p < kv_end)
                v[k][e] = __ldg(reinterpret_cast<const uint4 *>(vc + (size_t)p * kv_dim + (size_t)kvh * AT_HD + 16 * ch) +
                                (e & 1));
        }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int i = threadIdx.x + AT_THREADS * k, pp = i & 63, ch = i >> 6;
        const __half *a = reinterpret_cast<const __half *>(&v[k][0]);   // position 2 pp, dims 16 ch ..
        const __half *b = reinterpret_cast<const __half *>(&v[k][2]);   // position 2 pp + 1
#pragma unroll
        for (int d = 0; d < 16; ++d)
            *reinterpret_cast<__half2 *>(sv + at_off(16 * ch + d, 2 * pp)) = __halves2half2(a[d], b[d]);
    }
}

__global__ void __launch_bounds__(AT_THREADS, 1)
pf_attn_tc_kernel(float *__restrict__ att, const float *__restrict__ qkv, const __half *__restrict__ kc,
                  const __half *__restrict__ vc, const int *__restrict__ pos_p, int M, int group, int kv_dim,
                  size_t qkv_bs, size_t att_bs, size_t kv_bs, float sqrt_hd, int *status) {
    extern __shared__ uint8_t at_smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(at_smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sq = base, *sk = base + AT_TILE, *sv = base + 2 * AT_TILE, *sp = base + 3 * AT_TILE;
    AtBars &B = *reinterpret_cast<AtBars *>(base + 4 * AT_TILE);
    const int h = blockIdx.x, r0 = blockIdx.y * AT_ROWS, seq = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    qkv += (size_t)seq * M * qkv_bs;
    att += (size_t)seq * M * att_bs;
    kc += (size_t)seq * kv_bs;
    vc += (size_t)seq * kv_bs;
    const int pos0 = __ldg(pos_p);
    const int nrows = min(AT_ROWS, M - r0);
    const int kvh = h / group;
    const int kv_end = pos0 + r0 + nrows;             // positions the block's rows see
    const int ntiles = (kv_end + AT_KT - 1) / AT_KT;
    const int row = 32 * (warp & 3) + lane;           // this thread's query row = TMEM lane
    const int c0 = 64 * (warp >> 2);                  // and its half of the columns
    const int my_pos = pos0 + r0 + row;
    const bool row_live = row < nrows;

    if (tid == 0) {
        mbar_init(&B.mma, 1);
        fence_barrier_init();
    }
    if (warp == 0) tc_alloc(&B.tmem, AT_TMEM_COLS);
    {
        // Q rows, rounded to fp16: item i = (row i / 32, 4 dims i % 32), 16 a thread
        float4 v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const int i = tid + AT_THREADS * k, r = i >> 5;
            v[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (r < nrows) v[k] = __ldg(reinterpret_cast<const float4 *>(qkv + (size_t)(r0 + r) * qkv_bs + (size_t)h * AT_HD) + (i & 31));
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const int i = tid + AT_THREADS * k;
            const __half2 a = __floats2half2_rn(v[k].x, v[k].y), b = __floats2half2_rn(v[k].z, v[k].w);
            uint2 w;
            w.x = *reinterpret_cast<const uint32_t *>(&a);
            w.y = *reinterpret_cast<const uint32_t *>(&b);
            *reinterpret_cast<uint2 *>(sq + at_off(i >> 5, 4 * (i & 31))) = w;
        }
    }
    fence_proxy_async_smem();   // the tensor core reads Q through the async proxy
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tS = B.tmem, tO = B.tmem + AT_KT;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    uint32_t par = 0;
    bool ok = true;

    // scores of tile t into S (staging K first when asked); false on a time-out
    auto scores = [&](int t, bool stage) -> bool {
        if (stage) {
            at_stage_k(sk, kc, kv_dim, kvh, t, kv_end);
            fence_proxy_async_smem();
        }
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            at_mma_tile(tS, sq, sk, false);
            tc_commit(&B.mma);
        }
        const bool w = mbar_wait_bounded(&B.mma, par, status, HOLO_E_TIMEOUT);
        par ^= 1u;
        tc_fence_after();
        return __syncthreads_and(w) != 0;
    };

    // ---- pass 1: each row's maximum and sum of exp(score - max), per half row ----
    // (16 columns at a time: their maximum, then 16 independent exps)
    const float scale = 1.0f / sqrt_hd;
    float m = -FLT_MAX, l = 0.0f;
    for (int t = 0; t < ntiles && ok; ++t) {
        ok = scores(t, true);
        if (!ok) break;
#pragma unroll 1
        for (int cb = c0; cb < c0 + 64; cb += 16) {
            uint32_t v[16];
            tc_ld16(tS + lane_base + (uint32_t)cb, v);
            // live columns (no early exit: the next tcgen05.ld is warp-wide)
            const int nv = row_live ? min(16, my_pos - (t * AT_KT + cb) + 1) : 0;
            if (nv > 0) {
                float sc[16], cm = -FLT_MAX;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    sc[j] = __uint_as_float(v[j]) * scale;
                    if (j < nv) cm = fmaxf(cm, sc[j]);
                }
                const float mn = fmaxf(m, cm);
                float add = 0.0f;
#pragma unroll
                for (int j = 0; j < 16; ++j) add += j < nv ? __expf(sc[j] - mn) : 0.0f;
                l = l * __expf(m - mn) + add;
                m = mn;
            }
        }
    }
    // the two halves of the row: the same combination on both threads
    B.ml[tid] = make_float2(m, l);
    __syncthreads();
    {
        const float2 a = B.ml[tid & 127], b = B.ml[(tid & 127) + 128];
        m = fmaxf(a.x, b.x);
        l = (a.y > 0.0f ? a.y * __expf(a.x - m) : 0.0f) + (b.y > 0.0f ? b.y * __expf(b.x - m) : 0.0f);
    }
    const float inv_l = l > 0.0f ? 1.0f / l : 0.0f;

    // ---- pass 2: P = exp(score - max) / sum, O += P . V ----
    for (int t = 0; t < ntiles && ok; ++t) {
        // V of the tile (and K again unless the scores of the only tile are still in TMEM)
        const bool again = ntiles > 1;
        tc_fence_before();
        __syncthreads();   // the previous tile's MMAs have read sk / sv / sp (waited below)
        at_stage_vt(sv, vc, kv_dim, kvh, t, kv_end);
        fence_proxy_async_smem();
        if (again) ok = scores(t, true);
        if (!ok) break;
#pragma unroll 1
        for (int cb = c0; cb < c0 + 64; cb += 16) {
            uint32_t v[16];
            tc_ld16(tS + lane_base + (uint32_t)cb, v);
            __align__(16) __half pv[16];
            const int nv = row_live ? min(16, my_pos - (t * AT_KT + cb) + 1) : 0;   // live columns
#pragma unroll
            for (int j = 0; j < 16; ++j)
                pv[j] = __float2half_rn(j < nv ? __expf(__uint_as_float(v[j]) * scale - m) * inv_l : 0.0f);
            *reinterpret_cast<uint4 *>(sp + at_off(row, cb)) = *reinterpret_cast<const uint4 *>(&pv[0]);
            *reinterpret_cast<uint4 *>(sp + at_off(row, cb + 8)) = *reinterpret_cast<const uint4 *>(&pv[8]);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            at_mma_tile(tO, sp, sv, t > 0);
            tc_commit(&B.mma);
        }
        const bool w = mbar_wait_bounded(&B.mma, par, status, HOLO_E_TIMEOUT);
        par ^= 1u;
        tc_fence_after();
        ok = __syncthreads_and(w) != 0;
    }

    // ---- O -> att[row][h * hd + c0 ..] ----
    // (tcgen05.ld is warp-wide and aligned: every lane loads, live rows store;
    // a wait that gave up left the status word set and the rows untouched)
    if (ok) {
        float *o = att + (size_t)(r0 + row) * att_bs + (size_t)h * AT_HD;
#pragma unroll 1
        for (int cb = c0; cb < c0 + 64; cb += 16) {
            uint32_t v[16];
            tc_ld16(tO + lane_base + (uint32_t)cb, v);
            if (row_live) {
#pragma unroll
                for (int j = 0; j < 16; j += 4)
                    *reinterpret_cast<float4 *>(o + cb + j) = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                                                          __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tc_dealloc(B.tmem, AT_TMEM_COLS);
    }
}

constexpr size_t AT_SMEM = 1024 + 4 * (size_t)AT_TILE + sizeof(AtBars);

}  // namespace

// Causal prompt attention of nseq sequences x M rows on the tensor cores (see
// above): att [row][n_heads * 128] from the rotated queries in qkv (row stride
// qkv_bs) and the fp16 caches (kv_bs elements between sequences), positions
// *pos_p + row.  False (status set) if the launch fails.
bool holo_prompt_attn_tc(float *att, const float *qkv, const __half *kc, const __half *vc, const int *pos_p, int M,
                         int nseq, int n_heads, int group, int kv_dim, size_t qkv_bs, size_t att_bs, size_t kv_bs,
                         float sqrt_hd, int *status, cudaStream_t st) {
    static bool configured[16] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 16 && !configured[dev]) {
        if (cudaFuncSetAttribute(pf_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AT_SMEM) !=
            cudaSuccess)
            return holo_check_launch("prompt attention: kernel attributes");
        configured[dev] = true;
    }
    const dim3 grid(n_heads, (M + AT_ROWS - 1) / AT_ROWS, nseq);
    pf_attn_tc_kernel<<<grid, AT_THREADS, AT_SMEM, st>>>(att, qkv, kc, vc, pos_p, M, group, kv_dim, qkv_bs, att_bs,
                                                         kv_bs, sqrt_hd, status);
    return holo_check_launch("prompt attention (tensor cores)");
}
