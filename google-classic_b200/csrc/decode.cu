// decode.cu -- batch-1 decode of a Llama-family model on one GPU.
//
// One token step restates llm_forward for one position (src/ai/llm.c:1015-1269)
// and llm_sample (llm.c:1281-1328, tensor.c:460-667) on the device:
//
//   embed   x = emb[seq[pos]]                                  (llm.c:1058, 943-1008)
//   per layer l:
//     mv    qkv = [Wq;Wk;Wv] . rmsnorm(x, attn_norm)           (llm.c:1075-1087)
//     rope  rotate-half RoPE of q and k at pos, k and v appended to the
//           layer's cache at [pos][kv_dim]                       (llm.c:1131-1170)
//     attn  softmax(q.K^T / sqrt(hd)) . V over positions 0..pos, GQA
//           (llm.c:1172-1210), split over positions then merged
//     mv    x = x + Wo . att                                     (llm.c:1214-1222)
//     mv    h = silu(W1 . xn) * (W3 . xn), xn = rmsnorm(x, ffn_norm), with W1 and
//           W3 rows interleaved by 16 so one row-block yields 16 outputs
//                                                                (llm.c:1226-1240)
//     mv    x = x + W2 . h                                       (llm.c:1243-1252)
//   mv      logits = Wout . rmsnorm(x, norm)                     (llm.c:1256-1267)
//   sample  temperature, repetition penalty, softmax, top-k, top-p, draw
//
// pos, the token sequence and the history live in device memory, so the step
// is captured once as a CUDA graph and replayed for every position; every
// kernel of the step is launched with programmatic dependent launch, so the
// next matvec's CTAs are resident early and prefetch its weights into L2.
#include "holo_common.cuh"
#include "mv_device.cuh"
#include "matvec.cuh"
#include "sampler.cuh"
#include "step.cuh"

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace {

using namespace holo_dec;

__device__ __forceinline__ void dec_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void dec_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename KV> __device__ __forceinline__ KV to_kv(float v);
template <> __device__ __forceinline__ float to_kv<float>(float v) { return v; }
template <> __device__ __forceinline__ __half to_kv<__half>(float v) { return __float2half_rn(v); }

// ---------------------------------------------------------------------------
// embedding row of the token at pos (F32 copy, F16 exact widening).  Several
// rows: row blockIdx.y = b * rps + i is position pos + i of sequence b, whose
// token list starts seq_bs ints after sequence b-1's (batched decode: rps 1;
// prompt passes: rps positions a sequence)
// ---------------------------------------------------------------------------
template <bool F16>
__global__ void dec_embed_kernel(float *__restrict__ x, const void *__restrict__ emb, const int *__restrict__ seq,
                                 const int *__restrict__ pos_p, int dim, int vocab, int seq_bs, int rps) {
    dec_pdl_trigger();
    dec_pdl_wait();
    const int r = blockIdx.y, b = r / rps;
    seq += (size_t)b * seq_bs;
    x += (size_t)r * dim;
    const int tok = seq[*pos_p + (r - b * rps)];
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= dim) return;
    if (tok < 0 || tok >= vocab) {
        x[i] = 0.0f;
        return;
    }
    if constexpr (F16) x[i] = __half2float(reinterpret_cast<const __half *>(emb)[(size_t)tok * dim + i]);
    else x[i] = reinterpret_cast<const float *>(emb)[(size_t)tok * dim + i];
}

// ---------------------------------------------------------------------------
// RoPE of q (n_heads) and k (n_kv_heads) at pos (pairs by `mode`,
// holo_model_desc.rope_mode), then k and v appended to the layer's cache;
// one CTA per head, one thread per rotation pair.  Several
// rows: row blockIdx.y = b * rps + i (qkv_bs floats apart) is position pos + i
// of sequence b, whose cache starts kv_bs elements after sequence b-1's
// ---------------------------------------------------------------------------
template <typename KV>
__global__ void dec_rope_append_kernel(float *__restrict__ qkv, KV *__restrict__ kc, KV *__restrict__ vc,
                                       const int *__restrict__ pos_p, int hd, int n_heads, int n_kv_heads,
                                       float base, size_t qkv_bs, size_t kv_bs, int rps, int mode) {
    dec_pdl_trigger();
    dec_pdl_wait();
    const int r = blockIdx.y, b = r / rps;
    qkv += r * qkv_bs;
    kc += b * kv_bs;
    vc += b * kv_bs;
    const int pos = *pos_p + (r - b * rps);
    const int h = blockIdx.x, i = threadIdx.x, half = hd / 2;
    if (i >= half) return;
    const int q_dim = n_heads * hd, kv_dim = n_kv_heads * hd;
    float c, s;
    rope_cos_sin(pos, i, hd, base, c, s);
    // the rotation pair of frequency i: (i, i + hd/2), or (2i, 2i+1)
    const int i0 = mode == HOLO_ROPE_ADJACENT ? 2 * i : i, i1 = mode == HOLO_ROPE_ADJACENT ? 2 * i + 1 : i + half;
    if (h < n_heads) {
        float *qh = qkv + (size_t)h * hd;
        rope_rotate(qh[i0], qh[i1], c, s);
    }
    if (h < n_kv_heads) {
        const float *kh = qkv + q_dim + (size_t)h * hd;
        const float *vh = qkv + q_dim + kv_dim + (size_t)h * hd;
        float a = kh[i0], b = kh[i1];
        rope_rotate(a, b, c, s);
        KV *kd = kc + (size_t)pos * kv_dim + (size_t)h * hd;
        KV *vd = vc + (size_t)pos * kv_dim + (size_t)h * hd;
        kd[i0] = to_kv<KV>(a);
        kd[i1] = to_kv<KV>(b);
        vd[i0] = to_kv<KV>(vh[i0]);
        vd[i1] = to_kv<KV>(vh[i1]);
    }
}

// ---------------------------------------------------------------------------
// decode attention, split over positions (flash-decoding).  CTA (head h, split
// s) folds positions [s*per_split, ...) of 0..pos with an online softmax.  An
// 8-lane group owns one position at a time (HD/8 dims per lane), so a warp
// works on four positions at once and each score needs 3 shuffles.
// ---------------------------------------------------------------------------
constexpr int AT_WARPS = 4;
constexpr int AT_GROUPS = AT_WARPS * 4;     // position groups per CTA

template <typename KV, int N> struct KvVec;
template <int N> struct KvVec<float, N> {
    static __device__ __forceinline__ void load(const float *p, float (&o)[N]) {
#pragma unroll
        for (int i = 0; i < N; i += 4) {
            const float4 v = *reinterpret_cast<const float4 *>(p + i);
            o[i] = v.x; o[i + 1] = v.y; o[i + 2] = v.z; o[i + 3] = v.w;
        }
    }
};
template <int N> struct KvVec<__half, N> {
    static __device__ __forceinline__ void load(const __half *p, float (&o)[N]) {
#pragma unroll
        for (int i = 0; i < N; i += 8) {
            const uint4 v = *reinterpret_cast<const uint4 *>(p + i);
            const __half2 *h2 = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __half22float2(h2[k]);
                o[i + 2 * k] = f.x;
                o[i + 2 * k + 1] = f.y;
            }
        }
    }
};

// batched: sequence blockIdx.z, q_bs floats, kv_bs cache elements and
// part_bs partial floats apart
template <typename KV, int HD>
__global__ void __launch_bounds__(AT_WARPS * 32)
dec_attn_split_kernel(float *__restrict__ part, const float *__restrict__ q, const KV *__restrict__ kc,
                      const KV *__restrict__ vc, const int *__restrict__ pos_p, int kv_dim, int group,
                      int per_split, int max_splits, float sqrt_hd, size_t q_bs, size_t kv_bs, size_t part_bs) {
    constexpr int DPL = HD / 8;
    dec_pdl_trigger();
    dec_pdl_wait();
    part += blockIdx.z * part_bs;
    q += blockIdx.z * q_bs;
    kc += blockIdx.z * kv_bs;
    vc += blockIdx.z * kv_bs;
    const int kv_len = *pos_p + 1;
    const int h = blockIdx.x, sp = blockIdx.y;
    const int p0 = sp * per_split;
    float *out = part + ((size_t)h * max_splits + sp) * (HD + 2);
    if (p0 >= kv_len) {
        if (threadIdx.x == 0) { out[0] = -FLT_MAX; out[1] = 0.0f; }
        return;
    }
    const int p1 = min(kv_len, p0 + per_split);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 3, l8 = lane & 7;
    const int kvh = h / group;
    float qf[DPL], acc[DPL];
#pragma unroll
    for (int d = 0; d < DPL; ++d) {
        qf[d] = q[(size_t)h * HD + l8 * DPL + d];
        acc[d] = 0.0f;
    }
    float m = -FLT_MAX, l = 0.0f;
    for (int base = p0 + warp * 4; base < p1; base += AT_GROUPS) {
        const int p = base + g;
        const bool live = p < p1;
        float kf[DPL];
        float dot = 0.0f;
        if (live) {
            KvVec<KV, DPL>::load(kc + (size_t)p * kv_dim + (size_t)kvh * HD + l8 * DPL, kf);
#pragma unroll
            for (int d = 0; d < DPL; ++d) dot = fmaf(qf[d], kf[d], dot);
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        dot += __shfl_xor_sync(0xffffffffu, dot, 4);
        if (live) {
            const float sc = __fdiv_rn(dot, sqrt_hd);     // score / sqrtf(hd), llm.c:1187
            const float mn = fmaxf(m, sc);
            const float corr = __expf(m - mn), e = __expf(sc - mn);
            l = fmaf(l, corr, e);
            float vf[DPL];
            KvVec<KV, DPL>::load(vc + (size_t)p * kv_dim + (size_t)kvh * HD + l8 * DPL, vf);
#pragma unroll
            for (int d = 0; d < DPL; ++d) acc[d] = fmaf(acc[d], corr, e * vf[d]);
            m = mn;
        }
    }
    // merge the CTA's position groups
    __shared__ float sm_m[AT_GROUPS], sm_l[AT_GROUPS];
    __shared__ float sm_acc[AT_GROUPS][HD];
    const int gi = warp * 4 + g;
    if (l8 == 0) { sm_m[gi] = m; sm_l[gi] = l; }
#pragma unroll
    for (int d = 0; d < DPL; ++d) sm_acc[gi][l8 * DPL + d] = acc[d];
    __syncthreads();
    float M = -FLT_MAX;
#pragma unroll
    for (int k = 0; k < AT_GROUPS; ++k)
        if (sm_l[k] > 0.0f) M = fmaxf(M, sm_m[k]);
    for (int d = threadIdx.x; d < HD; d += blockDim.x) {
        float a = 0.0f;
#pragma unroll
        for (int k = 0; k < AT_GROUPS; ++k)
            if (sm_l[k] > 0.0f) a = fmaf(sm_acc[k][d], __expf(sm_m[k] - M), a);
        out[2 + d] = a;
    }
    if (threadIdx.x == 0) {
        float L = 0.0f;
#pragma unroll
        for (int k = 0; k < AT_GROUPS; ++k)
            if (sm_l[k] > 0.0f) L = fmaf(sm_l[k], __expf(sm_m[k] - M), L);
        out[0] = M;
        out[1] = L;
    }
}

// batched: sequence blockIdx.y, att_bs and part_bs floats apart
template <int HD>
__global__ void dec_attn_merge_kernel(float *__restrict__ att, const float *__restrict__ part,
                                      const int *__restrict__ pos_p, int per_split, int max_splits,
                                      size_t att_bs, size_t part_bs) {
    dec_pdl_trigger();
    dec_pdl_wait();
    att += blockIdx.y * att_bs;
    part += blockIdx.y * part_bs;
    const int kv_len = *pos_p + 1;
    const int nsp = min(max_splits, (kv_len + per_split - 1) / per_split);
    const int h = blockIdx.x;
    const float *ph = part + (size_t)h * max_splits * (HD + 2);
    float M = -FLT_MAX;
    for (int s = 0; s < nsp; ++s)
        if (ph[(size_t)s * (HD + 2) + 1] > 0.0f) M = fmaxf(M, ph[(size_t)s * (HD + 2)]);
    float L = 0.0f;
    for (int s = 0; s < nsp; ++s) {
        const float *ps = ph + (size_t)s * (HD + 2);
        if (ps[1] > 0.0f) L = fmaf(ps[1], __expf(ps[0] - M), L);
    }
    const float inv = 1.0f / L;
    for (int d = threadIdx.x; d < HD; d += blockDim.x) {
        float a = 0.0f;
        for (int s = 0; s < nsp; ++s) {
            const float *ps = ph + (size_t)s * (HD + 2);
            if (ps[1] > 0.0f) a = fmaf(ps[2 + d], __expf(ps[0] - M), a);
        }
        att[(size_t)h * HD + d] = a * inv;
    }
}

// ---------------------------------------------------------------------------
// prompt attention: the M consecutive positions p0 .. p0+M-1 (p0 = *pos_p) of
// sequence blockIdx.z (its rows from z * M, its cache kv_bs elements after the
// previous sequence's), each attending to cache positions 0 .. its own, whose
// keys and values are already appended (llm.c:1180-1200: score = q.k / sqrtf(hd),
// softmax over the positions, sum of p * v; here with an online softmax, as
// in the decode kernels).  CTA: KV head blockIdx.x and query tokens
// [blockIdx.y * qt, +qt) x the group's query heads: up to PA_ROWS rows, two
// a warp.  Each tile of PA_KT positions is staged once in shared memory for
// all rows (keys transposed, one float of padding a row: conflict-free for
// both the staging stores and the per-lane key reads).
// ---------------------------------------------------------------------------
constexpr int PA_WARPS = 8, PA_ROWS = 2 * PA_WARPS, PA_KT = 64;

__host__ __device__ constexpr size_t pa_smem(int hd) {
    return sizeof(float) * ((size_t)hd * (PA_KT + 1) + (size_t)PA_KT * hd + (size_t)PA_ROWS * hd);
}

template <typename KV> __device__ __forceinline__ float kv_f(KV v);
template <> __device__ __forceinline__ float kv_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float kv_f<__half>(__half v) { return __half2float(v); }

template <typename KV, int HD>
__global__ void __launch_bounds__(PA_WARPS * 32)
pf_attn_kernel(float *__restrict__ att, const float *__restrict__ qkv, const KV *__restrict__ kc,
               const KV *__restrict__ vc, const int *__restrict__ pos_p, int M, int qt, int group, int kv_dim,
               size_t qkv_bs, size_t att_bs, size_t kv_bs, float sqrt_hd) {
    constexpr int DPL = HD / 32, KS = PA_KT + 1;
    qkv += (size_t)blockIdx.z * M * qkv_bs;
    att += (size_t)blockIdx.z * M * att_bs;
    kc += blockIdx.z * kv_bs;
    vc += blockIdx.z * kv_bs;
    extern __shared__ float pa_sm[];
    float *kt = pa_sm;                 // [HD][KS]: keys, transposed
    float *vs = kt + HD * KS;          // [PA_KT][HD]
    float *qs = vs + PA_KT * HD;       // [PA_ROWS][HD]
    const int kvh = blockIdx.x, t0 = blockIdx.y * qt;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int p0 = *pos_p;
    const int nt = min(qt, M - t0), rows = nt * group;
    static_assert((PA_KT * (HD / 8)) % (PA_WARPS * 32) == 0, "staging loads tile the K/V tile");
    for (int e = tid; e < rows * HD / 4; e += blockDim.x) {   // float4 loads (HD % 4 == 0)
        const int r = e / (HD / 4), dd = (e - r * (HD / 4)) * 4;
        *reinterpret_cast<float4 *>(qs + r * HD + dd) = *reinterpret_cast<const float4 *>(
            qkv + (size_t)(t0 + r / group) * qkv_bs + (size_t)(kvh * group + r % group) * HD + dd);
    }
    const int nkeys = p0 + t0 + nt;    // the CTA's last token attends to all of them
    float mx[2], sum[2], acc[2][DPL];
    int last[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int r = 2 * warp + i;
        last[i] = r < rows ? p0 + t0 + r / group : -1;   // -1: no row
        mx[i] = -FLT_MAX;
        sum[i] = 0.0f;
#pragma unroll
        for (int k = 0; k < DPL; ++k) acc[i][k] = 0.0f;
    }
    for (int j0 = 0; j0 < nkeys; j0 += PA_KT) {
        __syncthreads();   // the previous tile is consumed (and, first, the queries are stored)
        // 8 dims a thread per vector load, PA_STAGE_IT loads of K and V each
        // in flight before any store
        constexpr int PA_STAGE_IT = PA_KT * (HD / 8) / (PA_WARPS * 32);
#pragma unroll
        for (int it = 0; it < PA_STAGE_IT; ++it) {
            const int e = tid + it * PA_WARPS * 32;
            const int j = e / (HD / 8), d0 = (e - j * (HD / 8)) * 8;
            float kf[8], vf[8];
            if (j0 + j < nkeys) {
                const size_t o = (size_t)(j0 + j) * kv_dim + (size_t)kvh * HD + d0;
                KvVec<KV, 8>::load(kc + o, kf);
                KvVec<KV, 8>::load(vc + o, vf);
            } else {
#pragma unroll
                for (int t = 0; t < 8; ++t) kf[t] = vf[t] = 0.0f;
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                kt[(d0 + t) * KS + j] = kf[t];
                vs[j * HD + d0 + t] = vf[t];
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            if (last[i] < j0) continue;   // no row, or no position of this tile is visible to it (warp-uniform)
            const float *q = qs + (2 * warp + i) * HD;
            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll 16
            for (int dd = 0; dd < HD; ++dd) {
                const float qd = q[dd];
                s0 = fmaf(qd, kt[dd * KS + lane], s0);
                s1 = fmaf(qd, kt[dd * KS + lane + 32], s1);
            }
            const bool va = j0 + lane <= last[i], vb = j0 + lane + 32 <= last[i];
            s0 = __fdiv_rn(s0, sqrt_hd);
            s1 = __fdiv_rn(s1, sqrt_hd);
            float mt = fmaxf(va ? s0 : -FLT_MAX, vb ? s1 : -FLT_MAX);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
            const float mn = fmaxf(mx[i], mt);
            const float corr = __expf(mx[i] - mn);
            const float e0 = va ? __expf(s0 - mn) : 0.0f, e1 = vb ? __expf(s1 - mn) : 0.0f;
            float es = e0 + e1;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) es += __shfl_xor_sync(0xffffffffu, es, o);
            sum[i] = fmaf(sum[i], corr, es);
#pragma unroll
            for (int k = 0; k < DPL; ++k) acc[i][k] *= corr;
#pragma unroll 8
            for (int jj = 0; jj < PA_KT; ++jj) {
                const float pj = __shfl_sync(0xffffffffu, jj < 32 ? e0 : e1, jj & 31);
                const float *v = vs + jj * HD + lane * DPL;
#pragma unroll
                for (int k = 0; k < DPL; ++k) acc[i][k] = fmaf(pj, v[k], acc[i][k]);
            }
            mx[i] = mn;
        }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        if (last[i] < 0) continue;
        const int r = 2 * warp + i;
        float *o = att + (size_t)(t0 + r / group) * att_bs + (size_t)(kvh * group + r % group) * HD + lane * DPL;
        const float inv = 1.0f / sum[i];
#pragma unroll
        for (int k = 0; k < DPL; ++k) o[k] = acc[i][k] * inv;
    }
}

// ---------------------------------------------------------------------------
// sharded prompt passes: every rank computes its row shard of a projection
// for all rows, then writes its column slice [M][w] into columns [c0, c0+w)
// of every rank's gathered copy [M][ld] (the peers' through their mapped
// communication buffers, plain stores over NVLink).  The last CTA to finish
// publishes the exchange's epoch in every rank's flag slot `rank`; a rank
// reads its gathered copy after row_wait_kernel has seen every other rank's
// epoch.  A gathered copy is rewritten two exchanges later at the earliest,
// and by then every rank has sent a slice computed after reading it.
// ---------------------------------------------------------------------------
struct RowPeers {
    float *dst[STEP_MAX_RANKS];
    unsigned long long *flag[STEP_MAX_RANKS];
};

__global__ void __launch_bounds__(256) row_share_kernel(RowPeers P, int world, int rank, const float *__restrict__ src,
                                                        int M, int w, int c0, int ld, unsigned long long epoch,
                                                        unsigned *done) {
    const int w4 = w >> 2;
    const long long n4 = (long long)M * w4;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / w4), c = (int)(i - (long long)m * w4) * 4;
        const float4 v = *reinterpret_cast<const float4 *>(src + (size_t)m * w + c);
        for (int r = 0; r < world; ++r)
            *reinterpret_cast<float4 *>(P.dst[r] + (size_t)m * ld + c0 + c) = v;
    }
    __threadfence_system();   // this thread's stores, to every rank, before the CTA's arrival
    __syncthreads();
    if (threadIdx.x == 0) {
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0u;   // the next exchange's count (stream-ordered after this kernel)
            __threadfence_system();
            for (int r = 0; r < world; ++r)
                asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(P.flag[r] + rank), "l"(epoch) : "memory");
        }
    }
}

// wait (bounded) until every other rank has published `epoch`; on time-out,
// or when an earlier wait already timed out, HOLO_E_TIMEOUT and return
__global__ void row_wait_kernel(const unsigned long long *flags, int world, int rank, unsigned long long epoch,
                                int *status) {
    const int r = threadIdx.x;
    if (r >= world || r == rank) return;
    if (status && *(volatile int *)status == HOLO_E_TIMEOUT) return;
    const unsigned long long t0 = holo_globaltimer();
    for (unsigned it = 0;; ++it) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flags + r) : "memory");
        if (v >= epoch) return;
        if ((it & 63u) == 63u && holo_globaltimer() - t0 > HOLO_WAIT_LIMIT_NS) {
            if (status) atomicExch(status, HOLO_E_TIMEOUT);
            return;
        }
        __nanosleep(64);
    }
}

// advance the position by n (after a prompt pass of n rows)
__global__ void dec_pos_add_kernel(int *pos_p, int n) {
    if (threadIdx.x == 0) *pos_p += n;
}

__global__ void dec_step_end_kernel(int *pos_p) {
    dec_pdl_trigger();
    dec_pdl_wait();
    if (threadIdx.x == 0) *pos_p += 1;
}

__global__ void dec_set_token_kernel(int *seq, const int *pos_p, int token) { seq[*pos_p] = token; }
__global__ void dec_push_kernel(int *hist, int *nhist_p, int token) {
    hist[*nhist_p] = token;
    *nhist_p += 1;
}

// ---------------------------------------------------------------------------
// batched decode: RMSNorm (rms_norm, tensor.c:242-255: 1/sqrt(sum x^2 / n +
// eps), then x * scale * w) of sequence blockIdx.x, residual add, SwiGLU of
// the W1/W3 output interleaved by 16 rows
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) bt_rmsnorm_kernel(float *__restrict__ out, const float *__restrict__ x,
                                                          const float *__restrict__ w, int dim, float eps) {
    x += (size_t)blockIdx.x * dim;
    out += (size_t)blockIdx.x * dim;
    __shared__ float sv[32];
    float ss = 0.0f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = block_sum(ss, sv);
    const float scale = 1.0f / sqrtf(ss / (float)dim + eps);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) out[i] = x[i] * scale * w[i];
}

__global__ void bt_add_kernel(float *__restrict__ x, const float *__restrict__ t, long long n) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        x[i] += t[i];
}

// h[b][f] = silu(W1 x)[f] * (W3 x)[f]; row-block k of the product holds W1
// rows 16k..16k+15, then W3 rows 16k..16k+15
__global__ void bt_swiglu_kernel(float *__restrict__ h, const float *__restrict__ hh, int ffn, long long n) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long b = i / ffn;
        const int f = (int)(i - b * ffn);
        const float *row = hh + (size_t)b * 2 * ffn + (size_t)(f >> 4) * 32 + (f & 15);
        const float v = row[0], u = row[16];
        h[i] = (v / (1.0f + expf(-v))) * u;
    }
}

// one CTA a sequence (blockIdx.x = b): its logits, scratch and candidate
// buffers vocab_bs floats apart, its token list, history, draws and outputs
// seq_bs apart (batch 1: both 0)
__global__ void __launch_bounds__(SM_THREADS)
dec_sample_kernel(float *__restrict__ logits, float *__restrict__ probs, int *__restrict__ kept_idx,
                  float *__restrict__ kept_p, int *__restrict__ seq, int *__restrict__ hist, int *__restrict__ nhist_p,
                  const int *__restrict__ pos_p, const float *__restrict__ rvals, int *__restrict__ out_tokens,
                  int *__restrict__ last_token, int *__restrict__ status, const SampleArgs a, size_t vocab_bs,
                  size_t seq_bs) {
    extern __shared__ __align__(16) uint8_t sm_raw[];
    SampleSmem &S = *reinterpret_cast<SampleSmem *>(sm_raw);
    dec_pdl_trigger();
    dec_pdl_wait();
    const int b = blockIdx.x;
    logits += b * vocab_bs;
    probs += b * vocab_bs;
    kept_idx += b * vocab_bs;
    kept_p += b * vocab_bs;
    seq += b * seq_bs;
    hist += b * seq_bs;
    rvals += b * seq_bs;
    out_tokens += b * seq_bs;
    nhist_p += b;
    last_token += b;
    const int pos = *pos_p;
    if (a.gen && pos < a.n_prompt - 1) return;
    const int gi = a.gen ? pos - (a.n_prompt - 1) : 0;
    const int nhist = *nhist_p;
    const int token = sample_body(S, logits, probs, kept_idx, kept_p, hist, nhist, rvals[gi], status, a);
    if (token < 0) return;
    if (threadIdx.x == 0) {
        *last_token = token;
        if (a.gen) {
            seq[pos + 1] = token;
            hist[nhist] = token;
            *nhist_p = nhist + 1;
            out_tokens[gi] = token;
        }
    }
}

template <typename K, typename... Args>
bool launch_pdl_smem(K kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, args...) != cudaSuccess) return holo_check_launch("decode kernel launch");
    return holo_check_launch("decode kernel launch");
}

template <typename K, typename... Args>
bool launch_pdl(K kern, dim3 grid, dim3 block, cudaStream_t st, bool pdl, Args... args) {
    return launch_pdl_smem(kern, grid, block, 0, st, pdl, args...);
}

}  // namespace

// ---------------------------------------------------------------------------
// model object
// ---------------------------------------------------------------------------
struct HoloLayer {
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    // [Wq; Wk; Wv] in one tiled weight -- [Wq; Wk] when Wv has its own type
    // (then in wv) -- Wo, [W1; W3] interleaved by 16 rows, W2
    uint8_t *wqkv = nullptr, *wo = nullptr, *w13 = nullptr, *w2 = nullptr, *wv = nullptr;
    WeightInfo i_qkv, i_o, i_13, i_2, i_v;
    // GGUF types of Wv and W2 (the reference keeps them per layer,
    // llm.c:445-507); the other five matrices have desc.layer_type
    int wv_type = -1, w2_type = -1;
    bool ready = false;
};

struct HoloModel {
    holo_model_desc d{};
    int q_dim = 0, kv_dim = 0;     // this rank's query / KV rows (all of them when world == 1)
    int q_dim_g = 0;               // query rows of the model (the attention output length)
    // row shard of this rank (StepArgs): heads [h0, h0 + nh), KV heads
    // [kh0, kh0 + nkv), Wo/W2 rows [d0, d0 + dim_loc), SwiGLU outputs
    // [f0, f0 + ffn_loc), output rows [v0, v0 + vocab_loc)
    int world = 1, rank = 0;
    int nh = 0, h0 = 0, nkv = 0, kh0 = 0, dim_loc = 0, d0 = 0, ffn_loc = 0, f0 = 0, vocab_loc = 0, v0 = 0;
    // the step kernel's LL vectors (step.cuh) of x, the attention output, the
    // SwiGLU output and the logits in one allocation that the other ranks map
    // (cudaIpc*), and the local LL QKV output
    uint8_t *comm = nullptr;
    size_t comm_bytes = 0, off_x = 0, off_att = 0, off_h = 0, off_log = 0;
    // sharded prompt passes: gathered row copies [PROMPT_ROWS][...] of the
    // attention output, a projection's output over dim, the SwiGLU output,
    // and the ranks' exchange epochs
    size_t off_rflag = 0, off_ratt = 0, off_rt = 0, off_rh = 0;
    unsigned long long row_epoch = 0;
    unsigned *d_row_done = nullptr;
    StepWord *qkv_ll = nullptr;
    uint8_t *peer[STEP_MAX_RANKS] = {};
    bool peers_ready = false;
    std::vector<HoloLayer> layers;
    void *emb = nullptr;
    float *final_norm = nullptr;
    uint8_t *out = nullptr;
    WeightInfo i_out;
    bool globals_ready = false;
    void *kc = nullptr, *vc = nullptr;
    float *x = nullptr, *qkv = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr;
    float *part = nullptr, *probs = nullptr, *kept_p = nullptr, *rvals = nullptr;
    int *kept_idx = nullptr;
    int *d_pos = nullptr, *d_seq = nullptr, *d_hist = nullptr, *d_nhist = nullptr, *d_out = nullptr, *d_last = nullptr;
    int per_split = 64, max_splits = 0, step_max_splits = 0;
    int h_pos = 0, h_nhist = 0;
    cudaGraphExec_t g_forward = nullptr, g_gen = nullptr;
    SampleArgs gen_args{};
    int gen_n_prompt = -1;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};   // generate: start, prefill done, end
    float last_prefill_ms = 0.0f, last_decode_ms = 0.0f;
    // the caller's embedding table type (desc.emb_type): F32 / F16 kept as
    // given, quantized tables dequantized once into an F32 table
    int emb_src = 1;
    // persistent step kernel (step.cu): step_kernel is the create-time choice,
    // use_step also needs types it serves (uniform layers, Q8_0/Q4_0/Q4_K)
    bool step_kernel = false;
    bool use_step = false;
    bool step_ready = false;
    StepLayer *d_layers = nullptr;
    StepPrefetch *d_pf = nullptr;
    unsigned long long *d_bar = nullptr;
    int *d_att_cnt = nullptr;
    // batched decode (desc.batch > 1): `batch` sequences in lockstep, every
    // projection one tensor-core matmul with M = batch; its own KV caches,
    // position and token lists ([b][...], b-major)
    int batch = 1;
    float *bx = nullptr, *bxn = nullptr, *bqkv = nullptr, *batt = nullptr, *bt = nullptr, *bhh = nullptr,
          *bh = nullptr, *blogits = nullptr, *bpart = nullptr, *brvals = nullptr;
    float *bprobs = nullptr, *bkept_p = nullptr;   // per-sequence sampler scratch [batch][vocab]
    int *bkept_idx = nullptr;
    void *bkc = nullptr, *bvc = nullptr;
    int *bseq = nullptr, *bhist = nullptr, *bnhist = nullptr, *bout = nullptr, *blast = nullptr, *bpos = nullptr;
    int h_bpos = 0;
    void *bscratch = nullptr;   // the batched matmuls' scratch (graphs capture its address)
    size_t bscratch_bytes = 0;
    cudaGraphExec_t g_bstep[3] = {nullptr, nullptr, nullptr};   // prompt step, logits, logits + sampler
    SampleArgs b_args{};
    // prompt passes (one GPU, one sequence): up to r_cap consecutive positions
    // a pass, every projection one tensor-core matmul over the rows
    int prompt_mode = 1;   // 1: prompts through row passes where supported, 0: one position a step
    int r_cap = 0;
    bool r_attr = false;
    float *rx = nullptr, *rxn = nullptr, *rqkv = nullptr, *ratt = nullptr, *rt = nullptr, *rhh = nullptr,
          *rh = nullptr;
    void *rscratch = nullptr;
    size_t rscratch_bytes = 0;
};

// the handle one rank gives the others
struct CommHandle {
    cudaIpcMemHandle_t ipc;
    int rank, world, grid, magic;
    unsigned long long comm_bytes;
};
static_assert(sizeof(CommHandle) <= HOLO_COMM_HANDLE_BYTES, "comm handle");
constexpr int COMM_MAGIC = 0x484f4c4f;

namespace {

bool dev_alloc(void **p, size_t bytes) {
    if (cudaMalloc(p, bytes) != cudaSuccess) {
        cudaGetLastError();
        holo_set_status(HOLO_E_NOMEM, "holo_model: device allocation");
        *p = nullptr;
        return false;
    }
    return true;
}

// copy raw GGUF blocks of `rows` x `cols` (host or device memory) and repack
// them into dst
bool upload_repack(uint8_t *dst, const void *src, int type, int rows, int cols, cudaStream_t st) {
    const size_t raw = (size_t)rows * (size_t)gguf_row_bytes(type, cols);
    void *staging = nullptr;
    if (!dev_alloc(&staging, raw)) return false;
    bool ok = cudaMemcpyAsync(staging, src, raw, cudaMemcpyDefault, st) == cudaSuccess;
    ok = ok && holo_repack_to(dst, staging, type, rows, cols, holo_q4k_layout(), st);
    cudaStreamSynchronize(st);
    cudaFree(staging);
    if (!ok) holo_set_status(HOLO_E_ARG, "holo_model: weight upload");
    return ok;
}

bool upload_plain(void **dst, const void *src, size_t bytes, cudaStream_t st) {
    if (!dev_alloc(dst, bytes)) return false;
    if (cudaMemcpyAsync(*dst, src, bytes, cudaMemcpyDefault, st) != cudaSuccess) {
        holo_check_launch("holo_model: upload");
        return false;
    }
    return true;
}

void drop_graphs(HoloModel *m) {
    if (m->g_forward) cudaGraphExecDestroy(m->g_forward);
    if (m->g_gen) cudaGraphExecDestroy(m->g_gen);
    m->g_forward = m->g_gen = nullptr;
    for (auto &g : m->g_bstep) {
        if (g) cudaGraphExecDestroy(g);
        g = nullptr;
    }
}

// enqueue one token step (embed .. logits [.. sample] .. pos+1)
bool enqueue_step(HoloModel *m, cudaStream_t st, bool sample, const SampleArgs &sa) {
    const holo_model_desc &d = m->d;
    const bool pdl = true;
    const int hd = d.head_dim;
    bool ok = true;
    // the step's first kernel follows whatever precedes the graph in full
    ok = ok && (d.emb_type == 1
                    ? launch_pdl(dec_embed_kernel<true>, dim3((d.dim + 255) / 256), dim3(256), st, false, m->x,
                                 (const void *)m->emb, (const int *)m->d_seq, (const int *)m->d_pos, d.dim, d.vocab, 0, 1)
                    : launch_pdl(dec_embed_kernel<false>, dim3((d.dim + 255) / 256), dim3(256), st, false, m->x,
                                 (const void *)m->emb, (const int *)m->d_seq, (const int *)m->d_pos, d.dim, d.vocab, 0, 1));
    const size_t kv_layer = (size_t)d.max_seq * m->kv_dim;
    const size_t kv_es = d.kv_f16 ? 2 : 4;
    const float sqrt_hd = sqrtf((float)hd);
    for (int l = 0; l < d.n_layers && ok; ++l) {
        HoloLayer &L = m->layers[l];
        MvLaunch a;
        a.x = m->x; a.y = m->qkv; a.norm_w = L.attn_norm; a.eps = d.eps; a.act = d.act_mode;
        a.epi = MV_EPI_STORE; a.pdl = pdl;
        ok = ok && holo_matvec_launch(L.wqkv, L.i_qkv, a, st);
        if (L.wv) {   // Wv of its own type: v after q and k
            MvLaunch av = a;
            av.y = m->qkv + m->q_dim + m->kv_dim;
            ok = ok && holo_matvec_launch(L.wv, L.i_v, av, st);
        }
        uint8_t *kc = (uint8_t *)m->kc + (size_t)l * kv_layer * kv_es;
        uint8_t *vc = (uint8_t *)m->vc + (size_t)l * kv_layer * kv_es;
        const int heads = max(d.n_heads, d.n_kv_heads);
        if (d.kv_f16)
            ok = ok && launch_pdl(dec_rope_append_kernel<__half>, dim3(heads), dim3(hd / 2), st, pdl, m->qkv,
                                  (__half *)kc, (__half *)vc, (const int *)m->d_pos, hd, d.n_heads, d.n_kv_heads,
                                  d.rope_base, (size_t)0, (size_t)0, 1, d.rope_mode);
        else
            ok = ok && launch_pdl(dec_rope_append_kernel<float>, dim3(heads), dim3(hd / 2), st, pdl, m->qkv,
                                  (float *)kc, (float *)vc, (const int *)m->d_pos, hd, d.n_heads, d.n_kv_heads,
                                  d.rope_base, (size_t)0, (size_t)0, 1, d.rope_mode);
        const int group = d.n_heads / d.n_kv_heads;
        const dim3 ag(d.n_heads, m->max_splits);
#define HOLO_ATTN(KVT, HDV)                                                                                   \
    launch_pdl(dec_attn_split_kernel<KVT, HDV>, ag, dim3(AT_WARPS * 32), st, pdl, m->part,                    \
               (const float *)m->qkv, (const KVT *)kc, (const KVT *)vc, (const int *)m->d_pos, m->kv_dim, group, \
               m->per_split, m->max_splits, sqrt_hd, (size_t)0, (size_t)0, (size_t)0) &&                       \
        launch_pdl(dec_attn_merge_kernel<HDV>, dim3(d.n_heads), dim3(HDV), st, pdl, m->att,                   \
                   (const float *)m->part, (const int *)m->d_pos, m->per_split, m->max_splits, (size_t)0, (size_t)0)
        if (d.kv_f16) {
            if (hd == 64) ok = ok && HOLO_ATTN(__half, 64);
            else if (hd == 128) ok = ok && HOLO_ATTN(__half, 128);
            else ok = ok && HOLO_ATTN(__half, 256);
        } else {
            if (hd == 64) ok = ok && HOLO_ATTN(float, 64);
            else if (hd == 128) ok = ok && HOLO_ATTN(float, 128);
            else ok = ok && HOLO_ATTN(float, 256);
        }
#undef HOLO_ATTN
        MvLaunch o;
        o.x = m->att; o.y = m->x; o.residual = m->x; o.act = d.act_mode; o.epi = MV_EPI_ADD; o.pdl = pdl;
        ok = ok && holo_matvec_launch(L.wo, L.i_o, o, st);
        MvLaunch f;
        f.x = m->x; f.y = m->h; f.norm_w = L.ffn_norm; f.eps = d.eps; f.act = d.act_mode;
        f.epi = MV_EPI_SILU_MUL; f.pdl = pdl;
        ok = ok && holo_matvec_launch(L.w13, L.i_13, f, st);
        MvLaunch w;
        w.x = m->h; w.y = m->x; w.residual = m->x; w.act = d.act_mode; w.epi = MV_EPI_ADD; w.pdl = pdl;
        ok = ok && holo_matvec_launch(L.w2, L.i_2, w, st);
    }
    MvLaunch lo;
    lo.x = m->x; lo.y = m->logits; lo.norm_w = m->final_norm; lo.eps = d.eps; lo.act = d.act_mode;
    lo.epi = MV_EPI_STORE; lo.pdl = pdl;
    ok = ok && holo_matvec_launch(m->out, m->i_out, lo, st);
    if (sample) {
        HoloDevice *D = holo_dev();
        ok = ok && launch_pdl_smem(dec_sample_kernel, dim3(1), dim3(SM_THREADS), sizeof(SampleSmem), st, pdl,
                                   m->logits, m->probs,
                              m->kept_idx, m->kept_p, m->d_seq, m->d_hist, m->d_nhist, (const int *)m->d_pos,
                              (const float *)m->rvals, m->d_out, m->d_last, D ? D->status : nullptr, sa, (size_t)0,
                              (size_t)0);
    }
    ok = ok && launch_pdl(dec_step_end_kernel, dim3(1), dim3(32), st, pdl, m->d_pos);
    return ok;
}

// the layers over M activation rows: row b * rps + i is position pos + i of
// sequence b (token lists seq_bs ints apart, caches kv_bs elements apart).
// Batched decode: one position a sequence (rps 1), split attention; prompt
// passes: rps consecutive positions a sequence, the prompt attention kernel.
struct RowPass {
    int M = 0, rps = 1, seq_bs = 0;
    bool prompt = false;
    float *x = nullptr, *xn = nullptr, *qkv = nullptr, *att = nullptr, *t = nullptr, *hh = nullptr, *h = nullptr,
          *part = nullptr;
    void *kc = nullptr, *vc = nullptr;
    size_t kv_bs = 0;
    const int *seq = nullptr, *pos = nullptr;
    void *scratch = nullptr;
    size_t scratch_bytes = 0;
};

bool rows_norm(const RowPass &p, const float *w, int dim, float eps, cudaStream_t st) {
    bt_rmsnorm_kernel<<<p.M, 1024, 0, st>>>(p.xn, p.x, w, dim, eps);
    return holo_check_launch("rows: rmsnorm");
}

// sharded: this rank's column slice src [M][w] into columns [c0, c0+w) of
// every rank's gathered copy at comm offset `off` ([M][ld]), then the wait
// for the other ranks' slices of the same exchange
bool row_exchange(HoloModel *m, cudaStream_t st, const float *src, int M, int w, int c0, size_t off, int ld) {
    HoloDevice *D = holo_dev();
    RowPeers P{};
    for (int r = 0; r < m->world; ++r) {
        uint8_t *c = r == m->rank ? m->comm : m->peer[r];
        P.dst[r] = reinterpret_cast<float *>(c + off);
        P.flag[r] = reinterpret_cast<unsigned long long *>(c + m->off_rflag);
    }
    const unsigned long long e = ++m->row_epoch;
    const long long n4 = (long long)M * (w / 4);
    const int grid = (int)std::max<long long>(1, std::min<long long>((n4 + 255) / 256, 2LL * (D ? D->sms : 148)));
    row_share_kernel<<<grid, 256, 0, st>>>(P, m->world, m->rank, src, M, w, c0, ld, e, m->d_row_done);
    row_wait_kernel<<<1, 32, 0, st>>>(P.flag[m->rank], m->world, m->rank, e, D ? D->status : nullptr);
    return holo_check_launch("rows: exchange");
}

// prompt attention on the tensor cores (fp16 cache, head_dim 128) unless
// HOLO_PROMPT_ATTN=simt selects the SIMT kernel (pf_attn_kernel)
bool prompt_attn_tc() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("HOLO_PROMPT_ATTN");
        v = (e && strcmp(e, "simt") == 0) ? 0 : 1;
    }
    return v == 1;
}

bool enqueue_rows(HoloModel *m, cudaStream_t st, const RowPass &p) {
    const holo_model_desc &d = m->d;
    const int M = p.M, hd = d.head_dim;
    const int qkv_dim = m->q_dim + 2 * m->kv_dim;
    const size_t kv_layer = (size_t)d.max_seq * m->kv_dim;
    const size_t part_bs = (size_t)m->nh * m->max_splits * (hd + 2);
    const float sqrt_hd = sqrtf((float)hd);
    const int group = d.n_heads / d.n_kv_heads;
    // sharded (prompt passes only): the gathered copies every projection reads
    const bool shard = m->world > 1;
    const float *att_in = shard ? reinterpret_cast<const float *>(m->comm + m->off_ratt) : p.att;
    const float *t_in = shard ? reinterpret_cast<const float *>(m->comm + m->off_rt) : p.t;
    const float *h_in = shard ? reinterpret_cast<const float *>(m->comm + m->off_rh) : p.h;
    bool ok = d.emb_type == 1
                  ? launch_pdl(dec_embed_kernel<true>, dim3((d.dim + 255) / 256, M), dim3(256), st, false, p.x,
                               (const void *)m->emb, p.seq, p.pos, d.dim, d.vocab, p.seq_bs, p.rps)
                  : launch_pdl(dec_embed_kernel<false>, dim3((d.dim + 255) / 256, M), dim3(256), st, false, p.x,
                               (const void *)m->emb, p.seq, p.pos, d.dim, d.vocab, p.seq_bs, p.rps);
    auto add = [&](const float *t) {
        const long long n = (long long)M * d.dim;
        bt_add_kernel<<<(unsigned)std::min<long long>((n + 255) / 256, 1024), 256, 0, st>>>(p.x, t, n);
        return holo_check_launch("rows: residual");
    };
    const int qt = std::max(1, PA_ROWS / group);
    // every projection's K split is planned for the whole matrix (not this
    // rank's rows), so a row shard sums each row exactly as one GPU does
    const int rows_qkv = (d.n_heads + 2 * d.n_kv_heads) * hd;
    // RMSNorm + projection: on the tensor-core path the norm is fused into the
    // activation quantize/tile kernel (same arithmetic), else its own kernel
    auto normed = [&](float *Y, const void *W, const WeightInfo &wi, const float *nw, int plan_rows) {
        if (M > MVB_MAX_M)
            return holo_matmul_batched(Y, W, wi, p.x, M, st, p.scratch, p.scratch_bytes, plan_rows, nw, d.eps);
        return rows_norm(p, nw, d.dim, d.eps, st) &&
               holo_matmul_batched(Y, W, wi, p.xn, M, st, p.scratch, p.scratch_bytes, plan_rows);
    };
    // projection + residual (Wo, W2): one GPU on the tensor-core path adds
    // into x inside the matmul's K-split reduction (same arithmetic); a
    // sharded pass exchanges the rank's slice first, then adds
    auto projected = [&](float *t, const void *W, const WeightInfo &wi, const float *in) {
        if (!shard && M > MVB_MAX_M)
            return holo_matmul_batched(t, W, wi, in, M, st, p.scratch, p.scratch_bytes, d.dim, nullptr, 0.0f, p.x);
        bool r = holo_matmul_batched(t, W, wi, in, M, st, p.scratch, p.scratch_bytes, d.dim);
        if (shard) r = r && row_exchange(m, st, t, M, m->dim_loc, m->d0, m->off_rt, d.dim);
        return r && add(t_in);
    };
    for (int l = 0; l < d.n_layers && ok; ++l) {
        HoloLayer &L = m->layers[l];
        ok = normed(p.qkv, L.wqkv, L.i_qkv, L.attn_norm, rows_qkv);
        const size_t es = d.kv_f16 ? 2 : 4;
        uint8_t *kc = (uint8_t *)p.kc + (size_t)l * kv_layer * es, *vc = (uint8_t *)p.vc + (size_t)l * kv_layer * es;
        const dim3 rg(std::max(m->nh, m->nkv), M), ag(m->nh, m->max_splits, M), mg(m->nh, M);
        const dim3 pg(m->nkv, (p.rps + qt - 1) / qt, M / p.rps);
#define BT_ATTN(KVT, HDV)                                                                                          \
    launch_pdl(dec_rope_append_kernel<KVT>, rg, dim3(hd / 2), st, false, p.qkv, (KVT *)kc, (KVT *)vc, p.pos, hd,     \
               m->nh, m->nkv, d.rope_base, (size_t)qkv_dim, p.kv_bs, p.rps, d.rope_mode) &&                         \
        (p.prompt ? launch_pdl_smem(pf_attn_kernel<KVT, HDV>, pg, dim3(PA_WARPS * 32), pa_smem(HDV), st, false,      \
                                    p.att, (const float *)p.qkv, (const KVT *)kc, (const KVT *)vc, p.pos, p.rps, qt, \
                                    group, m->kv_dim, (size_t)qkv_dim, (size_t)m->q_dim, p.kv_bs, sqrt_hd)          \
                   : launch_pdl(dec_attn_split_kernel<KVT, HDV>, ag, dim3(AT_WARPS * 32), st, false, p.part,        \
                                (const float *)p.qkv, (const KVT *)kc, (const KVT *)vc, p.pos, m->kv_dim, group,    \
                                m->per_split, m->max_splits, sqrt_hd, (size_t)qkv_dim, p.kv_bs, part_bs) &&         \
                         launch_pdl(dec_attn_merge_kernel<HDV>, mg, dim3(HDV), st, false, p.att,                    \
                                    (const float *)p.part, p.pos, m->per_split, m->max_splits, (size_t)m->q_dim,    \
                                    part_bs))
        if (p.prompt && d.kv_f16 && hd == 128 && prompt_attn_tc()) {
            // RoPE + append, then the causal attention on the tensor cores
            HoloDevice *D = holo_dev();
            ok = ok && launch_pdl(dec_rope_append_kernel<__half>, rg, dim3(hd / 2), st, false, p.qkv, (__half *)kc,
                                  (__half *)vc, p.pos, hd, m->nh, m->nkv, d.rope_base, (size_t)qkv_dim, p.kv_bs, p.rps,
                                  d.rope_mode) &&
                 holo_prompt_attn_tc(p.att, p.qkv, (const __half *)kc, (const __half *)vc, p.pos, p.rps, M / p.rps,
                                     m->nh, group, m->kv_dim, (size_t)qkv_dim, (size_t)m->q_dim, p.kv_bs, sqrt_hd,
                                     D ? D->status : nullptr, st);
        } else if (d.kv_f16) {
            if (hd == 64) ok = ok && BT_ATTN(__half, 64);
            else if (hd == 128) ok = ok && BT_ATTN(__half, 128);
            else ok = ok && BT_ATTN(__half, 256);
        } else {
            if (hd == 64) ok = ok && BT_ATTN(float, 64);
            else if (hd == 128) ok = ok && BT_ATTN(float, 128);
            else ok = ok && BT_ATTN(float, 256);
        }
#undef BT_ATTN
        if (shard) ok = ok && row_exchange(m, st, p.att, M, m->q_dim, m->h0 * hd, m->off_ratt, m->q_dim_g);
        ok = ok && projected(p.t, L.wo, L.i_o, att_in);
        ok = ok && normed(p.hh, L.w13, L.i_13, L.ffn_norm, 2 * d.ffn_dim);
        if (ok) {
            const long long n = (long long)M * m->ffn_loc;
            bt_swiglu_kernel<<<(unsigned)std::min<long long>((n + 255) / 256, 2048), 256, 0, st>>>(p.h, p.hh,
                                                                                               m->ffn_loc, n);
            ok = holo_check_launch("rows: swiglu");
        }
        if (shard) ok = ok && row_exchange(m, st, p.h, M, m->ffn_loc, m->f0, m->off_rh, d.ffn_dim);
        ok = ok && projected(p.t, L.w2, L.i_2, h_in);
    }
    return ok;
}

// One position of all `batch` sequences (llm_forward per sequence, llm.c
// 1015-1269): mode 0 the prompt step (no logits), 1 with the logits, 2 with
// the logits and the sampler of every sequence (llm_sample, llm.c:1281-1328).
bool enqueue_batch_step(HoloModel *m, cudaStream_t st, int mode, const SampleArgs &sa) {
    const holo_model_desc &d = m->d;
    const int B = m->batch, S = d.max_seq + 1;
    RowPass p;
    p.M = B;
    p.x = m->bx; p.xn = m->bxn; p.qkv = m->bqkv; p.att = m->batt; p.t = m->bt; p.hh = m->bhh; p.h = m->bh;
    p.part = m->bpart;
    p.kc = m->bkc; p.vc = m->bvc;
    p.kv_bs = (size_t)d.n_layers * d.max_seq * m->kv_dim;
    p.seq = m->bseq; p.seq_bs = S; p.pos = m->bpos;
    p.scratch = m->bscratch; p.scratch_bytes = m->bscratch_bytes;
    bool ok = enqueue_rows(m, st, p);
    auto norm = [&](const float *w) { return rows_norm(p, w, d.dim, d.eps, st); };
    if (mode >= 1)
        ok = ok && norm(m->final_norm) && holo_matmul_batched(m->blogits, m->out, m->i_out, m->bxn, B, st, m->bscratch, m->bscratch_bytes);
    if (mode == 2) {   // the samplers of all sequences side by side, one CTA each
        HoloDevice *D = holo_dev();
        ok = ok && launch_pdl_smem(dec_sample_kernel, dim3(B), dim3(SM_THREADS), sizeof(SampleSmem), st, false,
                                   m->blogits, m->bprobs, m->bkept_idx, m->bkept_p, m->bseq, m->bhist, m->bnhist,
                                   (const int *)m->bpos, (const float *)m->brvals, m->bout, m->blast,
                                   D ? D->status : nullptr, sa, (size_t)d.vocab, (size_t)S);
    }
    return ok && launch_pdl(dec_step_end_kernel, dim3(1), dim3(32), st, false, m->bpos);
}

// the batched step of `mode` as a graph (first: one run outside capture, so
// the kernels' one-time set-up and the scratch sizes are settled)
bool run_batch_step(HoloModel *m, int mode, const SampleArgs &sa, cudaStream_t st);

// the sampler's shared memory exceeds the default 48 KB
bool prepare_sampler() {
    if (cudaFuncSetAttribute(dec_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(SampleSmem)) != cudaSuccess)
        return holo_check_launch("sampler attributes");
    return true;
}

bool run_batch_step(HoloModel *m, int mode, const SampleArgs &sa, cudaStream_t st) {
    if (m->g_bstep[mode] && mode == 2 && memcmp(&sa, &m->b_args, sizeof(sa)) != 0) {
        cudaGraphExecDestroy(m->g_bstep[2]);
        m->g_bstep[2] = nullptr;
    }
    if (!m->bscratch) {
        size_t need = holo_matmul_batched_scratch(m->i_out, m->batch);
        for (auto &L : m->layers)
            for (const WeightInfo *wi : {&L.i_qkv, &L.i_o, &L.i_13, &L.i_2})
                need = std::max(need, holo_matmul_batched_scratch(*wi, m->batch));
        if (!dev_alloc(&m->bscratch, need)) return false;
        m->bscratch_bytes = need;
    }
    if (!m->g_bstep[mode]) {
        // one plain step first (the kernels' one-time set-up), then the capture
        if (!prepare_sampler() || !enqueue_batch_step(m, st, mode, sa)) return false;
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
            return holo_check_launch("batched step: begin capture");
        const bool ok = enqueue_batch_step(m, st, mode, sa);
        const cudaError_t e = cudaStreamEndCapture(st, &g);
        if (!ok || e != cudaSuccess || !g) {
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
            holo_set_status(HOLO_E_ARG, "batched step: capture failed");
            return false;
        }
        const bool inst = cudaGraphInstantiate(&m->g_bstep[mode], g, 0) == cudaSuccess;
        cudaGraphDestroy(g);
        if (!inst) {
            cudaGetLastError();
            m->g_bstep[mode] = nullptr;
            holo_set_status(HOLO_E_ARG, "batched step: graph instantiation failed");
            return false;
        }
        if (mode == 2) m->b_args = sa;
        return true;   // the plain run above was this step
    }
    if (cudaGraphLaunch(m->g_bstep[mode], st) != cudaSuccess) return holo_check_launch("batched step launch");
    return true;
}

// ---------------------------------------------------------------------------
// prompt passes: the positions of a prompt before its last token need no
// logits, and each layer's projections over all of them (of every sequence of
// a batched model) are one tensor-core matmul instead of one matvec, or one
// M = batch matmul, per position.  One GPU; batch 1 with Q8 activations (the
// matmul quantizes its input rows as the matvecs do); otherwise prompts go one
// position a step.
// ---------------------------------------------------------------------------
constexpr int PROMPT_ROWS = 1024;   // rows a pass (longer prompts: several passes)

bool prompt_supported(const HoloModel *m) {
    const holo_model_desc &d = m->d;
    if (m->prompt_mode != 1 || (m->batch == 1 && d.act_mode != HOLO_ACT_Q8)) return false;
    // sharded: connected peers, and every exchanged slice in whole float4s
    if (m->world > 1 && (!m->peers_ready || m->q_dim % 4 || (m->h0 * d.head_dim) % 4 || m->dim_loc % 4 ||
                         m->d0 % 4 || m->ffn_loc % 4 || m->f0 % 4))
        return false;
    if (d.n_heads / d.n_kv_heads > PA_ROWS || (d.head_dim != 64 && d.head_dim != 128 && d.head_dim != 256))
        return false;
    for (const HoloLayer &L : m->layers) {
        if (L.wv) return false;   // the row passes read [Wq; Wk; Wv] as one weight
        for (const WeightInfo *wi : {&L.i_qkv, &L.i_o, &L.i_13, &L.i_2})
            if (wi->type != GT_Q4_K && wi->type != GT_Q4_0 && wi->type != GT_Q8_0)
                return false;
    }
    return true;
}

// buffers for passes of up to `rows` positions (grown on demand)
bool prompt_buffers(HoloModel *m, int rows) {
    const holo_model_desc &d = m->d;
    size_t need = 0;
    const int plan[4] = {(d.n_heads + 2 * d.n_kv_heads) * d.head_dim, d.dim, 2 * d.ffn_dim, d.dim};
    for (const HoloLayer &L : m->layers) {
        const WeightInfo *wis[4] = {&L.i_qkv, &L.i_o, &L.i_13, &L.i_2};
        for (int k = 0; k < 4; ++k) need = std::max(need, holo_matmul_batched_scratch(*wis[k], rows, plan[k]));
    }
    if (need > m->rscratch_bytes) {
        cudaFree(m->rscratch);
        m->rscratch = nullptr;
        m->rscratch_bytes = 0;
        if (!dev_alloc(&m->rscratch, need)) return false;
        m->rscratch_bytes = need;
    }
    if (rows <= m->r_cap) return true;
    for (float *p : {m->rx, m->rxn, m->rqkv, m->ratt, m->rt, m->rhh, m->rh}) cudaFree(p);
    m->r_cap = 0;
    const size_t R = rows;
    bool ok = dev_alloc((void **)&m->rx, sizeof(float) * R * d.dim) &&
              dev_alloc((void **)&m->rxn, sizeof(float) * R * d.dim) &&
              dev_alloc((void **)&m->rqkv, sizeof(float) * R * (m->q_dim + 2 * m->kv_dim)) &&
              dev_alloc((void **)&m->ratt, sizeof(float) * R * m->q_dim) &&
              dev_alloc((void **)&m->rt, sizeof(float) * R * d.dim) &&
              dev_alloc((void **)&m->rhh, sizeof(float) * R * 2 * d.ffn_dim) &&
              dev_alloc((void **)&m->rh, sizeof(float) * R * d.ffn_dim);
    if (!ok) return false;
    m->r_cap = rows;
    if (!m->r_attr) {   // the prompt attention's shared memory exceeds the default 48 KB (per device)
        bool a = true;
        a = a && cudaFuncSetAttribute(pf_attn_kernel<__half, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)pa_smem(128)) == cudaSuccess;
        a = a && cudaFuncSetAttribute(pf_attn_kernel<float, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)pa_smem(128)) == cudaSuccess;
        a = a && cudaFuncSetAttribute(pf_attn_kernel<__half, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)pa_smem(256)) == cudaSuccess;
        a = a && cudaFuncSetAttribute(pf_attn_kernel<float, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)pa_smem(256)) == cudaSuccess;
        a = a && cudaFuncSetAttribute(pf_attn_kernel<__half, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)pa_smem(64)) == cudaSuccess;
        a = a && cudaFuncSetAttribute(pf_attn_kernel<float, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)pa_smem(64)) == cudaSuccess;
        if (!a) return holo_check_launch("prompt attention attributes");
        m->r_attr = true;
    }
    return true;
}

// the n positions from the current one (tokens already in the token lists)
// of every sequence through the layers, their keys and values appended; the
// position advances by n.  The last pass's rows stay in rx (batch 1: the last
// position's row is last_rows - 1).
bool prompt_rows(HoloModel *m, cudaStream_t st, int n, int *last_rows) {
    const holo_model_desc &d = m->d;
    const int B = m->batch;
    const int cap = std::max(1, std::min(n, PROMPT_ROWS / B));   // positions a pass
    if (!prompt_buffers(m, B * cap)) return false;
    int *pos = B == 1 ? m->d_pos : m->bpos;
    for (int done = 0; done < n;) {
        const int c = std::min(cap, n - done);
        RowPass p;
        p.M = B * c;
        p.rps = c;
        p.prompt = true;
        p.x = m->rx; p.xn = m->rxn; p.qkv = m->rqkv; p.att = m->ratt; p.t = m->rt; p.hh = m->rhh; p.h = m->rh;
        if (B == 1) {
            p.kc = m->kc; p.vc = m->vc;
            p.seq = m->d_seq;
        } else {
            p.kc = m->bkc; p.vc = m->bvc;
            p.kv_bs = (size_t)d.n_layers * d.max_seq * m->kv_dim;
            p.seq = m->bseq; p.seq_bs = d.max_seq + 1;
        }
        p.pos = pos;
        p.scratch = m->rscratch; p.scratch_bytes = m->rscratch_bytes;
        if (!enqueue_rows(m, st, p)) return false;
        dec_pos_add_kernel<<<1, 32, 0, st>>>(pos, c);
        if (!holo_check_launch("prompt: position")) return false;
        done += c;
        if (last_rows) *last_rows = c;
    }
    return true;
}

// one-time per-kernel set-up of every matvec variant of the step, which must
// not happen inside a stream capture
bool prepare_step(HoloModel *m) {
    const holo_model_desc &d = m->d;
    HoloLayer &L = m->layers[0];
    MvLaunch a;
    a.norm_w = L.attn_norm; a.act = d.act_mode; a.epi = MV_EPI_STORE;
    MvLaunch o;
    o.residual = m->x; o.act = d.act_mode; o.epi = MV_EPI_ADD;
    MvLaunch f;
    f.norm_w = L.ffn_norm; f.act = d.act_mode; f.epi = MV_EPI_SILU_MUL;
    return prepare_sampler() && holo_matvec_prepare(L.i_qkv, a) && holo_matvec_prepare(L.i_o, o) &&
           holo_matvec_prepare(L.i_13, f) && holo_matvec_prepare(L.i_2, o) && holo_matvec_prepare(m->i_out, a);
}

cudaGraphExec_t capture_step(HoloModel *m, bool sample, const SampleArgs &sa) {
    cudaStream_t st = holo_stream();
    cudaGraph_t g = nullptr;
    if (!prepare_step(m)) return nullptr;
    if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        holo_check_launch("holo_model: begin capture");
        return nullptr;
    }
    const bool ok = enqueue_step(m, st, sample, sa);
    const cudaError_t e = cudaStreamEndCapture(st, &g);
    if (!ok || e != cudaSuccess || !g) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        holo_set_status(HOLO_E_ARG, "holo_model: step capture failed");
        return nullptr;
    }
    cudaGraphExec_t ex = nullptr;
    if (cudaGraphInstantiate(&ex, g, 0) != cudaSuccess) {
        cudaGetLastError();
        ex = nullptr;
        holo_set_status(HOLO_E_ARG, "holo_model: graph instantiation failed");
    }
    cudaGraphDestroy(g);
    return ex;
}

// the types the persistent step kernel is built for (step.cu holo_step_launch)
bool step_type(int t) { return t == GT_Q8_0 || t == GT_Q4_0 || t == GT_Q4_K; }

// the step kernel runs when chosen at create and every matrix type is one it
// serves, uniform across the layers; otherwise the one-launch-per-op graph
void refresh_use_step(HoloModel *m) {
    bool ok = m->step_kernel && step_type(m->d.layer_type) && step_type(m->d.out_type);
    for (const HoloLayer &L : m->layers) ok = ok && L.wv_type == m->d.layer_type && L.w2_type == m->d.layer_type;
    if (ok != m->use_step) {
        m->use_step = ok;
        m->step_ready = false;
    }
}

// token embedding tables the engine takes: F32, F16, or GGUF blocks of Q8_0,
// Q4_0, Q4_K, Q6_K (get_embedding, src/ai/llm.c:941-1008)
bool emb_type_ok(int t, int dim) {
    if (t == GT_F32 || t == GT_F16) return true;
    return (t == GT_Q8_0 || t == GT_Q4_0 || t == GT_Q4_K || t == GT_Q6_K) && holo_quant_shape_ok(t, 1, dim);
}

bool model_ready(HoloModel *m) {
    if (!m) return false;
    for (auto &L : m->layers)
        if (!L.ready) {
            holo_set_status(HOLO_E_ARG, "holo_model: a layer has no weights");
            return false;
        }
    if (!m->globals_ready) {
        holo_set_status(HOLO_E_ARG, "holo_model: embeddings / output not set");
        return false;
    }
    return true;
}

// L2 prefetch table of the step kernel: the matvec weights in execution order
// form one circular byte sequence; at each phase every CTA requests its share
// of the bytes up to STEP_PF_WINDOW past the end of the phase's matvec.  The
// table is the steady state (second of two simulated steps), so the output
// phase of one token already requests the first matrices of the next.
constexpr unsigned long long STEP_PF_WINDOW_DEFAULT = 32ull << 20;

bool build_step(HoloModel *m) {
    const holo_model_desc &d = m->d;
    // window: HOLO_PF_MB (MB ahead of the current matrix), default 32
    unsigned long long STEP_PF_WINDOW = STEP_PF_WINDOW_DEFAULT;
    if (const char *e = getenv("HOLO_PF_MB")) STEP_PF_WINDOW = (unsigned long long)atoi(e) << 20;
    const int L = d.n_layers, P = step_phases(L);
    std::vector<StepLayer> layers(L);
    struct Seg { const uint8_t *p; unsigned long long n; int phase; };
    std::vector<Seg> seg;
    for (int l = 0; l < L; ++l) {
        const HoloLayer &H = m->layers[l];
        layers[l] = StepLayer{H.wqkv, H.wo, H.w13, H.w2, H.attn_norm, H.ffn_norm};
        seg.push_back({H.wqkv, H.i_qkv.bytes, 1 + 5 * l});
        seg.push_back({H.wo, H.i_o.bytes, 3 + 5 * l});
        seg.push_back({H.w13, H.i_13.bytes, 4 + 5 * l});
        seg.push_back({H.w2, H.i_2.bytes, 5 + 5 * l});
    }
    seg.push_back({m->out, m->i_out.bytes, P - 1});
    std::vector<unsigned long long> start(seg.size() + 1, 0);
    for (size_t i = 0; i < seg.size(); ++i) start[i + 1] = start[i] + seg[i].n;
    const unsigned long long T = start.back();
    // end offset (within a step) of the matvec of each phase; attention and
    // embedding phases keep the previous one
    std::vector<unsigned long long> end(P, 0);
    {
        unsigned long long cur = 0;
        size_t si = 0;
        for (int ph = 0; ph < P; ++ph) {
            if (si < seg.size() && seg[si].phase == ph) { cur = start[si + 1]; ++si; }
            end[ph] = cur;
        }
    }
    std::vector<StepPrefetch> pf((size_t)P * STEP_PF_MAX, StepPrefetch{nullptr, 0});
    unsigned long long done = 0;   // bytes requested so far (absolute, over steps)
    for (int step = 0; step < 2; ++step)
        for (int ph = 0; ph < P; ++ph) {
            const unsigned long long target = (unsigned long long)step * T + end[ph] + STEP_PF_WINDOW;
            unsigned long long lo = std::max(done, target > T ? target - T : 0ull), hi = target;
            if (hi <= lo) continue;
            done = hi;
            if (step == 0) continue;
            int k = 0;
            while (lo < hi && k < STEP_PF_MAX) {
                const unsigned long long off = lo % T;
                size_t si = 0;
                while (start[si + 1] <= off) ++si;
                const unsigned long long n = std::min(hi - lo, start[si + 1] - off);
                pf[(size_t)ph * STEP_PF_MAX + k++] = StepPrefetch{seg[si].p + (off - start[si]), n};
                lo += n;
            }
        }
    bool ok = dev_alloc((void **)&m->d_layers, sizeof(StepLayer) * L) &&
              dev_alloc((void **)&m->d_pf, sizeof(StepPrefetch) * pf.size());
    if (!ok) return false;
    cudaMemcpy(m->d_layers, layers.data(), sizeof(StepLayer) * L, cudaMemcpyHostToDevice);
    cudaMemcpy(m->d_pf, pf.data(), sizeof(StepPrefetch) * pf.size(), cudaMemcpyHostToDevice);
    m->step_ready = holo_check_launch("decode step: tables");
    return m->step_ready;
}

StepArgs step_args(HoloModel *m, bool sample, const SampleArgs &sa) {
    const holo_model_desc &d = m->d;
    StepArgs a{};
    a.n_layers = d.n_layers; a.dim = d.dim; a.n_heads = m->nh; a.n_kv_heads = m->nkv; a.h0 = m->h0;
    a.n_heads_g = d.n_heads;
    a.dim_loc = m->dim_loc; a.d0 = m->d0; a.ffn_loc = m->ffn_loc; a.f0 = m->f0;
    a.vocab_loc = m->vocab_loc; a.v0 = m->v0;
    a.hd = d.head_dim; a.ffn = d.ffn_dim; a.vocab = d.vocab; a.max_seq = d.max_seq;
    a.eps = d.eps; a.rope_base = d.rope_base; a.out_type = d.out_type; a.emb_f16 = d.emb_type == 1;
    a.rope_mode = d.rope_mode;
    a.layers = m->d_layers; a.emb = m->emb; a.final_norm = m->final_norm; a.out_w = m->out;
    a.qkv = m->qkv_ll; a.logits = m->logits;
    a.kc = m->kc; a.vc = m->vc; a.att_part = m->part; a.att_cnt = m->d_att_cnt;
    a.per_split = 16; a.max_splits = m->step_max_splits;
    a.pos = m->d_pos; a.seq = m->d_seq; a.hist = m->d_hist; a.nhist = m->d_nhist; a.out_tokens = m->d_out;
    a.last = m->d_last; a.rvals = m->rvals; a.probs = m->probs; a.kept_p = m->kept_p; a.kept_idx = m->kept_idx;
    a.sa = sa; a.sample = sample; a.prefetch = m->d_pf; a.bar = m->d_bar;
    HoloDevice *D = holo_dev();
    a.status = D ? D->status : nullptr;
    a.grid = D ? D->sms : 1;
    a.world = m->world;
    a.rank = m->rank;
    for (int r = 0; r < m->world; ++r) {
        uint8_t *c = r == m->rank ? m->comm : m->peer[r];
        a.px[r] = reinterpret_cast<StepWord *>(c + m->off_x);
        a.patt[r] = reinterpret_cast<StepWord *>(c + m->off_att);
        a.ph[r] = reinterpret_cast<StepWord *>(c + m->off_h);
        a.plog[r] = reinterpret_cast<StepWord *>(c + m->off_log);
    }
    return a;
}

bool run_step(HoloModel *m, bool sample, const SampleArgs &sa, cudaStream_t st) {
    if (m->world > 1 && !m->peers_ready) {
        holo_set_status(HOLO_E_ARG, "holo_model: sharded model without peers (holo_model_open_peers)");
        return false;
    }
    if (!m->step_ready && !build_step(m)) return false;
    return holo_step_launch(step_args(m, sample, sa), m->d.layer_type, m->d.act_mode, m->d.kv_f16, st);
}

// the row shard of d.rank (host only): ranges = first and count of query
// heads, KV heads, Wo/W2 rows, SwiGLU outputs (16-row bands), output rows
bool shard_of(const holo_model_desc &d, int ranges[10]) {
    const int world = d.world <= 1 ? 1 : d.world, r = d.rank;
    if (world > STEP_MAX_RANKS || r < 0 || r >= world || d.n_heads <= 0 || d.n_kv_heads <= 0 ||
        d.n_heads % world || d.n_kv_heads % world || d.dim < 32 * world || d.ffn_dim % 16 ||
        d.ffn_dim < 16 * world || d.vocab < world)
        return false;
    auto split = [&](int n, int unit, int *o) {
        const long long b = n / unit;
        const int lo = (int)(b * r / world), hi = (int)(b * (r + 1) / world);
        o[0] = unit * lo;
        o[1] = unit * (hi - lo);
    };
    split(d.n_heads, 1, ranges);
    split(d.n_kv_heads, 1, ranges + 2);
    split(d.dim, 1, ranges + 4);
    split(d.ffn_dim, 16, ranges + 6);
    split(d.vocab, 1, ranges + 8);
    return true;
}

SampleArgs make_args(const HoloModel *m, const holo_sampler_desc *s) {
    SampleArgs a{};
    a.vocab = m->d.vocab;
    a.greedy = s->temperature == 0.0f;
    a.use_temp = s->temperature > 0.0f && s->temperature != 1.0f;
    a.tscale = a.use_temp ? 1.0f / s->temperature : 1.0f;
    a.penalty = s->repeat_penalty;
    a.last_n = s->repeat_last_n;
    a.top_k = s->top_k;
    a.top_p = s->top_p;
    return a;
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

void *holo_model_create(const holo_model_desc *desc) {
    if (!desc) return nullptr;
    const holo_model_desc &d = *desc;
    const int hd = d.head_dim;
    const int world = d.world <= 1 ? 1 : d.world;
    int sh[10];
    if (!shard_of(d, sh) || (world > 1 && hd != 128)) {
        holo_set_status(HOLO_E_ARG, "holo_model_create: unsupported sharding");
        return nullptr;
    }
    if (d.rope_mode != HOLO_ROPE_HALF && d.rope_mode != HOLO_ROPE_ADJACENT) {
        holo_set_status(HOLO_E_ARG, "holo_model_create: rope_mode must be HOLO_ROPE_HALF or HOLO_ROPE_ADJACENT");
        return nullptr;
    }
    if (d.batch > 1 && (world > 1 || d.batch > 64)) {
        holo_set_status(HOLO_E_ARG, "holo_model_create: batch 2..64 on one GPU (no sharding)");
        return nullptr;
    }
    if (d.n_layers <= 0 || d.dim <= 0 || d.n_heads <= 0 || d.n_kv_heads <= 0 || d.n_heads % d.n_kv_heads ||
        !(hd == 64 || hd == 128 || hd == 256) || d.ffn_dim <= 0 || d.ffn_dim % 16 || d.vocab <= 0 ||
        d.max_seq <= 0 || (d.act_mode != HOLO_ACT_Q8 && d.act_mode != HOLO_ACT_F32) ||
        !emb_type_ok(d.emb_type, d.dim) ||
        !holo_quant_shape_ok(d.layer_type, d.n_heads * hd, d.dim) ||
        !holo_quant_shape_ok(d.layer_type, d.dim, d.n_heads * hd) ||
        !holo_quant_shape_ok(d.layer_type, d.ffn_dim, d.dim) ||
        !holo_quant_shape_ok(d.layer_type, d.dim, d.ffn_dim) ||
        !holo_quant_shape_ok(d.out_type, d.vocab, d.dim)) {
        holo_set_status(HOLO_E_ARG, "holo_model_create: unsupported shape or type");
        return nullptr;
    }
    HoloDevice *D = holo_dev();
    if (!D) return nullptr;
    HoloModel *m = new HoloModel();
    m->d = d;
    m->d.world = world;
    m->world = world;
    m->rank = d.rank;
    m->h0 = sh[0]; m->nh = sh[1];
    m->kh0 = sh[2]; m->nkv = sh[3];
    m->d0 = sh[4]; m->dim_loc = sh[5];
    m->f0 = sh[6]; m->ffn_loc = sh[7];
    m->v0 = sh[8]; m->vocab_loc = sh[9];
    m->q_dim = m->nh * hd;
    m->kv_dim = m->nkv * hd;
    m->q_dim_g = d.n_heads * hd;
    m->layers.resize(d.n_layers);
    m->max_splits = (d.max_seq + m->per_split - 1) / m->per_split;
    // the step kernel splits attention into 16-position pieces at the least
    m->step_max_splits = (d.max_seq + 15) / 16;
    const size_t kv_bytes = (size_t)d.n_layers * d.max_seq * m->kv_dim * (d.kv_f16 ? 2 : 4);
    bool ok = dev_alloc(&m->kc, kv_bytes) && dev_alloc(&m->vc, kv_bytes);
    // comm: the LL vectors x, att, h, logits (full length), 256-byte aligned
    {
        auto a256 = [](size_t v) { return (v + 255) & ~(size_t)255; };
        size_t o = 0;
        m->off_x = o; o = a256(o + sizeof(StepWord) * d.dim);
        m->off_att = o; o = a256(o + sizeof(StepWord) * m->q_dim_g);
        m->off_h = o; o = a256(o + sizeof(StepWord) * d.ffn_dim);
        m->off_log = o; o = a256(o + sizeof(StepWord) * d.vocab);
        if (world > 1) {   // sharded prompt passes
            m->off_rflag = o; o = a256(o + sizeof(unsigned long long) * STEP_MAX_RANKS);
            m->off_ratt = o; o = a256(o + sizeof(float) * PROMPT_ROWS * m->q_dim_g);
            m->off_rt = o; o = a256(o + sizeof(float) * PROMPT_ROWS * d.dim);
            m->off_rh = o; o = a256(o + sizeof(float) * PROMPT_ROWS * d.ffn_dim);
        }
        m->comm_bytes = o;
    }
    if (world > 1) {
        ok = ok && dev_alloc((void **)&m->d_row_done, sizeof(unsigned));
        if (ok) cudaMemset(m->d_row_done, 0, sizeof(unsigned));
    }
    ok = ok && dev_alloc((void **)&m->comm, m->comm_bytes);
    ok = ok && dev_alloc((void **)&m->qkv_ll, sizeof(StepWord) * (m->q_dim + 2 * m->kv_dim));
    // plain vectors of the one-launch-per-op graph (and the logits of both)
    ok = ok && dev_alloc((void **)&m->x, sizeof(float) * d.dim);
    ok = ok && dev_alloc((void **)&m->qkv, sizeof(float) * (m->q_dim + 2 * m->kv_dim));
    ok = ok && dev_alloc((void **)&m->att, sizeof(float) * m->q_dim_g);
    ok = ok && dev_alloc((void **)&m->h, sizeof(float) * d.ffn_dim);
    ok = ok && dev_alloc((void **)&m->logits, sizeof(float) * d.vocab);
    ok = ok && dev_alloc((void **)&m->probs, sizeof(float) * d.vocab);
    ok = ok && dev_alloc((void **)&m->kept_p, sizeof(float) * d.vocab);
    ok = ok && dev_alloc((void **)&m->kept_idx, sizeof(int) * d.vocab);
    ok = ok && dev_alloc((void **)&m->part,
                         sizeof(float) * (size_t)m->nh * std::max(m->max_splits, m->step_max_splits) * (hd + 4));
    ok = ok && dev_alloc((void **)&m->rvals, sizeof(float) * (d.max_seq + 1));
    ok = ok && dev_alloc((void **)&m->d_pos, sizeof(int) * 4);
    ok = ok && dev_alloc((void **)&m->d_seq, sizeof(int) * (d.max_seq + 1));
    ok = ok && dev_alloc((void **)&m->d_hist, sizeof(int) * (d.max_seq + 1));
    ok = ok && dev_alloc((void **)&m->d_nhist, sizeof(int) * 4);
    ok = ok && dev_alloc((void **)&m->d_out, sizeof(int) * (d.max_seq + 1));
    ok = ok && dev_alloc((void **)&m->d_last, sizeof(int) * 4);
    ok = ok && dev_alloc((void **)&m->d_bar, sizeof(unsigned long long) * 4);
    ok = ok && dev_alloc((void **)&m->d_att_cnt, sizeof(int) * m->nh);
    if (!ok) {
        holo_model_free(m);
        return nullptr;
    }
    for (auto &e : m->ev)
        if (cudaEventCreate(&e) != cudaSuccess) {
            holo_check_launch("holo_model_create: events");
            holo_model_free(m);
            return nullptr;
        }
    {
        // the persistent step kernel serves head_dim 128; HOLO_STEP=graph keeps
        // the one-launch-per-op graph
        const char *e = getenv("HOLO_STEP");
        m->step_kernel = hd == 128 && !(e && strcmp(e, "graph") == 0);
    }
    for (HoloLayer &L : m->layers) L.wv_type = L.w2_type = d.layer_type;
    m->emb_src = d.emb_type;
    m->d.emb_type = d.emb_type == 1 ? 1 : 0;   // quantized tables become F32 (set_globals)
    refresh_use_step(m);
    if (world > 1 && !m->use_step) {
        holo_set_status(HOLO_E_UNSUPPORTED,
                        "holo_model_create: sharding needs the step kernel (HOLO_STEP; Q8_0/Q4_0/Q4_K layers and output)");
        holo_model_free(m);
        return nullptr;
    }
    m->batch = d.batch <= 1 ? 1 : d.batch;
    if (m->batch > 1) {
        const int B = m->batch, S = d.max_seq + 1;
        const size_t kv_all = (size_t)B * d.n_layers * d.max_seq * m->kv_dim * (d.kv_f16 ? 2 : 4);
        bool bok = dev_alloc(&m->bkc, kv_all) && dev_alloc(&m->bvc, kv_all);
        bok = bok && dev_alloc((void **)&m->bx, sizeof(float) * B * d.dim) &&
              dev_alloc((void **)&m->bxn, sizeof(float) * B * d.dim) &&
              dev_alloc((void **)&m->bqkv, sizeof(float) * B * (m->q_dim + 2 * m->kv_dim)) &&
              dev_alloc((void **)&m->batt, sizeof(float) * B * m->q_dim) &&
              dev_alloc((void **)&m->bt, sizeof(float) * B * d.dim) &&
              dev_alloc((void **)&m->bhh, sizeof(float) * B * 2 * d.ffn_dim) &&
              dev_alloc((void **)&m->bh, sizeof(float) * B * d.ffn_dim) &&
              dev_alloc((void **)&m->blogits, sizeof(float) * B * d.vocab) &&
              dev_alloc((void **)&m->bprobs, sizeof(float) * B * d.vocab) &&
              dev_alloc((void **)&m->bkept_p, sizeof(float) * B * d.vocab) &&
              dev_alloc((void **)&m->bkept_idx, sizeof(int) * B * d.vocab) &&
              dev_alloc((void **)&m->bpart, sizeof(float) * B * d.n_heads * m->max_splits * (hd + 2)) &&
              dev_alloc((void **)&m->brvals, sizeof(float) * B * S) &&
              dev_alloc((void **)&m->bseq, sizeof(int) * B * S) && dev_alloc((void **)&m->bhist, sizeof(int) * B * S) &&
              dev_alloc((void **)&m->bout, sizeof(int) * B * S) && dev_alloc((void **)&m->bnhist, sizeof(int) * B) &&
              dev_alloc((void **)&m->blast, sizeof(int) * B) && dev_alloc((void **)&m->bpos, sizeof(int) * 4);
        if (!bok) {
            holo_model_free(m);
            return nullptr;
        }
        cudaMemset(m->bkc, 0, kv_all);
        cudaMemset(m->bvc, 0, kv_all);
        cudaMemset(m->bpos, 0, sizeof(int) * 4);
        cudaMemset(m->bnhist, 0, sizeof(int) * B);
        cudaMemset(m->bseq, 0, sizeof(int) * B * S);
        cudaMemset(m->brvals, 0, sizeof(float) * B * S);
    }
    cudaMemset(m->comm, 0, m->comm_bytes);
    cudaMemset(m->qkv_ll, 0, sizeof(StepWord) * (m->q_dim + 2 * m->kv_dim));
    cudaMemset(m->d_bar, 0, sizeof(unsigned long long) * 4);
    cudaMemset(m->d_att_cnt, 0, sizeof(int) * m->nh);
    cudaMemset(m->kc, 0, kv_bytes);
    cudaMemset(m->vc, 0, kv_bytes);
    cudaMemset(m->d_pos, 0, sizeof(int) * 4);
    cudaMemset(m->d_nhist, 0, sizeof(int) * 4);
    cudaMemset(m->d_seq, 0, sizeof(int) * (d.max_seq + 1));
    cudaMemset(m->rvals, 0, sizeof(float) * (d.max_seq + 1));
    cudaDeviceSynchronize();
    return m;
}

int holo_model_set_layer_types(void *model, int l, int wv_type, int w2_type) {
    HoloModel *m = (HoloModel *)model;
    if (!m || l < 0 || l >= m->d.n_layers) {
        holo_set_status(HOLO_E_ARG, "holo_model_set_layer_types: bad arguments");
        return HOLO_E_ARG;
    }
    const holo_model_desc &d = m->d;
    auto quant = [](int t) { return t == GT_Q8_0 || t == GT_Q4_0 || t == GT_Q4_K || t == GT_Q6_K; };
    if (!quant(wv_type) || !quant(w2_type) || !holo_quant_shape_ok(wv_type, m->kv_dim, d.dim) ||
        !holo_quant_shape_ok(w2_type, m->dim_loc, d.ffn_dim)) {
        holo_set_status(HOLO_E_ARG, "holo_model_set_layer_types: Wv / W2 type must be Q8_0, Q4_0, Q4_K or Q6_K "
                                    "and divide the matrix rows");
        return HOLO_E_ARG;
    }
    const bool mixed = wv_type != d.layer_type || w2_type != d.layer_type;
    if (mixed && (m->world > 1 || m->batch > 1)) {
        holo_set_status(HOLO_E_UNSUPPORTED, "holo_model_set_layer_types: per-layer types need batch 1 on one GPU");
        return HOLO_E_UNSUPPORTED;
    }
    HoloLayer &L = m->layers[l];
    if (L.wv_type != wv_type || L.w2_type != w2_type) {
        L.wv_type = wv_type;
        L.w2_type = w2_type;
        L.ready = false;   // the weights follow in holo_model_set_layer
        drop_graphs(m);
        refresh_use_step(m);
    }
    return HOLO_OK;
}

int holo_model_set_layer(void *model, int l, const float *attn_norm, const void *wq, const void *wk, const void *wv,
                         const void *wo, const float *ffn_norm, const void *w1, const void *w2, const void *w3) {
    HoloModel *m = (HoloModel *)model;
    if (!m || l < 0 || l >= m->d.n_layers || !attn_norm || !wq || !wk || !wv || !wo || !ffn_norm || !w1 || !w2 ||
        !w3) {
        holo_set_status(HOLO_E_ARG, "holo_model_set_layer: bad arguments");
        return HOLO_E_ARG;
    }
    const holo_model_desc &d = m->d;
    const int t = d.layer_type;
    cudaStream_t st = holo_stream();
    HoloLayer &L = m->layers[l];
    const int tv = L.wv_type, t2 = L.w2_type;
    drop_graphs(m);
    m->step_ready = false;
    if (!L.attn_norm && !upload_plain((void **)&L.attn_norm, attn_norm, sizeof(float) * d.dim, st))
        return HOLO_E_NOMEM;
    if (!L.ffn_norm && !upload_plain((void **)&L.ffn_norm, ffn_norm, sizeof(float) * d.dim, st))
        return HOLO_E_NOMEM;
    cudaMemcpyAsync(L.attn_norm, attn_norm, sizeof(float) * d.dim, cudaMemcpyDefault, st);
    cudaMemcpyAsync(L.ffn_norm, ffn_norm, sizeof(float) * d.dim, cudaMemcpyDefault, st);
    // this rank's rows of each matrix (all rows when world == 1); GGUF rows
    // are contiguous, so a row range is a byte range of the source
    const size_t row_dim = (size_t)gguf_row_bytes(t, d.dim);
    const int hd = d.head_dim;
    auto rows_of = [](const void *p, size_t first_row, size_t row_bytes) {
        return static_cast<const void *>(static_cast<const uint8_t *>(p) + first_row * row_bytes);
    };
    // [Wq; Wk; Wv] in one tiled buffer (each part a whole number of row-blocks);
    // a Wv of another type goes into a tiled buffer of its own
    const bool own_v = tv != t;
    const size_t bq = cuda_quant_tiled_bytes(t, m->q_dim, d.dim), bk = cuda_quant_tiled_bytes(t, m->kv_dim, d.dim);
    if (!L.wqkv && !dev_alloc((void **)&L.wqkv, bq + 2 * bk)) return HOLO_E_NOMEM;
    if (!upload_repack(L.wqkv, rows_of(wq, (size_t)m->h0 * hd, row_dim), t, m->q_dim, d.dim, st) ||
        !upload_repack(L.wqkv + bq, rows_of(wk, (size_t)m->kh0 * hd, row_dim), t, m->kv_dim, d.dim, st))
        return cuda_last_status();
    if (!own_v) {
        if (!upload_repack(L.wqkv + bq + bk, rows_of(wv, (size_t)m->kh0 * hd, row_dim), t, m->kv_dim, d.dim, st))
            return cuda_last_status();
        if (L.wv) cudaFree(L.wv);
        L.wv = nullptr;
    } else {
        if (L.wv) cudaFree(L.wv);
        L.wv = nullptr;
        if (!dev_alloc((void **)&L.wv, cuda_quant_tiled_bytes(tv, m->kv_dim, d.dim))) return HOLO_E_NOMEM;
        if (!upload_repack(L.wv, rows_of(wv, (size_t)m->kh0 * hd, gguf_row_bytes(tv, d.dim)), tv, m->kv_dim, d.dim,
                           st))
            return cuda_last_status();
        L.i_v = holo_weight_info(tv, m->kv_dim, d.dim, holo_q4k_layout());
    }
    L.i_qkv = holo_weight_info(t, m->q_dim + (own_v ? 1 : 2) * m->kv_dim, d.dim, holo_q4k_layout());
    if (!L.wo && !dev_alloc((void **)&L.wo, cuda_quant_tiled_bytes(t, m->dim_loc, m->q_dim_g))) return HOLO_E_NOMEM;
    if (!upload_repack(L.wo, rows_of(wo, m->d0, gguf_row_bytes(t, m->q_dim_g)), t, m->dim_loc, m->q_dim_g, st))
        return cuda_last_status();
    L.i_o = holo_weight_info(t, m->dim_loc, m->q_dim_g, holo_q4k_layout());
    // W1 and W3 interleaved by 16 rows: row-block b = W1 rows 16b..16b+15, W3 rows 16b..16b+15
    void *inter = nullptr;
    if (!dev_alloc(&inter, (size_t)2 * m->ffn_loc * row_dim)) return HOLO_E_NOMEM;
    const size_t band = 16 * row_dim;
    bool ok = cudaMemcpy2DAsync(inter, 2 * band, rows_of(w1, m->f0, row_dim), band, band, m->ffn_loc / 16,
                                cudaMemcpyDefault, st) == cudaSuccess &&
              cudaMemcpy2DAsync((uint8_t *)inter + band, 2 * band, rows_of(w3, m->f0, row_dim), band, band,
                                m->ffn_loc / 16, cudaMemcpyDefault, st) == cudaSuccess;
    if (!L.w13 && !dev_alloc((void **)&L.w13, cuda_quant_tiled_bytes(t, 2 * m->ffn_loc, d.dim))) {
        cudaFree(inter);
        return HOLO_E_NOMEM;
    }
    ok = ok && upload_repack(L.w13, inter, t, 2 * m->ffn_loc, d.dim, st);
    cudaStreamSynchronize(st);
    cudaFree(inter);
    if (!ok) {
        holo_check_launch("holo_model_set_layer: w1/w3");
        return cuda_last_status() ? cuda_last_status() : HOLO_E_ARG;
    }
    L.i_13 = holo_weight_info(t, 2 * m->ffn_loc, d.dim, holo_q4k_layout());
    if (L.w2 && L.i_2.type != t2) {   // a new type: the buffer size differs
        cudaFree(L.w2);
        L.w2 = nullptr;
    }
    if (!L.w2 && !dev_alloc((void **)&L.w2, cuda_quant_tiled_bytes(t2, m->dim_loc, d.ffn_dim))) return HOLO_E_NOMEM;
    if (!upload_repack(L.w2, rows_of(w2, m->d0, gguf_row_bytes(t2, d.ffn_dim)), t2, m->dim_loc, d.ffn_dim, st))
        return cuda_last_status();
    L.i_2 = holo_weight_info(t2, m->dim_loc, d.ffn_dim, holo_q4k_layout());
    cudaStreamSynchronize(st);
    L.ready = cuda_last_status() == HOLO_OK;
    return L.ready ? HOLO_OK : cuda_last_status();
}

int holo_model_set_globals(void *model, const void *tok_embeddings, const float *final_norm, const void *output) {
    HoloModel *m = (HoloModel *)model;
    if (!m || !tok_embeddings || !final_norm || !output) {
        holo_set_status(HOLO_E_ARG, "holo_model_set_globals: bad arguments");
        return HOLO_E_ARG;
    }
    const holo_model_desc &d = m->d;
    cudaStream_t st = holo_stream();
    drop_graphs(m);
    m->step_ready = false;
    const size_t eb = (size_t)d.vocab * d.dim * (d.emb_type == 1 ? 2 : 4);
    if (!m->emb && !dev_alloc(&m->emb, eb)) return HOLO_E_NOMEM;
    if (m->emb_src == GT_F32 || m->emb_src == GT_F16) {
        cudaMemcpyAsync(m->emb, tok_embeddings, eb, cudaMemcpyDefault, st);
    } else {
        // GGUF blocks: the table dequantized once, each row as get_embedding
        // (src/ai/llm.c:941-1008) decodes it
        const size_t raw = (size_t)d.vocab * gguf_row_bytes(m->emb_src, d.dim);
        void *staging = nullptr;
        if (!dev_alloc(&staging, raw)) return HOLO_E_NOMEM;
        bool ok = cudaMemcpyAsync(staging, tok_embeddings, raw, cudaMemcpyDefault, st) == cudaSuccess &&
                  holo_embedding_table_f32((float *)m->emb, staging, m->emb_src, d.vocab, d.dim,
                                           holo_q4k_layout() == HOLO_Q4K_GGML, st);
        cudaStreamSynchronize(st);
        cudaFree(staging);
        if (!ok) return cuda_last_status() ? cuda_last_status() : HOLO_E_ARG;
    }
    if (!m->final_norm && !dev_alloc((void **)&m->final_norm, sizeof(float) * d.dim)) return HOLO_E_NOMEM;
    cudaMemcpyAsync(m->final_norm, final_norm, sizeof(float) * d.dim, cudaMemcpyDefault, st);
    if (!m->out && !dev_alloc((void **)&m->out, cuda_quant_tiled_bytes(d.out_type, m->vocab_loc, d.dim)))
        return HOLO_E_NOMEM;
    const void *out_rows =
        static_cast<const uint8_t *>(output) + (size_t)m->v0 * gguf_row_bytes(d.out_type, d.dim);
    if (!upload_repack(m->out, out_rows, d.out_type, m->vocab_loc, d.dim, st)) return cuda_last_status();
    m->i_out = holo_weight_info(d.out_type, m->vocab_loc, d.dim, holo_q4k_layout());
    cudaStreamSynchronize(st);
    m->globals_ready = cuda_last_status() == HOLO_OK;
    return m->globals_ready ? HOLO_OK : cuda_last_status();
}

int holo_model_forward(void *model, int token, float *logits) {
    HoloModel *m = (HoloModel *)model;
    if (!model_ready(m)) return HOLO_E_ARG;
    if (m->h_pos >= m->d.max_seq || token < 0 || token >= m->d.vocab) {
        holo_set_status(HOLO_E_ARG, "holo_model_forward: position past max_seq or token out of range");
        return HOLO_E_ARG;
    }
    cudaStream_t st = holo_stream();
    dec_set_token_kernel<<<1, 1, 0, st>>>(m->d_seq, m->d_pos, token);
    if (m->use_step) {
        SampleArgs none{};
        if (!run_step(m, false, none, st)) return cuda_last_status() ? cuda_last_status() : HOLO_E_ARG;
        m->h_pos++;
        if (logits) {
            if (cudaMemcpyAsync(logits, m->logits, sizeof(float) * m->d.vocab, cudaMemcpyDeviceToHost, st) !=
                cudaSuccess)
                holo_check_launch("holo_model_forward: logits copy");
            cudaStreamSynchronize(st);
        }
        return cuda_last_status();
    }
    if (!m->g_forward) {
        SampleArgs none{};
        m->g_forward = capture_step(m, false, none);
        if (!m->g_forward) return cuda_last_status();
    }
    if (cudaGraphLaunch(m->g_forward, st) != cudaSuccess) {
        holo_check_launch("holo_model_forward: graph launch");
        return cuda_last_status();
    }
    m->h_pos++;
    if (logits) {
        if (cudaMemcpyAsync(logits, m->logits, sizeof(float) * m->d.vocab, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            holo_check_launch("holo_model_forward: logits copy");
        cudaStreamSynchronize(st);
    }
    return cuda_last_status();
}

int holo_model_prefill(void *model, const int *tokens, int n, float *logits) {
    HoloModel *m = (HoloModel *)model;
    if (!model_ready(m)) return HOLO_E_ARG;
    const int B = m->batch, S = m->d.max_seq + 1;
    int &hpos = B == 1 ? m->h_pos : m->h_bpos;
    if (!tokens || n <= 0 || hpos + n > m->d.max_seq) {
        holo_set_status(HOLO_E_ARG, "holo_model_prefill: no tokens or past max_seq");
        return HOLO_E_ARG;
    }
    for (long long i = 0; i < (long long)B * n; ++i)
        if (tokens[i] < 0 || tokens[i] >= m->d.vocab) {
            holo_set_status(HOLO_E_ARG, "holo_model_prefill: token out of range");
            return HOLO_E_ARG;
        }
    if (m->world > 1 && logits) {
        holo_set_status(HOLO_E_UNSUPPORTED, "holo_model_prefill: sharded, the logits come from the next step");
        return HOLO_E_UNSUPPORTED;
    }
    if (!prompt_supported(m)) {
        holo_set_status(HOLO_E_UNSUPPORTED, "holo_model_prefill: row passes need HOLO_ACT_Q8 at batch 1, "
                                            "Q8_0/Q4_0/Q4_K layers, head_dim 64/128/256, "
                                            "n_heads / n_kv_heads <= 16");
        return HOLO_E_UNSUPPORTED;
    }
    cudaStream_t st = holo_stream();
    const cudaError_t ce =
        B == 1 ? cudaMemcpyAsync(m->d_seq + hpos, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, st)
               : cudaMemcpy2DAsync(m->bseq + hpos, sizeof(int) * S, tokens, sizeof(int) * n, sizeof(int) * n, B,
                                   cudaMemcpyHostToDevice, st);
    if (ce != cudaSuccess) {
        holo_check_launch("holo_model_prefill: tokens");
        return cuda_last_status();
    }
    int last = 0;
    if (!prompt_rows(m, st, n, &last)) return cuda_last_status() ? cuda_last_status() : HOLO_E_ARG;
    hpos += n;
    if (logits) {
        // each sequence's last position: final RMSNorm fused into the output matvec
        float *dst = B == 1 ? m->logits : m->blogits;
        for (int b = 0; b < B; ++b) {
            MvLaunch a;
            a.x = m->rx + ((size_t)b * last + last - 1) * m->d.dim;
            a.y = dst + (size_t)b * m->d.vocab;
            a.norm_w = m->final_norm;
            a.eps = m->d.eps;
            a.act = m->d.act_mode;
            a.epi = MV_EPI_STORE;
            if (!holo_matvec_launch(m->out, m->i_out, a, st)) return cuda_last_status();
        }
        if (cudaMemcpyAsync(logits, dst, sizeof(float) * B * m->d.vocab, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            holo_check_launch("holo_model_prefill: logits copy");
    }
    cudaStreamSynchronize(st);
    return cuda_last_status();
}

int holo_model_set_prompt_mode(void *model, int rows) {
    HoloModel *m = (HoloModel *)model;
    if (!m || (rows != 0 && rows != 1)) {
        holo_set_status(HOLO_E_ARG, "holo_model_set_prompt_mode: mode 0 or 1");
        return HOLO_E_ARG;
    }
    m->prompt_mode = rows;
    return HOLO_OK;
}

int holo_model_load_logits(void *model, const float *logits) {
    HoloModel *m = (HoloModel *)model;
    if (!m || !logits) {
        holo_set_status(HOLO_E_ARG, "holo_model_load_logits: bad arguments");
        return HOLO_E_ARG;
    }
    cudaStream_t st = holo_stream();
    if (cudaMemcpyAsync(m->logits, logits, sizeof(float) * m->d.vocab, cudaMemcpyHostToDevice, st) != cudaSuccess)
        holo_check_launch("holo_model_load_logits");
    cudaStreamSynchronize(st);
    return cuda_last_status();
}

int holo_model_push_token(void *model, int token) {
    HoloModel *m = (HoloModel *)model;
    if (!m || m->h_nhist >= m->d.max_seq) {
        holo_set_status(HOLO_E_ARG, "holo_model_push_token: history full");
        return HOLO_E_ARG;
    }
    dec_push_kernel<<<1, 1, 0, holo_stream()>>>(m->d_hist, m->d_nhist, token);
    m->h_nhist++;
    return holo_check_launch("holo_model_push_token") ? HOLO_OK : cuda_last_status();
}

int holo_model_sample(void *model, const holo_sampler_desc *s, float r) {
    HoloModel *m = (HoloModel *)model;
    if (!m || !s) {
        holo_set_status(HOLO_E_ARG, "holo_model_sample: bad arguments");
        return -1;
    }
    cudaStream_t st = holo_stream();
    HoloDevice *D = holo_dev();
    SampleArgs a = make_args(m, s);
    a.gen = 0;
    if (!prepare_sampler()) return -1;
    cudaMemcpyAsync(m->rvals, &r, sizeof(float), cudaMemcpyHostToDevice, st);
    launch_pdl_smem(dec_sample_kernel, dim3(1), dim3(SM_THREADS), sizeof(SampleSmem), st, false, m->logits,
                    m->probs, m->kept_idx, m->kept_p, m->d_seq, m->d_hist, m->d_nhist, (const int *)m->d_pos,
                    (const float *)m->rvals, m->d_out, m->d_last, D ? D->status : nullptr, a, (size_t)0, (size_t)0);
    int tok = -1;
    cudaMemcpyAsync(&tok, m->d_last, sizeof(int), cudaMemcpyDeviceToHost, st);
    cudaStreamSynchronize(st);
    return cuda_last_status() == HOLO_OK ? tok : -1;
}

int holo_model_generate(void *model, const int *prompt, int n_prompt, int n_new, const holo_sampler_desc *s,
                        int seed, int *out) {
    HoloModel *m = (HoloModel *)model;
    if (!model_ready(m) || !prompt || !s || !out || n_prompt <= 0 || n_new <= 0 ||
        n_prompt + n_new > m->d.max_seq) {
        holo_set_status(HOLO_E_ARG, "holo_model_generate: bad arguments");
        return -1;
    }
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->d.vocab) {
            holo_set_status(HOLO_E_ARG, "holo_model_generate: prompt token out of range");
            return -1;
        }
    cudaStream_t st = holo_stream();
    // llm_generate (llm.c:1340-1420): srand(seed); one rand() per sampled token
    // when T != 0 (llm.c:1318-1321)
    std::vector<float> r(n_new, 0.0f);
    srand((unsigned)seed);
    if (s->temperature != 0.0f)
        for (int i = 0; i < n_new; ++i) r[i] = (float)rand() / RAND_MAX;
    holo_model_reset(m);
    cudaMemcpyAsync(m->rvals, r.data(), sizeof(float) * n_new, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(m->d_seq, prompt, sizeof(int) * n_prompt, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(m->d_hist, prompt, sizeof(int) * n_prompt, cudaMemcpyHostToDevice, st);
    const int nh = n_prompt;
    cudaMemcpyAsync(m->d_nhist, &nh, sizeof(int), cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
    SampleArgs a = make_args(m, s);
    a.gen = 1;
    a.n_prompt = n_prompt;
    const int steps = n_prompt + n_new - 1;
    // the prompt before its last token in row passes where supported; the
    // steps then start at the last prompt token
    const bool rows = n_prompt > 1 && prompt_supported(m);
    const int first = rows ? n_prompt - 1 : 0;
    if (m->use_step) {
        m->gen_args = a;
        cudaEventRecord(m->ev[0], st);
        if (rows && !prompt_rows(m, st, n_prompt - 1, nullptr)) return -1;
        for (int i = first; i < steps; ++i) {
            if (i == n_prompt - 1) cudaEventRecord(m->ev[1], st);
            if (!run_step(m, true, a, st)) return -1;
        }
        cudaEventRecord(m->ev[2], st);
        cudaMemcpyAsync(out, m->d_out, sizeof(int) * n_new, cudaMemcpyDeviceToHost, st);
        cudaStreamSynchronize(st);
        cudaEventElapsedTime(&m->last_prefill_ms, m->ev[0], m->ev[1]);
        cudaEventElapsedTime(&m->last_decode_ms, m->ev[1], m->ev[2]);
        m->h_pos = steps;
        m->h_nhist = n_prompt + n_new;
        return cuda_last_status() == HOLO_OK ? n_new : -1;
    }
    if (m->g_gen && memcmp(&a, &m->gen_args, sizeof(a)) != 0) {
        cudaGraphExecDestroy(m->g_gen);
        m->g_gen = nullptr;
    }
    if (!m->g_gen) {
        m->g_gen = capture_step(m, true, a);
        if (!m->g_gen) return -1;
        m->gen_args = a;
    }
    // steps 0 .. n_prompt-2 are prefill; each later step forwards one position
    // and samples one token (the first forwards the last prompt token)
    cudaEventRecord(m->ev[0], st);
    if (rows && !prompt_rows(m, st, n_prompt - 1, nullptr)) return -1;
    for (int i = first; i < steps; ++i) {
        if (i == n_prompt - 1) cudaEventRecord(m->ev[1], st);
        if (cudaGraphLaunch(m->g_gen, st) != cudaSuccess) {
            holo_check_launch("holo_model_generate: graph launch");
            return -1;
        }
    }
    cudaEventRecord(m->ev[2], st);
    cudaMemcpyAsync(out, m->d_out, sizeof(int) * n_new, cudaMemcpyDeviceToHost, st);
    cudaStreamSynchronize(st);
    cudaEventElapsedTime(&m->last_prefill_ms, m->ev[0], m->ev[1]);
    cudaEventElapsedTime(&m->last_decode_ms, m->ev[1], m->ev[2]);
    m->h_pos = steps;
    m->h_nhist = n_prompt + n_new;
    return cuda_last_status() == HOLO_OK ? n_new : -1;
}

int holo_model_launch_steps(void *model, int n_steps) {
    HoloModel *m = (HoloModel *)model;
    if (m && m->use_step && n_steps >= 0 && m->h_pos + n_steps <= m->d.max_seq - 1) {
        cudaStream_t st = holo_stream();
        for (int i = 0; i < n_steps; ++i)
            if (!run_step(m, true, m->gen_args, st)) return cuda_last_status();
        m->h_pos += n_steps;
        return HOLO_OK;
    }
    if (!m || !m->g_gen || n_steps < 0 || m->h_pos + n_steps > m->d.max_seq - 1) {
        holo_set_status(HOLO_E_ARG, "holo_model_launch_steps: no generation graph or past max_seq");
        return HOLO_E_ARG;
    }
    cudaStream_t st = holo_stream();
    for (int i = 0; i < n_steps; ++i)
        if (cudaGraphLaunch(m->g_gen, st) != cudaSuccess) {
            holo_check_launch("holo_model_launch_steps");
            return cuda_last_status();
        }
    m->h_pos += n_steps;
    return HOLO_OK;
}

int holo_model_debug_vector(void *model, int which, float *dst) {
    HoloModel *m = (HoloModel *)model;
    if (!m || !dst) return -1;
    const float *src = nullptr;
    int n = 0;
    switch (which) {
    case 0: src = m->x; n = m->d.dim; break;
    case 1: src = m->qkv; n = m->q_dim + 2 * m->kv_dim; break;
    case 2: src = m->att; n = m->q_dim_g; break;
    case 3: src = m->h; n = m->d.ffn_dim; break;
    case 4: src = m->logits; n = m->d.vocab; break;
    default: return -1;
    }
    cudaStream_t st = holo_stream();
    if (cudaMemcpyAsync(dst, src, sizeof(float) * n, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
        holo_check_launch("holo_model_debug_vector");
        return -1;
    }
    return n;
}

int holo_model_pos(void *model) { return model ? ((HoloModel *)model)->h_pos : -1; }

int holo_model_last_timing(void *model, float *prefill_ms, float *decode_ms) {
    HoloModel *m = (HoloModel *)model;
    if (!m) return HOLO_E_ARG;
    if (prefill_ms) *prefill_ms = m->last_prefill_ms;
    if (decode_ms) *decode_ms = m->last_decode_ms;
    return HOLO_OK;
}

int holo_model_forward_batch(void *model, const int *tokens, float *logits) {
    HoloModel *m = (HoloModel *)model;
    if (!model_ready(m) || m->batch < 2 || !tokens || m->h_bpos >= m->d.max_seq) {
        holo_set_status(HOLO_E_ARG, "holo_model_forward_batch: batched model, tokens, position below max_seq");
        return HOLO_E_ARG;
    }
    const int B = m->batch, S = m->d.max_seq + 1;
    for (int b = 0; b < B; ++b)
        if (tokens[b] < 0 || tokens[b] >= m->d.vocab) {
            holo_set_status(HOLO_E_ARG, "holo_model_forward_batch: token out of range");
            return HOLO_E_ARG;
        }
    cudaStream_t st = holo_stream();
    // column h_bpos of every sequence's token list
    if (cudaMemcpy2DAsync(m->bseq + m->h_bpos, sizeof(int) * S, tokens, sizeof(int), sizeof(int), B,
                          cudaMemcpyHostToDevice, st) != cudaSuccess)
        return holo_check_launch("holo_model_forward_batch: tokens") ? HOLO_E_ARG : cuda_last_status();
    SampleArgs none{};
    if (!run_batch_step(m, 1, none, st)) return cuda_last_status() ? cuda_last_status() : HOLO_E_ARG;
    m->h_bpos++;
    if (logits) {
        if (cudaMemcpyAsync(logits, m->blogits, sizeof(float) * B * m->d.vocab, cudaMemcpyDeviceToHost, st) !=
            cudaSuccess)
            holo_check_launch("holo_model_forward_batch: logits copy");
    }
    cudaStreamSynchronize(st);
    return cuda_last_status();
}

int holo_model_generate_batch(void *model, const int *prompts, int n_prompt, int n_new, const holo_sampler_desc *s,
                              const int *seeds, int *out) {
    HoloModel *m = (HoloModel *)model;
    if (!model_ready(m) || m->batch < 2 || !prompts || !s || !seeds || !out || n_prompt <= 0 || n_new <= 0 ||
        n_prompt + n_new > m->d.max_seq) {
        holo_set_status(HOLO_E_ARG, "holo_model_generate_batch: bad arguments");
        return -1;
    }
    const int B = m->batch, S = m->d.max_seq + 1;
    for (int i = 0; i < B * n_prompt; ++i)
        if (prompts[i] < 0 || prompts[i] >= m->d.vocab) {
            holo_set_status(HOLO_E_ARG, "holo_model_generate_batch: prompt token out of range");
            return -1;
        }
    cudaStream_t st = holo_stream();
    // llm_generate per sequence (llm.c:1340-1420): srand(seed_b), one rand()
    // per sampled token when T != 0
    std::vector<float> r((size_t)B * S, 0.0f);
    for (int b = 0; b < B; ++b) {
        srand((unsigned)seeds[b]);
        if (s->temperature != 0.0f)
            for (int i = 0; i < n_new; ++i) r[(size_t)b * S + i] = (float)rand() / RAND_MAX;
    }
    holo_model_reset(m);
    std::vector<int> nh(B, n_prompt);
    cudaMemcpyAsync(m->brvals, r.data(), sizeof(float) * B * S, cudaMemcpyHostToDevice, st);
    cudaMemcpy2DAsync(m->bseq, sizeof(int) * S, prompts, sizeof(int) * n_prompt, sizeof(int) * n_prompt, B,
                      cudaMemcpyHostToDevice, st);
    cudaMemcpy2DAsync(m->bhist, sizeof(int) * S, prompts, sizeof(int) * n_prompt, sizeof(int) * n_prompt, B,
                      cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(m->bnhist, nh.data(), sizeof(int) * B, cudaMemcpyHostToDevice, st);
    SampleArgs a = make_args(m, s);
    a.gen = 1;
    a.n_prompt = n_prompt;
    const int steps = n_prompt + n_new - 1;
    SampleArgs none{};
    // the prompts before their last token in row passes where supported
    const bool rows = n_prompt > 1 && prompt_supported(m);
    cudaEventRecord(m->ev[0], st);
    if (rows && !prompt_rows(m, st, n_prompt - 1, nullptr)) return -1;
    for (int i = rows ? n_prompt - 1 : 0; i < steps; ++i) {
        if (i == n_prompt - 1) cudaEventRecord(m->ev[1], st);
        if (!run_batch_step(m, i < n_prompt - 1 ? 0 : 2, i < n_prompt - 1 ? none : a, st)) return -1;
    }
    cudaEventRecord(m->ev[2], st);
    cudaMemcpy2DAsync(out, sizeof(int) * n_new, m->bout, sizeof(int) * S, sizeof(int) * n_new, B,
                      cudaMemcpyDeviceToHost, st);
    cudaStreamSynchronize(st);
    cudaEventElapsedTime(&m->last_prefill_ms, m->ev[0], m->ev[1]);
    cudaEventElapsedTime(&m->last_decode_ms, m->ev[1], m->ev[2]);
    m->h_bpos = steps;
    return cuda_last_status() == HOLO_OK ? n_new : -1;
}

int holo_model_shard(const holo_model_desc *desc, int *ranges) {
    if (!desc || !ranges || !shard_of(*desc, ranges)) {
        holo_set_status(HOLO_E_ARG, "holo_model_shard: desc cannot be sharded");
        return HOLO_E_ARG;
    }
    return HOLO_OK;
}

int holo_model_comm_handle(void *model, void *handle) {
    HoloModel *m = (HoloModel *)model;
    if (!m || !handle) {
        holo_set_status(HOLO_E_ARG, "holo_model_comm_handle: bad arguments");
        return HOLO_E_ARG;
    }
    CommHandle h{};
    if (cudaIpcGetMemHandle(&h.ipc, m->comm) != cudaSuccess) {
        holo_check_launch("holo_model_comm_handle: cudaIpcGetMemHandle");
        return cuda_last_status() ? cuda_last_status() : HOLO_E_COMM;
    }
    HoloDevice *D = holo_dev();
    h.rank = m->rank;
    h.world = m->world;
    h.grid = D ? D->sms : 0;
    h.magic = COMM_MAGIC;
    h.comm_bytes = m->comm_bytes;
    memset(handle, 0, HOLO_COMM_HANDLE_BYTES);
    memcpy(handle, &h, sizeof(h));
    return HOLO_OK;
}

int holo_model_open_peers(void *model, const void *handles) {
    HoloModel *m = (HoloModel *)model;
    if (!m || !handles) {
        holo_set_status(HOLO_E_ARG, "holo_model_open_peers: bad arguments");
        return HOLO_E_ARG;
    }
    HoloDevice *D = holo_dev();
    const int grid = D ? D->sms : 0;
    // every rank's handle must describe the same model and grid, in rank order
    for (int r = 0; r < m->world; ++r) {
        CommHandle h;
        memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)r * HOLO_COMM_HANDLE_BYTES, sizeof(h));
        if (h.magic != COMM_MAGIC || h.rank != r || h.world != m->world || h.grid != grid ||
            h.comm_bytes != m->comm_bytes) {
            holo_set_status(HOLO_E_COMM, "holo_model_open_peers: handles differ in rank, world, grid or model");
            return HOLO_E_COMM;
        }
    }
    for (int r = 0; r < m->world; ++r) {
        if (r == m->rank || m->peer[r]) continue;
        CommHandle h;
        memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)r * HOLO_COMM_HANDLE_BYTES, sizeof(h));
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h.ipc, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            holo_check_launch("holo_model_open_peers: cudaIpcOpenMemHandle");
            return cuda_last_status() ? cuda_last_status() : HOLO_E_COMM;
        }
        m->peer[r] = static_cast<uint8_t *>(p);
    }
    m->peers_ready = true;
    return HOLO_OK;
}

void holo_model_reset(void *model) {
    HoloModel *m = (HoloModel *)model;
    if (!m) return;
    cudaStream_t st = holo_stream();
    cudaMemsetAsync(m->d_pos, 0, sizeof(int), st);
    cudaMemsetAsync(m->d_nhist, 0, sizeof(int), st);
    // one GPU: launch counters (the LL epochs) restart with cleared LL
    // vectors.  Sharded, they only grow: the epochs must agree across ranks,
    // which reset at different times.
    if (m->world == 1) {
        cudaMemsetAsync(m->d_bar, 0, sizeof(unsigned long long) * 4, st);
        cudaMemsetAsync(m->comm, 0, m->comm_bytes, st);
        cudaMemsetAsync(m->qkv_ll, 0, sizeof(StepWord) * (m->q_dim + 2 * m->kv_dim), st);
    }
    cudaMemsetAsync(m->d_att_cnt, 0, sizeof(int) * m->nh, st);
    if (m->batch > 1) {
        cudaMemsetAsync(m->bpos, 0, sizeof(int), st);
        cudaMemsetAsync(m->bnhist, 0, sizeof(int) * m->batch, st);
        m->h_bpos = 0;
    }
    cudaStreamSynchronize(st);
    m->h_pos = 0;
    m->h_nhist = 0;
}

void holo_model_free(void *model) {
    HoloModel *m = (HoloModel *)model;
    if (!m) return;
    cudaDeviceSynchronize();
    drop_graphs(m);
    for (auto &e : m->ev)
        if (e) cudaEventDestroy(e);
    for (uint8_t *&p : m->peer)
        if (p) {
            cudaIpcCloseMemHandle(p);
            p = nullptr;
        }
    for (auto &L : m->layers) {
        cudaFree(L.attn_norm); cudaFree(L.ffn_norm); cudaFree(L.wqkv); cudaFree(L.wo); cudaFree(L.w13);
        cudaFree(L.w2); cudaFree(L.wv);
    }
    void *bbufs[] = {m->bx, m->bxn, m->bqkv, m->batt, m->bt, m->bhh, m->bh, m->blogits, m->bpart, m->brvals,
                     m->bprobs, m->bkept_p, m->bkept_idx,
                     m->bkc, m->bvc, m->bseq, m->bhist, m->bout, m->bnhist, m->blast, m->bpos, m->bscratch};
    for (void *p : bbufs) cudaFree(p);
    void *rbufs[] = {m->rx, m->rxn, m->rqkv, m->ratt, m->rt, m->rhh, m->rh, m->rscratch};
    for (void *p : rbufs) cudaFree(p);
    void *bufs[] = {m->emb, m->final_norm, m->out, m->kc, m->vc, m->comm, m->qkv_ll, m->x, m->qkv, m->att,
                    m->h, m->logits, m->part, m->probs, m->kept_p, m->rvals, m->kept_idx, m->d_pos, m->d_seq, m->d_hist,
                    m->d_nhist, m->d_out, m->d_last, m->d_layers, m->d_pf, m->d_bar, m->d_att_cnt, m->d_row_done};
    for (void *p : bufs) cudaFree(p);
    delete m;
}

}  // extern "C"
