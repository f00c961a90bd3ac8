// ops.cu -- the non-matvec entry points of the reference ABI: vectors,
// activations, norms, softmax, attention over fp32 caches, RoPE, embedding
// rows and argmax (src/ai/cuda_ops.cu:247-340, 1401-1595, 1600-2413).
// Arithmetic follows the reference CPU engine (src/ai/tensor.c, llm.c) where
// the two differ.
#include "holo_common.cuh"
#include "mv_device.cuh"

#include <cfloat>
#include <cstdio>

namespace {

constexpr int EW_THREADS = 256;

inline unsigned ew_grid(long long n, int per_thread = 1) {
    long long g = (n + (long long)EW_THREADS * per_thread - 1) / ((long long)EW_THREADS * per_thread);
    return (unsigned)(g < 1 ? 1 : g);
}

__global__ void vec_add_kernel(float *dst, const float *a, const float *b, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = a[i] + b[i];
}
__global__ void vec_mul_kernel(float *dst, const float *a, const float *b, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = a[i] * b[i];
}
__global__ void vec_scale_kernel(float *dst, const float *a, float s, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = a[i] * s;
}

template <int OP>   // 0 silu, 1 gelu, 2 relu
__global__ void act_kernel(float *x, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v = x[i];
    if (OP == 0) x[i] = v / (1.0f + expf(-v));                       // tensor.c:218
    else if (OP == 1) x[i] = 0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * v * v * v)));
    else x[i] = v < 0.0f ? 0.0f : v;
}
// dst = silu(a) * b (llm.c:1235-1236: silu then vec_mul)
__global__ void silu_mul_kernel(float *dst, const float *a, const float *b, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v = a[i];
    dst[i] = (v / (1.0f + expf(-v))) * b[i];
}

// ---------------------------------------------------------------------------
// block reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
template <bool MAX>
__device__ float block_reduce(float v, float *sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = MAX ? warp_max(v) : warp_sum(v);
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float r = MAX ? -FLT_MAX : 0.0f;
    for (int i = 0; i < nw; i++) r = MAX ? fmaxf(r, sh[i]) : r + sh[i];
    return r;
}

// tensor.c:242-255: rms = sqrt(sum(x^2)/n + eps); dst = x * (1/rms) * w
__global__ void rms_norm_kernel(float *dst, const float *x, const float *w, int n, float eps) {
    __shared__ float sh[32];
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(x[i], x[i], s);
    s = block_reduce<false>(s, sh);
    const float scale = 1.0f / sqrtf(s / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = x[i] * scale * w[i];
}

// tensor.c:300-319
__global__ void softmax_kernel(float *dst, const float *x, int n) {
    __shared__ float sh[32];
    float m = -FLT_MAX;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
    m = block_reduce<true>(m, sh);
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float e = expf(x[i] - m);
        dst[i] = e;
        s += e;
    }
    s = block_reduce<false>(s, sh);
    const float inv = 1.0f / s;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] *= inv;
}

// ---------------------------------------------------------------------------
// decode attention over fp32 caches, split over positions (flash-decoding):
// CTA (head h, split s) folds positions [p0, p1) with an online softmax into
// (m, l, acc[hd]); a second kernel merges the splits.  GQA: query head h reads
// KV head kv_base + h / group (src/ai/llm.c:1173-1177).
// ---------------------------------------------------------------------------
constexpr int ATT_WARPS = 4;
constexpr int ATT_MAX_HD = 256;

// the cache element as float (fp32 caches: the reference's; an fp16 cache
// would convert here)
template <typename KV>
__device__ __forceinline__ float kv_load(const KV *p) { return static_cast<float>(*p); }

template <typename KV>
__global__ void __launch_bounds__(ATT_WARPS * 32)
attn_split_kernel(float *__restrict__ part, const float *__restrict__ q, const KV *__restrict__ kc,
                  const KV *__restrict__ vc, int kv_len, int hd, int kv_stride, int kv_base, int group,
                  int per_split, float scale) {
    const int h = blockIdx.x, s = blockIdx.y, nsplit = gridDim.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvh = kv_base + h / group;
    const int p0 = s * per_split, p1 = min(kv_len, p0 + per_split);
    constexpr int PER = ATT_MAX_HD / 32;
    float qf[PER], acc[PER];
#pragma unroll
    for (int i = 0; i < PER; i++) {
        int d = lane + 32 * i;
        qf[i] = d < hd ? q[(size_t)h * hd + d] : 0.0f;
        acc[i] = 0.0f;
    }
    float m = -FLT_MAX, l = 0.0f;
    for (int p = p0 + warp; p < p1; p += ATT_WARPS) {
        const KV *kr = kc + (size_t)p * kv_stride + (size_t)kvh * hd;
        const KV *vr = vc + (size_t)p * kv_stride + (size_t)kvh * hd;
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < PER; i++) {
            int d = lane + 32 * i;
            if (d < hd) dot = fmaf(qf[i], kv_load(kr + d), dot);
        }
        dot = warp_sum(dot) * scale;
        float mn = fmaxf(m, dot);
        float corr = expf(m - mn), e = expf(dot - mn);
        l = l * corr + e;
#pragma unroll
        for (int i = 0; i < PER; i++) {
            int d = lane + 32 * i;
            if (d < hd) acc[i] = acc[i] * corr + e * kv_load(vr + d);
        }
        m = mn;
    }
    // merge the warps of this CTA
    __shared__ float sm_m[ATT_WARPS], sm_l[ATT_WARPS];
    __shared__ float sm_acc[ATT_WARPS][ATT_MAX_HD];
    if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
#pragma unroll
    for (int i = 0; i < PER; i++) {
        int d = lane + 32 * i;
        if (d < hd) sm_acc[warp][d] = acc[i];
    }
    __syncthreads();
    float M = -FLT_MAX;
    for (int w = 0; w < ATT_WARPS; w++) M = fmaxf(M, sm_m[w]);
    float *out = part + ((size_t)h * nsplit + s) * (hd + 2);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float a = 0.0f;
        for (int w = 0; w < ATT_WARPS; w++)
            if (sm_l[w] > 0.0f) a += sm_acc[w][d] * expf(sm_m[w] - M);
        out[2 + d] = a;
    }
    if (threadIdx.x == 0) {
        float L = 0.0f;
        for (int w = 0; w < ATT_WARPS; w++)
            if (sm_l[w] > 0.0f) L += sm_l[w] * expf(sm_m[w] - M);
        out[0] = M;
        out[1] = L;
    }
}

__global__ void attn_merge_kernel(float *__restrict__ dst, const float *__restrict__ part, int hd, int nsplit) {
    const int h = blockIdx.x;
    const float *ph = part + (size_t)h * nsplit * (hd + 2);
    float M = -FLT_MAX;
    for (int s = 0; s < nsplit; s++)
        if (ph[(size_t)s * (hd + 2) + 1] > 0.0f) M = fmaxf(M, ph[(size_t)s * (hd + 2)]);
    float L = 0.0f;
    for (int s = 0; s < nsplit; s++) {
        const float *ps = ph + (size_t)s * (hd + 2);
        if (ps[1] > 0.0f) L += ps[1] * expf(ps[0] - M);
    }
    const float inv = 1.0f / L;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float a = 0.0f;
        for (int s = 0; s < nsplit; s++) {
            const float *ps = ph + (size_t)s * (hd + 2);
            if (ps[1] > 0.0f) a += ps[2 + d] * expf(ps[0] - M);
        }
        dst[(size_t)h * hd + d] = a * inv;
    }
}

// naive attention pieces of the reference ABI (src/ai/cuda_ops.cu:1600-1640)
__global__ void att_scores_kernel(float *dst, const float *Q, const float *K, int seq_len, int kv_len,
                                  int hd, float scale) {
    int i = blockIdx.y, j = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= seq_len || j >= kv_len) return;
    float s = 0.0f;
    for (int d = 0; d < hd; d++) s = fmaf(Q[(size_t)i * hd + d], K[(size_t)j * hd + d], s);
    dst[(size_t)i * kv_len + j] = s * scale;
}
__global__ void att_apply_kernel(float *dst, const float *S, const float *V, int seq_len, int kv_len, int hd) {
    int i = blockIdx.y, d = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= seq_len || d >= hd) return;
    float s = 0.0f;
    for (int j = 0; j < kv_len; j++) s = fmaf(S[(size_t)i * kv_len + j], V[(size_t)j * hd + d], s);
    dst[(size_t)i * hd + d] = s;
}

// RoPE, rotate-half pairs (i, i + hd/2), frequency 1/base^(2i/hd) (llm.c:1135-1163)
__global__ void rope_kernel(float *q, float *k, int pos, int hd, int n_heads, int n_kv_heads, float base) {
    const int h = blockIdx.x, i = threadIdx.x, half = hd / 2;
    if (i >= half) return;
    float c, s;
    rope_cos_sin(pos, i, hd, base, c, s);
    if (h < n_heads) {
        float *qh = q + (size_t)h * hd;
        rope_rotate(qh[i], qh[i + half], c, s);
    }
    if (h < n_kv_heads) {
        float *kh = k + (size_t)h * hd;
        rope_rotate(kh[i], kh[i + half], c, s);
    }
}

// embedding rows (llm.c:943-1008 value semantics): value i of row `token`
template <int TYPE>
__device__ __forceinline__ float emb_value(const uint8_t *table, int token, int dim, int i) {
    if (TYPE == GT_F32) {
        return reinterpret_cast<const float *>(table)[(size_t)token * dim + i];
    } else if (TYPE == GT_F16) {
        return __half2float(reinterpret_cast<const __half *>(table)[(size_t)token * dim + i]);
    } else if (TYPE == GT_Q8_0) {
        const uint8_t *blk = table + ((size_t)token * (dim / 32) + i / 32) * 34;
        return half_bits_to_float(blk[0] | (blk[1] << 8)) * (float)(int8_t)blk[2 + i % 32];
    } else if (TYPE == GT_Q4_0) {
        const uint8_t *blk = table + ((size_t)token * (dim / 32) + i / 32) * 18;
        int j = i % 32;
        int nib = j < 16 ? (blk[2 + j] & 0xf) : (blk[2 + j - 16] >> 4);
        return half_bits_to_float(blk[0] | (blk[1] << 8)) * (float)(nib - 8);
    } else {  // Q6_K, value layout of quant.c:241-271
        const uint8_t *blk = table + ((size_t)token * (dim / 256) + i / 256) * 210;
        int j = i % 256, n = j / 128, pc = j % 128, l = pc % 32, which = pc / 32;
        const uint8_t *ql = blk + n * 64, *qh = blk + 128 + n * 32;
        const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192) + n * 8;
        int lowbits = (which == 0) ? (ql[l] & 0xF) : (which == 1) ? (ql[l + 32] & 0xF)
                    : (which == 2) ? (ql[l] >> 4) : (ql[l + 32] >> 4);
        int q = (lowbits | (((qh[l] >> (2 * which)) & 3) << 4)) - 32;
        float d = half_bits_to_float(blk[208] | (blk[209] << 8));
        return d * (float)sc[l / 16 + 2 * which] * (float)q;
    }
}

template <int TYPE>
__global__ void embedding_kernel(float *dst, const uint8_t *table, int token, int dim) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < dim) dst[i] = emb_value<TYPE>(table, token, dim, i);
}

// Q4_K embedding row (the reference's GPU dispatcher, llm_cuda.c:166-186, has
// no Q4_K case): value i of the row, decoded as quant.c:277-311 does (scale
// unpack quant.c:290-297, sub-block j = 16 bytes, low nibble -> position l,
// high -> l + 16) or, ggml != 0, as llama.cpp packs the block
// (get_scale_min_k4, cuda_ops.cu:684-692; 32 bytes per 64 values, low
// nibbles the first 32).  y = (d*sc)*q - dmin*m, each product rounded once.
__device__ __forceinline__ float q4k_emb_value(const uint8_t *table, int token, int dim, int i, int ggml) {
    const uint8_t *blk = table + ((size_t)token * (dim / 256) + i / 256) * 144;
    const int v = i % 256, j = v / 32, l = v % 32;
    const uint8_t *q = blk + 4;
    int sc, mn, nib;
    if (!ggml) {
        if (j < 4) {
            sc = q[j] & 0x3f;
            mn = q[j + 4] & 0x3f;
        } else {
            sc = ((q[j + 4] & 0x0f) << 2) | (q[j - 4] >> 6);
            mn = ((q[j + 4] >> 4) << 2) | (q[j] >> 6);
        }
        const uint8_t byte = blk[16 + j * 16 + (l & 15)];
        nib = l < 16 ? (byte & 0x0f) : (byte >> 4);
    } else {
        if (j < 4) {
            sc = q[j] & 63;
            mn = q[j + 4] & 63;
        } else {
            sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
            mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
        }
        const uint8_t byte = blk[16 + (j >> 1) * 32 + l];
        nib = (j & 1) ? (byte >> 4) : (byte & 0x0f);
    }
    const float d = half_bits_to_float(blk[0] | (blk[1] << 8)), dmin = half_bits_to_float(blk[2] | (blk[3] << 8));
    const float scale = __fmul_rn(d, (float)sc), mval = __fmul_rn(dmin, (float)mn);
    return __fsub_rn(__fmul_rn(scale, (float)nib), mval);
}

__global__ void q4k_embedding_kernel(float *dst, const uint8_t *table, int token, int dim, int ggml) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < dim) dst[i] = q4k_emb_value(table, token, dim, i, ggml);
}

// every row of a table (row = blockIdx.y): dst [rows][dim] fp32
template <int TYPE>
__global__ void embedding_table_kernel(float *dst, const uint8_t *table, int dim, int ggml) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x, token = blockIdx.y;
    if (i >= dim) return;
    dst[(size_t)token * dim + i] = TYPE == GT_Q4_K ? q4k_emb_value(table, token, dim, i, ggml)
                                                   : emb_value<TYPE>(table, token, dim, i);
}

// argmax, first maximum wins (tensor.c:460-470)
__device__ __forceinline__ void argmax_merge(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}
__global__ void argmax_partial_kernel(const float *x, int n, float *vals, int *idxs) {
    const int per = (n + gridDim.x - 1) / gridDim.x;
    const int lo = blockIdx.x * per, hi = min(n, lo + per);
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) argmax_merge(bv, bi, x[i], i);
    __shared__ float sv[EW_THREADS];
    __shared__ int si[EW_THREADS];
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            float v = sv[threadIdx.x + s];
            int i = si[threadIdx.x + s];
            float b = sv[threadIdx.x];
            int j = si[threadIdx.x];
            argmax_merge(b, j, v, i);
            sv[threadIdx.x] = b;
            si[threadIdx.x] = j;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) { vals[blockIdx.x] = sv[0]; idxs[blockIdx.x] = si[0]; }
}
__global__ void argmax_final_kernel(const float *vals, const int *idxs, int nparts, int *out) {
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    for (int i = 0; i < nparts; i++) argmax_merge(bv, bi, vals[i], idxs[i]);
    *out = bi == INT_MAX ? 0 : bi;
}

__global__ void dot_partial_kernel(const float *a, const float *b, int n, float *part) {
    __shared__ float sh[32];
    float s = 0.0f;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) s = fmaf(a[i], b[i], s);
    s = block_reduce<false>(s, sh);
    if (threadIdx.x == 0) part[blockIdx.x] = s;
}
__global__ void sum_parts_kernel(const float *part, int n, float *out) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += part[i];
    *out = s;
}

bool args_ok(const void *a, int n, const char *what) {
    if (!a || n < 0) { holo_set_status(HOLO_E_ARG, what); return false; }
    return holo_dev() != nullptr;
}

void run_attention(float *dst, const float *q, const float *kc, const float *vc, int kv_len, int hd,
                   int n_heads, int kv_stride, int kv_base, int group) {
    if (hd <= 0 || hd > ATT_MAX_HD || kv_len <= 0 || n_heads <= 0 || group <= 0) {
        holo_set_status(HOLO_E_ARG, "attention: bad shape");
        return;
    }
    HoloDevice *D = holo_dev();
    cudaStream_t st = holo_stream();
    int target = max(1, (2 * D->sms + n_heads - 1) / n_heads);
    int per_split = max(64, (kv_len + target - 1) / target);
    int nsplit = (kv_len + per_split - 1) / per_split;
    float *part = (float *)holo_tmp((size_t)n_heads * nsplit * (hd + 2) * sizeof(float));
    if (!part) return;
    attn_split_kernel<float><<<dim3(n_heads, nsplit), ATT_WARPS * 32, 0, st>>>(
        part, q, kc, vc, kv_len, hd, kv_stride, kv_base, group, per_split, 1.0f / sqrtf((float)hd));
    attn_merge_kernel<<<n_heads, 128, 0, st>>>(dst, part, hd, nsplit);
    holo_check_launch("attention launch");
}

}  // namespace

// The fp32 values of every row of a raw GGUF embedding table (Q8_0, Q4_0,
// Q4_K in the quant.c or, ggml_q4k, the llama.cpp packing, Q6_K), each as
// get_embedding (src/ai/llm.c:941-1008) decodes it: dst [rows][dim].
bool holo_embedding_table_f32(float *dst, const void *table, int type, int rows, int dim, bool ggml_q4k,
                              cudaStream_t st) {
    const dim3 grid((dim + EW_THREADS - 1) / EW_THREADS, rows);
    const uint8_t *t = (const uint8_t *)table;
    switch (type) {
    case GT_Q8_0: embedding_table_kernel<GT_Q8_0><<<grid, EW_THREADS, 0, st>>>(dst, t, dim, 0); break;
    case GT_Q4_0: embedding_table_kernel<GT_Q4_0><<<grid, EW_THREADS, 0, st>>>(dst, t, dim, 0); break;
    case GT_Q4_K: embedding_table_kernel<GT_Q4_K><<<grid, EW_THREADS, 0, st>>>(dst, t, dim, ggml_q4k ? 1 : 0); break;
    case GT_Q6_K: embedding_table_kernel<GT_Q6_K><<<grid, EW_THREADS, 0, st>>>(dst, t, dim, 0); break;
    default:
        holo_set_status(HOLO_E_ARG, "embedding table: type");
        return false;
    }
    return holo_check_launch("embedding table");
}

extern "C" {

void cuda_vec_add(float *dst, const float *a, const float *b, int n) {
    if (!args_ok(dst, n, "cuda_vec_add") || n == 0) return;
    vec_add_kernel<<<ew_grid(n), EW_THREADS, 0, holo_stream()>>>(dst, a, b, n);
    holo_check_launch("cuda_vec_add");
}
void cuda_vec_mul(float *dst, const float *a, const float *b, int n) {
    if (!args_ok(dst, n, "cuda_vec_mul") || n == 0) return;
    vec_mul_kernel<<<ew_grid(n), EW_THREADS, 0, holo_stream()>>>(dst, a, b, n);
    holo_check_launch("cuda_vec_mul");
}
void cuda_vec_scale(float *dst, const float *a, float scale, int n) {
    if (!args_ok(dst, n, "cuda_vec_scale") || n == 0) return;
    vec_scale_kernel<<<ew_grid(n), EW_THREADS, 0, holo_stream()>>>(dst, a, scale, n);
    holo_check_launch("cuda_vec_scale");
}
float cuda_vec_dot(const float *a, const float *b, int n) {
    if (!args_ok(a, n, "cuda_vec_dot") || n == 0) return 0.0f;
    HoloDevice *D = holo_dev();
    cudaStream_t st = holo_stream();
    float *part = (float *)D->reduce_buf;
    int g = min(256, (int)ew_grid(n));
    dot_partial_kernel<<<g, EW_THREADS, 0, st>>>(a, b, n, part);
    sum_parts_kernel<<<1, 1, 0, st>>>(part, g, part + 1024);
    float r = 0.0f;
    HOLO_CUDA_TRY(cudaMemcpyAsync(D->pinned, part + 1024, sizeof(float), cudaMemcpyDeviceToHost, st), "cuda_vec_dot");
    HOLO_CUDA_TRY(cudaStreamSynchronize(st), "cuda_vec_dot");
    r = *(float *)D->pinned;
    return r;
}

void cuda_silu(float *x, int n) {
    if (!args_ok(x, n, "cuda_silu") || n == 0) return;
    act_kernel<0><<<ew_grid(n), EW_THREADS, 0, holo_stream()>>>(x, n);
    holo_check_launch("cuda_silu");
}
void cuda_gelu(float *x, int n) {
    if (!args_ok(x, n, "cuda_gelu") || n == 0) return;
    act_kernel<1><<<ew_grid(n), EW_THREADS, 0, holo_stream()>>>(x, n);
    holo_check_launch("cuda_gelu");
}
void cuda_relu(float *x, int n) {
    if (!args_ok(x, n, "cuda_relu") || n == 0) return;
    act_kernel<2><<<ew_grid(n), EW_THREADS, 0, holo_stream()>>>(x, n);
    holo_check_launch("cuda_relu");
}
void cuda_silu_mul(float *dst, const float *a, const float *b, int n) {
    if (!args_ok(dst, n, "cuda_silu_mul") || n == 0) return;
    silu_mul_kernel<<<ew_grid(n), EW_THREADS, 0, holo_stream()>>>(dst, a, b, n);
    holo_check_launch("cuda_silu_mul");
}

void cuda_batched_ffn_gate_up_q8_0(float *out, const void *W1, const void *W3, const float *x, int ffn_dim,
                                   int in_dim) {
    if (!args_ok(out, ffn_dim, "cuda_batched_ffn_gate_up_q8_0") || ffn_dim == 0) return;
    float *up = (float *)holo_tmp((size_t)ffn_dim * sizeof(float));
    if (!up) return;
    WeightInfo a, b;
    if (holo_registry_find(W1, &a) && holo_registry_find(W3, &b) && a.type == GT_Q8_0 && b.type == GT_Q8_0 &&
        a.rows == ffn_dim && b.rows == ffn_dim && a.cols == in_dim && b.cols == in_dim && x) {
        // tiled weights: gate and up in one batched launch
        float *dst[2] = {out, up};
        const void *M[2] = {W1, W3};
        const float *v[2] = {x, x};
        cuda_matvec_batch(2, dst, M, v, holo_act_mode());
    } else {
        cuda_matvec(out, W1, x, ffn_dim, in_dim, GT_Q8_0, holo_act_mode(), nullptr);
        cuda_matvec(up, W3, x, ffn_dim, in_dim, GT_Q8_0, holo_act_mode(), nullptr);
    }
    silu_mul_kernel<<<ew_grid(ffn_dim), EW_THREADS, 0, holo_stream()>>>(out, out, up, ffn_dim);
    holo_check_launch("cuda_batched_ffn_gate_up_q8_0");
}

void cuda_rms_norm(float *dst, const float *x, const float *weight, int n, float eps) {
    if (!args_ok(dst, n, "cuda_rms_norm") || n == 0) return;
    rms_norm_kernel<<<1, 1024, 0, holo_stream()>>>(dst, x, weight, n, eps);
    holo_check_launch("cuda_rms_norm");
}
void cuda_layer_norm(float *dst, const float *x, const float *weight, const float *bias, int n, float eps) {
    (void)bias;   // the reference applies RMS normalisation here (src/ai/cuda_ops.cu:1506-1511)
    cuda_rms_norm(dst, x, weight, n, eps);
}

void cuda_softmax(float *dst, const float *x, int n) {
    if (!args_ok(dst, n, "cuda_softmax") || n == 0) return;
    softmax_kernel<<<1, 1024, 0, holo_stream()>>>(dst, x, n);
    holo_check_launch("cuda_softmax");
}
void cuda_softmax_inplace(float *x, int n) { cuda_softmax(x, x, n); }

void cuda_attention_scores(float *dst, const float *Q, const float *K, int seq_len, int kv_len, int head_dim,
                           float scale) {
    if (!args_ok(dst, seq_len, "cuda_attention_scores") || seq_len == 0 || kv_len <= 0) return;
    att_scores_kernel<<<dim3((kv_len + 127) / 128, seq_len), 128, 0, holo_stream()>>>(dst, Q, K, seq_len, kv_len,
                                                                                      head_dim, scale);
    holo_check_launch("cuda_attention_scores");
}
void cuda_attention_apply(float *dst, const float *scores, const float *V, int seq_len, int kv_len, int head_dim) {
    if (!args_ok(dst, seq_len, "cuda_attention_apply") || seq_len == 0 || head_dim <= 0) return;
    att_apply_kernel<<<dim3((head_dim + 127) / 128, seq_len), 128, 0, holo_stream()>>>(dst, scores, V, seq_len,
                                                                                       kv_len, head_dim);
    holo_check_launch("cuda_attention_apply");
}
void cuda_attention_single(float *dst, const float *q, const float *k_cache, const float *v_cache, float *att_buf,
                           int kv_len, int head_dim, int kv_head, int kv_dim) {
    (void)att_buf;   // unused by the reference GPU kernels as well
    if (!args_ok(dst, kv_len, "cuda_attention_single")) return;
    run_attention(dst, q, k_cache, v_cache, kv_len, head_dim, 1, kv_dim, kv_head, 1);
}
void cuda_multi_head_attention(float *dst, const float *q, const float *k_cache, const float *v_cache, int kv_len,
                               int head_dim, int n_heads, int n_kv_heads) {
    if (!args_ok(dst, kv_len, "cuda_multi_head_attention")) return;
    if (n_kv_heads <= 0 || n_heads % n_kv_heads) {
        holo_set_status(HOLO_E_ARG, "cuda_multi_head_attention: n_heads must be a multiple of n_kv_heads");
        return;
    }
    run_attention(dst, q, k_cache, v_cache, kv_len, head_dim, n_heads, n_kv_heads * head_dim, 0,
                  n_heads / n_kv_heads);
}

void cuda_rope_apply(float *q, float *k, int pos, int head_dim, int n_heads, int n_kv_heads, float freq_base) {
    if (!args_ok(q, head_dim, "cuda_rope_apply") || head_dim < 2 || head_dim > 2048) return;
    int heads = max(n_heads, n_kv_heads);
    if (heads <= 0) return;
    rope_kernel<<<heads, head_dim / 2, 0, holo_stream()>>>(q, k, pos, head_dim, n_heads, n_kv_heads, freq_base);
    holo_check_launch("cuda_rope_apply");
}

#define HOLO_EMB(NAME, TYPE, CHECK)                                                                      \
    void NAME(float *dst, const void *emb, int token, int dim, int vocab_size) {                         \
        if (!args_ok(dst, dim, #NAME) || dim == 0 || !emb || token < 0 || (vocab_size > 0 && token >= vocab_size) || \
            !(CHECK)) {                                                                                  \
            holo_set_status(HOLO_E_ARG, #NAME);                                                          \
            return;                                                                                      \
        }                                                                                                \
        embedding_kernel<TYPE><<<ew_grid(dim), EW_THREADS, 0, holo_stream()>>>(dst, (const uint8_t *)emb, token, dim); \
        holo_check_launch(#NAME);                                                                        \
    }
HOLO_EMB(cuda_get_embedding_f16, GT_F16, true)
HOLO_EMB(cuda_get_embedding_q8_0, GT_Q8_0, dim % 32 == 0)
HOLO_EMB(cuda_get_embedding_q4_0, GT_Q4_0, dim % 32 == 0)
HOLO_EMB(cuda_get_embedding_q6_k, GT_Q6_K, dim % 256 == 0)
void cuda_get_embedding_q4_k(float *dst, const void *emb, int token, int dim, int vocab_size) {
    if (!args_ok(dst, dim, "cuda_get_embedding_q4_k") || dim == 0 || !emb || token < 0 ||
        (vocab_size > 0 && token >= vocab_size) || dim % 256) {
        holo_set_status(HOLO_E_ARG, "cuda_get_embedding_q4_k");
        return;
    }
    q4k_embedding_kernel<<<ew_grid(dim), EW_THREADS, 0, holo_stream()>>>(dst, (const uint8_t *)emb, token, dim,
                                                                         holo_q4k_layout() == HOLO_Q4K_GGML);
    holo_check_launch("cuda_get_embedding_q4_k");
}
void cuda_get_embedding_f32(float *dst, const float *embeddings, int token, int dim, int vocab_size) {
    if (!args_ok(dst, dim, "cuda_get_embedding_f32") || !embeddings || token < 0 ||
        (vocab_size > 0 && token >= vocab_size)) {
        holo_set_status(HOLO_E_ARG, "cuda_get_embedding_f32");
        return;
    }
    embedding_kernel<GT_F32><<<ew_grid(dim), EW_THREADS, 0, holo_stream()>>>(dst, (const uint8_t *)embeddings,
                                                                            token, dim);
    holo_check_launch("cuda_get_embedding_f32");
}

int cuda_argmax(const float *x, int n) {
    if (!args_ok(x, n, "cuda_argmax") || n == 0) return 0;
    HoloDevice *D = holo_dev();
    cudaStream_t st = holo_stream();
    int parts = min(256, (int)ew_grid(n, 4));
    float *vals = (float *)D->reduce_buf;
    int *idxs = (int *)((char *)D->reduce_buf + 4096);
    int *res = (int *)((char *)D->reduce_buf + 8192);
    argmax_partial_kernel<<<parts, EW_THREADS, 0, st>>>(x, n, vals, idxs);
    argmax_final_kernel<<<1, 1, 0, st>>>(vals, idxs, parts, res);
    holo_check_launch("cuda_argmax");
    HOLO_CUDA_TRY(cudaMemcpyAsync(D->pinned, res, sizeof(int), cudaMemcpyDeviceToHost, st), "cuda_argmax");
    HOLO_CUDA_TRY(cudaStreamSynchronize(st), "cuda_argmax");
    return *(int *)D->pinned;
}

}  // extern "C"
