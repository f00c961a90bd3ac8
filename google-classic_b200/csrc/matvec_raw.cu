// matvec_raw.cu -- matvecs over raw GGUF blocks, the parity probes, and the
// cuda_matmul_* entry points of the reference ABI (src/ai/cuda_ops.cu:784-845,
// 1132-1395).
//
// Raw pointers (weights uploaded with cuda_malloc + cuda_memcpy_h2d, as the
// reference's upload_tensor does, src/ai/llm_cuda.c:189-196) run a warp-per-row
// kernel that decodes the 34/18/144/210-byte blocks in place; pointers from
// cuda_upload_quant run the tiled kernels of matvec.cu.
#include "holo_common.cuh"
#include "mv_device.cuh"

#include <cstdio>

namespace {

constexpr int RAW_WARPS = 8;

__device__ __forceinline__ uint32_t ld_u16x2(const uint8_t *p) {   // 2-byte aligned
    const uint16_t *h = reinterpret_cast<const uint16_t *>(p);
    return (uint32_t)h[0] | ((uint32_t)h[1] << 16);
}
__device__ __forceinline__ uint4 ld16_a2(const uint8_t *p) {        // 16 bytes, 2-byte aligned
    return make_uint4(ld_u16x2(p), ld_u16x2(p + 4), ld_u16x2(p + 8), ld_u16x2(p + 12));
}

// canonical (quant.c) 16-byte nibble word of sub-block j from a ggml Q4_K block
__device__ __forceinline__ uint4 q4k_ggml_sub(const uint8_t *qs, int j) {
    const uint4 A = *reinterpret_cast<const uint4 *>(qs + (j >> 1) * 32);
    const uint4 B = *reinterpret_cast<const uint4 *>(qs + (j >> 1) * 32 + 16);
    if ((j & 1) == 0)
        return make_uint4((A.x & LO4) | ((B.x & LO4) << 4), (A.y & LO4) | ((B.y & LO4) << 4),
                          (A.z & LO4) | ((B.z & LO4) << 4), (A.w & LO4) | ((B.w & LO4) << 4));
    return make_uint4(((A.x >> 4) & LO4) | (B.x & 0xF0F0F0F0u), ((A.y >> 4) & LO4) | (B.y & 0xF0F0F0F0u),
                      ((A.z >> 4) & LO4) | (B.z & 0xF0F0F0F0u), ((A.w >> 4) & LO4) | (B.w & 0xF0F0F0F0u));
}
// header of a ggml Q4_K block re-expressed as the quant.c packing
__device__ __forceinline__ uint4 q4k_ggml_head(const uint8_t *blk) {
    uint8_t sc[8], mn[8];
    const uint8_t *q = blk + 4;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        if (j < 4) { sc[j] = q[j] & 63; mn[j] = q[j + 4] & 63; }
        else {
            sc[j] = (uint8_t)((q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4));
            mn[j] = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
        }
    }
    uint32_t w1 = 0, w2 = 0, w3 = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        w1 |= (uint32_t)(sc[j] | ((sc[j + 4] & 3) << 6)) << (8 * j);
        w2 |= (uint32_t)(mn[j] | ((mn[j + 4] & 3) << 6)) << (8 * j);
        w3 |= (uint32_t)((sc[j + 4] >> 2) | ((mn[j + 4] >> 2) << 4)) << (8 * j);
    }
    return make_uint4(*reinterpret_cast<const uint32_t *>(blk), w1, w2, w3);
}

// ---------------------------------------------------------------------------
// Block access for (row r, 32-block b) in either layout.
// ---------------------------------------------------------------------------
struct BlockRef {
    const uint8_t *W;
    bool tiled;
    int nblk32;            // 32-blocks per row
    int units;             // tiled: units per row
    size_t row_bytes;
    int ggml;              // raw Q4_K semantics
};

template <int TYPE>
__device__ __forceinline__ void load_block(const BlockRef &R, int r, int b, uint4 &q0, uint4 &q1, float &d,
                                           Q4KHead *kh) {
    if constexpr (TYPE == GT_Q8_0) {
        if (R.tiled) {
            const uint8_t *u = unit_ptr<GT_Q8_0>(R.W, R.units, r, b / 4);
            const int lr = r % TILE_ROWS, bi = b % 4;
            q0 = *reinterpret_cast<const uint4 *>(u + unit_plane_off<GT_Q8_0>(bi * 2, lr));
            q1 = *reinterpret_cast<const uint4 *>(u + unit_plane_off<GT_Q8_0>(bi * 2 + 1, lr));
            d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(u + unit_head_off<GT_Q8_0>(lr) + 2 * bi));
        } else {
            const uint8_t *blk = R.W + (size_t)r * R.row_bytes + (size_t)b * 34;
            d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
            q0 = ld16_a2(blk + 2);
            q1 = ld16_a2(blk + 18);
        }
    } else if constexpr (TYPE == GT_Q4_0) {
        if (R.tiled) {
            const uint8_t *u = unit_ptr<GT_Q4_0>(R.W, R.units, r, b / 8);
            const int lr = r % TILE_ROWS, bi = b % 8;
            q0 = *reinterpret_cast<const uint4 *>(u + unit_plane_off<GT_Q4_0>(bi, lr));
            d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(u + unit_head_off<GT_Q4_0>(lr) + 2 * bi));
        } else {
            const uint8_t *blk = R.W + (size_t)r * R.row_bytes + (size_t)b * 18;
            d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
            q0 = ld16_a2(blk + 2);
        }
    } else {  // Q4_K: b is the 32-block index, sub-block j = b % 8
        int s = b >> 3, j = b & 7;
        if (R.tiled) {
            const uint8_t *u = unit_ptr<GT_Q4_K>(R.W, R.units, r, s);
            const int lr = r % TILE_ROWS;
            *kh = q4k_head(*reinterpret_cast<const uint4 *>(u + unit_head_off<GT_Q4_K>(lr)));
            q0 = *reinterpret_cast<const uint4 *>(u + unit_plane_off<GT_Q4_K>(j, lr));
            d = 0.0f;
            return;
        }
        const uint8_t *blk = R.W + (size_t)r * R.row_bytes + (size_t)s * 144;
        if (R.ggml) {
            *kh = q4k_head(q4k_ggml_head(blk));
            q0 = q4k_ggml_sub(blk + 16, j);
        } else {
            *kh = q4k_head(*reinterpret_cast<const uint4 *>(blk));
            q0 = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * j);
        }
        d = 0.0f;
    }
}

// ---------------------------------------------------------------------------
// raw-layout matvec: warp per row, lanes over 32-blocks, CTA-shared Q8 act
// ---------------------------------------------------------------------------
template <int TYPE, int ACT>
__global__ void __launch_bounds__(RAW_WARPS * 32) mv_raw_kernel(BlockRef R, const float *__restrict__ x,
                                                                float *y, const float *residual, int out_dim) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int nblk = R.nblk32;
    uint8_t *aq = smem;
    float *ad = reinterpret_cast<float *>(smem + (size_t)nblk * 32);
    int *as = reinterpret_cast<int *>(ad + nblk);
    float *xs = reinterpret_cast<float *>(smem);
    if constexpr (ACT == HOLO_ACT_Q8) {
        for (int b = threadIdx.x; b < nblk; b += blockDim.x) {
            uint32_t w[8];
            float d;
            int s;
            quantize_block_q8(x + (size_t)b * 32, w, d, s);
            uint4 *dst = reinterpret_cast<uint4 *>(aq + (size_t)b * 32);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
            ad[b] = d;
            as[b] = s;
        }
    } else {
        for (int b = threadIdx.x; b < nblk; b += blockDim.x) {
            float s = 0.0f;
            for (int i = 0; i < 32; i++) s += x[(size_t)b * 32 + i];
            xs[b] = s;
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = blockIdx.x * RAW_WARPS + warp; r < out_dim; r += gridDim.x * RAW_WARPS) {
        float acc = 0.0f;
        for (int b = lane; b < nblk; b += 32) {
            uint4 q0, q1 = make_uint4(0, 0, 0, 0);
            float dw;
            Q4KHead kh;
            load_block<TYPE>(R, r, b, q0, q1, dw, &kh);
            if constexpr (ACT == HOLO_ACT_Q8) {
                uint4 a0 = *reinterpret_cast<const uint4 *>(aq + (size_t)b * 32);
                uint4 a1 = *reinterpret_cast<const uint4 *>(aq + (size_t)b * 32 + 16);
                if constexpr (TYPE == GT_Q8_0) {
                    acc += (dw * ad[b]) * int_to_float_exact(dot_i8x32_q8(q0, q1, a0, a1));
                } else if constexpr (TYPE == GT_Q4_0) {
                    acc += (dw * ad[b]) * int_to_float_exact(dot_nib16_q8(q0, a0, a1) - 8 * as[b]);
                } else {
                    int j = b & 7;
                    acc += ad[b] * ((kh.d * q4k_scale(kh, j)) * int_to_float_exact(dot_nib16_q8(q0, a0, a1)) -
                                    (kh.dmin * q4k_min(kh, j)) * int_to_float_exact(as[b]));
                }
            } else {
                const float *xb = x + (size_t)b * 32;
                if constexpr (TYPE == GT_Q8_0) {
                    acc += dw * dot_i8x32_f32(q0, q1, xb);
                } else if constexpr (TYPE == GT_Q4_0) {
                    acc += dw * (dot_nib16_f32(q0, xb) - 8.0f * xs[b]);
                } else {
                    int j = b & 7;
                    acc += (kh.d * q4k_scale(kh, j)) * dot_nib16_f32(q0, xb) - (kh.dmin * q4k_min(kh, j)) * xs[b];
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) y[r] = residual ? residual[r] + acc : acc;
    }
}

// Q6_K (src/ai/quant.c:241-271 value layout), F16 and F32 rows: warp per row.
__device__ __forceinline__ float q6k_dot(const uint8_t *blk, const float *__restrict__ xb, int lane) {
    // lane handles, for both 128-halves n, the l = lane column: 4 values each
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk + 208));
    float acc = 0.0f;
#pragma unroll
    for (int n = 0; n < 2; n++) {
        const uint8_t *ql = blk + n * 64, *qh = blk + 128 + n * 32;
        const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192) + n * 8;
        const float *yb = xb + n * 128;
        int l = lane, is = l / 16;
        int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
        int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
        int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
        int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
        acc += (d * (float)sc[is + 0]) * (float)q1 * yb[l];
        acc += (d * (float)sc[is + 2]) * (float)q2 * yb[l + 32];
        acc += (d * (float)sc[is + 4]) * (float)q3 * yb[l + 64];
        acc += (d * (float)sc[is + 6]) * (float)q4 * yb[l + 96];
    }
    return acc;
}

template <int TYPE>
__global__ void __launch_bounds__(RAW_WARPS * 32) mv_plain_kernel(const uint8_t *__restrict__ W,
                                                                  const float *__restrict__ x, float *y,
                                                                  int out_dim, int in_dim, size_t row_bytes) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = blockIdx.x * RAW_WARPS + warp; r < out_dim; r += gridDim.x * RAW_WARPS) {
        const uint8_t *row = W + (size_t)r * row_bytes;
        float acc = 0.0f;
        if constexpr (TYPE == GT_Q6_K) {
            for (int s = 0; s < in_dim / 256; s++) acc += q6k_dot(row + (size_t)s * 210, x + (size_t)s * 256, lane);
        } else if constexpr (TYPE == GT_F16) {
            const __half *h = reinterpret_cast<const __half *>(row);
            for (int i = lane; i < in_dim; i += 32) acc = fmaf(__half2float(h[i]), x[i], acc);
        } else {
            const float *f = reinterpret_cast<const float *>(row);
            for (int i = lane; i < in_dim; i += 32) acc = fmaf(f[i], x[i], acc);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) y[r] = acc;
    }
}

// ---------------------------------------------------------------------------
// parity probes
// ---------------------------------------------------------------------------
// dequantized values, one thread per (row, 32-block); each value rounded as in
// src/ai/quant.c:125 (Q8_0), 149-150 (Q4_0), 301-307 (Q4_K).
template <int TYPE>
__global__ void dequant_kernel(BlockRef R, float *dst, int rows) {
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)rows * R.nblk32) return;
    int r = (int)(gid / R.nblk32), b = (int)(gid % R.nblk32);
    uint4 q0, q1 = make_uint4(0, 0, 0, 0);
    float d;
    Q4KHead kh;
    load_block<TYPE>(R, r, b, q0, q1, d, &kh);
    float *o = dst + (size_t)r * R.nblk32 * 32 + (size_t)b * 32;
    if constexpr (TYPE == GT_Q8_0) {
        uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        for (int i = 0; i < 32; i++) o[i] = __fmul_rn(d, (float)(int8_t)((w[i / 4] >> (8 * (i % 4))) & 0xff));
    } else {
        uint32_t w[4] = {q0.x, q0.y, q0.z, q0.w};
        float sc = 0.0f, mn = 0.0f;
        if constexpr (TYPE == GT_Q4_K) {
            int j = b & 7;
            sc = __fmul_rn(kh.d, q4k_scale(kh, j));
            mn = __fmul_rn(kh.dmin, q4k_min(kh, j));
        }
        for (int l = 0; l < 16; l++) {
            int lo = (w[l / 4] >> (8 * (l % 4))) & 0xf, hi = (w[l / 4] >> (8 * (l % 4) + 4)) & 0xf;
            if constexpr (TYPE == GT_Q4_0) {
                o[l] = __fmul_rn(d, (float)(lo - 8));
                o[l + 16] = __fmul_rn(d, (float)(hi - 8));
            } else {
                o[l] = __fsub_rn(__fmul_rn(sc, (float)lo), mn);
                o[l + 16] = __fsub_rn(__fmul_rn(sc, (float)hi), mn);
            }
        }
    }
}

__global__ void quantize_act_kernel(const float *__restrict__ x, int nblk, int8_t *q, float *d, int32_t *asum) {
    int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    uint32_t w[8];
    float db;
    int s;
    quantize_block_q8(x + (size_t)b * 32, w, db, s);
    uint4 *dst = reinterpret_cast<uint4 *>(q + (size_t)b * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    d[b] = db;
    asum[b] = s;
}

template <int TYPE>
__global__ void block_sums_kernel(BlockRef R, const int8_t *__restrict__ aq, const int32_t *__restrict__ as,
                                  int32_t *dst, int rows) {
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)rows * R.nblk32) return;
    int r = (int)(gid / R.nblk32), b = (int)(gid % R.nblk32);
    uint4 q0, q1 = make_uint4(0, 0, 0, 0);
    float d;
    Q4KHead kh;
    load_block<TYPE>(R, r, b, q0, q1, d, &kh);
    uint4 a0 = *reinterpret_cast<const uint4 *>(aq + (size_t)b * 32);
    uint4 a1 = *reinterpret_cast<const uint4 *>(aq + (size_t)b * 32 + 16);
    int s;
    if constexpr (TYPE == GT_Q8_0) s = dot_i8x32_q8(q0, q1, a0, a1);
    else if constexpr (TYPE == GT_Q4_0) s = dot_nib16_q8(q0, a0, a1) - 8 * as[b];
    else s = dot_nib16_q8(q0, a0, a1);
    dst[gid] = s;
}

bool quant_shape_ok(int type, int rows, int cols) {
    if (rows <= 0 || cols <= 0) return false;
    int be = gguf_block_elems(type);
    return cols % be == 0;
}

BlockRef make_ref(const void *M, int type, int cols, bool tiled, int ggml) {
    BlockRef R;
    R.W = (const uint8_t *)M;
    R.tiled = tiled;
    R.nblk32 = cols / 32;
    R.row_bytes = (size_t)gguf_row_bytes(type, cols);
    R.units = units_per_row(type, cols);
    R.ggml = ggml;
    return R;
}

template <int TYPE, int ACT>
void launch_raw(const BlockRef &R, const float *v, float *dst, const float *residual, int out_dim, cudaStream_t st) {
    HoloDevice *D = holo_dev();
    size_t smem = ACT == HOLO_ACT_Q8 ? (size_t)R.nblk32 * 40 : (size_t)R.nblk32 * 4;
    auto kern = mv_raw_kernel<TYPE, ACT>;
    if (smem > 48 * 1024) {
        if (smem > 227 * 1024) { holo_set_status(HOLO_E_UNSUPPORTED, "raw matvec: in_dim too large"); return; }
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    }
    int rows_per_cta = RAW_WARPS * 4;
    int grid = min((out_dim + rows_per_cta - 1) / rows_per_cta, D->sms * 4);
    kern<<<max(grid, 1), RAW_WARPS * 32, smem, st>>>(R, v, dst, residual, out_dim);
    holo_check_launch("raw matvec launch");
}

}  // namespace

void holo_matvec_raw(float *dst, const void *M, int type, const float *v, int out_dim, int in_dim,
                     int act_mode, int q4k_layout, cudaStream_t st, const float *residual) {
    HoloDevice *D = holo_dev();
    if (!D) return;
    BlockRef R = make_ref(M, type, in_dim, false, q4k_layout == HOLO_Q4K_GGML);
    const bool q8 = act_mode == HOLO_ACT_Q8;
    switch (type) {
    case GT_Q8_0: q8 ? launch_raw<GT_Q8_0, HOLO_ACT_Q8>(R, v, dst, residual, out_dim, st)
                     : launch_raw<GT_Q8_0, HOLO_ACT_F32>(R, v, dst, residual, out_dim, st); break;
    case GT_Q4_0: q8 ? launch_raw<GT_Q4_0, HOLO_ACT_Q8>(R, v, dst, residual, out_dim, st)
                     : launch_raw<GT_Q4_0, HOLO_ACT_F32>(R, v, dst, residual, out_dim, st); break;
    case GT_Q4_K: q8 ? launch_raw<GT_Q4_K, HOLO_ACT_Q8>(R, v, dst, residual, out_dim, st)
                     : launch_raw<GT_Q4_K, HOLO_ACT_F32>(R, v, dst, residual, out_dim, st); break;
    default: holo_set_status(HOLO_E_ARG, "raw matvec: type");
    }
}

namespace {

void matvec_any(float *dst, const void *M, const float *v, int out_dim, int in_dim, int type, int act,
                const float *residual) {
    if (!dst || !M || !v || !quant_shape_ok(type, out_dim, in_dim)) {
        holo_set_status(HOLO_E_ARG, "matvec: bad arguments");
        return;
    }
    HoloDevice *D = holo_dev();
    if (!D) return;
    cudaStream_t st = holo_stream();
    WeightInfo wi;
    if (holo_registry_find(M, &wi)) {
        if (wi.type != type) { holo_set_status(HOLO_E_ARG, "matvec: type differs from the uploaded weight"); return; }
        holo_matvec_tiled(dst, M, wi, v, out_dim, in_dim, act, residual, st);
        return;
    }
    if (type == GT_Q8_0 || type == GT_Q4_0 || type == GT_Q4_K) {
        holo_matvec_raw(dst, M, type, v, out_dim, in_dim, act, holo_q4k_layout(), st, residual);
        return;
    }
    size_t rb = (size_t)gguf_row_bytes(type, in_dim);
    int grid = min((out_dim + RAW_WARPS - 1) / RAW_WARPS, D->sms * 8);
    if (type == GT_Q6_K) mv_plain_kernel<GT_Q6_K><<<grid, RAW_WARPS * 32, 0, st>>>((const uint8_t *)M, v, dst, out_dim, in_dim, rb);
    else if (type == GT_F16) mv_plain_kernel<GT_F16><<<grid, RAW_WARPS * 32, 0, st>>>((const uint8_t *)M, v, dst, out_dim, in_dim, rb);
    else mv_plain_kernel<GT_F32><<<grid, RAW_WARPS * 32, 0, st>>>((const uint8_t *)M, v, dst, out_dim, in_dim, rb);
    holo_check_launch("plain matvec launch");
    if (residual) holo_set_status(HOLO_E_UNSUPPORTED, "matvec: residual needs a quantized type");
}

}  // namespace

extern "C" {

void cuda_matvec(float *dst, const void *M, const float *v, int out_dim, int in_dim, int ggml_type,
                 int act_mode, const float *residual) {
    matvec_any(dst, M, v, out_dim, in_dim, ggml_type, act_mode == HOLO_ACT_F32 ? HOLO_ACT_F32 : HOLO_ACT_Q8, residual);
}

void cuda_matmul_f32(float *dst, const float *M, const float *v, int out_dim, int in_dim) {
    matvec_any(dst, M, v, out_dim, in_dim, GT_F32, HOLO_ACT_F32, nullptr);
}
void cuda_matmul_f16(float *dst, const void *M, const float *v, int out_dim, int in_dim) {
    matvec_any(dst, M, v, out_dim, in_dim, GT_F16, HOLO_ACT_F32, nullptr);
}
void cuda_matmul_q8_0(float *dst, const void *M, const float *v, int out_dim, int in_dim) {
    matvec_any(dst, M, v, out_dim, in_dim, GT_Q8_0, holo_act_mode(), nullptr);
}
void cuda_matmul_q4_0(float *dst, const void *M, const float *v, int out_dim, int in_dim) {
    matvec_any(dst, M, v, out_dim, in_dim, GT_Q4_0, holo_act_mode(), nullptr);
}
void cuda_matmul_q4_k(float *dst, const void *M, const float *v, int out_dim, int in_dim) {
    matvec_any(dst, M, v, out_dim, in_dim, GT_Q4_K, holo_act_mode(), nullptr);
}
void cuda_matmul_q6_k(float *dst, const void *M, const float *v, int out_dim, int in_dim) {
    matvec_any(dst, M, v, out_dim, in_dim, GT_Q6_K, HOLO_ACT_F32, nullptr);
}

void cuda_batched_qkv_q8_0(float *q_out, float *k_out, float *v_out, const void *Wq, const void *Wk,
                           const void *Wv, const float *x, int q_dim, int kv_dim, int in_dim) {
    int act = holo_act_mode();
    WeightInfo a, b, c;
    // tiled weights of the expected shapes: the three matvecs in one batched launch
    if (holo_registry_find(Wq, &a) && holo_registry_find(Wk, &b) && holo_registry_find(Wv, &c) &&
        a.type == GT_Q8_0 && b.type == GT_Q8_0 && c.type == GT_Q8_0 && a.rows == q_dim && b.rows == kv_dim &&
        c.rows == kv_dim && a.cols == in_dim && b.cols == in_dim && c.cols == in_dim && x) {
        float *dst[3] = {q_out, k_out, v_out};
        const void *M[3] = {Wq, Wk, Wv};
        const float *v[3] = {x, x, x};
        cuda_matvec_batch(3, dst, M, v, act);
        return;
    }
    matvec_any(q_out, Wq, x, q_dim, in_dim, GT_Q8_0, act, nullptr);
    matvec_any(k_out, Wk, x, kv_dim, in_dim, GT_Q8_0, act, nullptr);
    matvec_any(v_out, Wv, x, kv_dim, in_dim, GT_Q8_0, act, nullptr);
}

void cuda_dequantize_rows(float *dst, const void *M, int ggml_type, int rows, int cols) {
    if (!dst || !M || !quant_shape_ok(ggml_type, rows, cols) ||
        !(ggml_type == GT_Q8_0 || ggml_type == GT_Q4_0 || ggml_type == GT_Q4_K)) {
        holo_set_status(HOLO_E_ARG, "cuda_dequantize_rows: bad arguments");
        return;
    }
    if (!holo_dev()) return;
    WeightInfo wi;
    bool tiled = holo_registry_find(M, &wi);
    if (tiled && (wi.type != ggml_type || wi.rows != rows || wi.cols != cols)) {
        holo_set_status(HOLO_E_ARG, "cuda_dequantize_rows: shape differs from the uploaded weight");
        return;
    }
    BlockRef R = make_ref(M, ggml_type, cols, tiled, holo_q4k_layout() == HOLO_Q4K_GGML);
    int64_t n = (int64_t)rows * R.nblk32;
    unsigned grid = (unsigned)((n + 255) / 256);
    cudaStream_t st = holo_stream();
    if (ggml_type == GT_Q8_0) dequant_kernel<GT_Q8_0><<<grid, 256, 0, st>>>(R, dst, rows);
    else if (ggml_type == GT_Q4_0) dequant_kernel<GT_Q4_0><<<grid, 256, 0, st>>>(R, dst, rows);
    else dequant_kernel<GT_Q4_K><<<grid, 256, 0, st>>>(R, dst, rows);
    holo_check_launch("dequantize launch");
}

void cuda_quantize_act_q8(int8_t *q, float *d, int32_t *asum, const float *x, int n) {
    if (!q || !d || !asum || !x || n <= 0 || n % 32) {
        holo_set_status(HOLO_E_ARG, "cuda_quantize_act_q8: bad arguments");
        return;
    }
    if (!holo_dev()) return;
    int nblk = n / 32;
    quantize_act_kernel<<<(nblk + 127) / 128, 128, 0, holo_stream()>>>(x, nblk, q, d, asum);
    holo_check_launch("quantize launch");
}

void cuda_block_sums_q8(int32_t *dst, const void *M, const float *v, int ggml_type, int rows, int cols) {
    if (!dst || !M || !v || !quant_shape_ok(ggml_type, rows, cols) ||
        !(ggml_type == GT_Q8_0 || ggml_type == GT_Q4_0 || ggml_type == GT_Q4_K)) {
        holo_set_status(HOLO_E_ARG, "cuda_block_sums_q8: bad arguments");
        return;
    }
    if (!holo_dev()) return;
    WeightInfo wi;
    bool tiled = holo_registry_find(M, &wi);
    if (tiled && (wi.type != ggml_type || wi.rows != rows || wi.cols != cols)) {
        holo_set_status(HOLO_E_ARG, "cuda_block_sums_q8: shape differs from the uploaded weight");
        return;
    }
    cudaStream_t st = holo_stream();
    int nblk = cols / 32;
    // probe-only temporaries (not on any timed path)
    int8_t *aq = nullptr;
    float *ad = nullptr;
    int32_t *as = nullptr;
    if (cudaMalloc(&aq, (size_t)cols) != cudaSuccess || cudaMalloc(&ad, (size_t)nblk * 4) != cudaSuccess ||
        cudaMalloc(&as, (size_t)nblk * 4) != cudaSuccess) {
        holo_set_status(HOLO_E_NOMEM, "cuda_block_sums_q8: allocation");
        cudaFree(aq); cudaFree(ad); cudaFree(as);
        return;
    }
    quantize_act_kernel<<<(nblk + 127) / 128, 128, 0, st>>>(v, nblk, aq, ad, as);
    BlockRef R = make_ref(M, ggml_type, cols, tiled, holo_q4k_layout() == HOLO_Q4K_GGML);
    int64_t n = (int64_t)rows * nblk;
    unsigned grid = (unsigned)((n + 255) / 256);
    if (ggml_type == GT_Q8_0) block_sums_kernel<GT_Q8_0><<<grid, 256, 0, st>>>(R, aq, as, dst, rows);
    else if (ggml_type == GT_Q4_0) block_sums_kernel<GT_Q4_0><<<grid, 256, 0, st>>>(R, aq, as, dst, rows);
    else block_sums_kernel<GT_Q4_K><<<grid, 256, 0, st>>>(R, aq, as, dst, rows);
    holo_check_launch("block sums launch");
    cudaStreamSynchronize(st);
    cudaFree(aq); cudaFree(ad); cudaFree(as);
}

}  // extern "C"
