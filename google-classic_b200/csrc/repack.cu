// repack.cu -- one-time rewrite of raw GGUF blocks into the tiled layout
// (holo_common.cuh).  Takes over from upload_tensor (src/ai/llm_cuda.c:189-196),
// which copies the raw blocks as they are.
#include "holo_common.cuh"

#include <cstdio>

namespace {

// Q8_0: one thread per (row, 32-block); padding blocks stay zero.
__global__ void repack_q8_0_kernel(uint8_t *__restrict__ out, const uint8_t *__restrict__ in,
                                   int rows, int nblk, int units) {
    using G = UnitGeom<GT_Q8_0>;
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)rows * nblk) return;
    int r = (int)(gid / nblk), b = (int)(gid % nblk);
    const uint8_t *src = in + (size_t)r * nblk * G::BLK_BYTES + (size_t)b * G::BLK_BYTES;
    int lr = r % TILE_ROWS, s = b / G::BLKS32, bi = b % G::BLKS32;
    uint8_t *unit = out + ((size_t)(r / TILE_ROWS) * units + s) * G::UNIT_BYTES;
    uint8_t *q0 = unit + unit_plane_off<GT_Q8_0>(bi * 2, lr);
    uint8_t *q1 = unit + unit_plane_off<GT_Q8_0>(bi * 2 + 1, lr);
    for (int i = 0; i < 16; i++) { q0[i] = src[2 + i]; q1[i] = src[18 + i]; }
    uint8_t *dd = unit + unit_head_off<GT_Q8_0>(lr) + 2 * bi;
    dd[0] = src[0]; dd[1] = src[1];
}

__global__ void repack_q4_0_kernel(uint8_t *__restrict__ out, const uint8_t *__restrict__ in,
                                   int rows, int nblk, int units) {
    using G = UnitGeom<GT_Q4_0>;
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)rows * nblk) return;
    int r = (int)(gid / nblk), b = (int)(gid % nblk);
    const uint8_t *src = in + (size_t)r * nblk * G::BLK_BYTES + (size_t)b * G::BLK_BYTES;
    int lr = r % TILE_ROWS, s = b / G::BLKS32, bi = b % G::BLKS32;
    uint8_t *unit = out + ((size_t)(r / TILE_ROWS) * units + s) * G::UNIT_BYTES;
    uint8_t *q = unit + unit_plane_off<GT_Q4_0>(bi, lr);
    for (int i = 0; i < 16; i++) q[i] = src[2 + i];
    uint8_t *dd = unit + unit_head_off<GT_Q4_0>(lr) + 2 * bi;
    dd[0] = src[0]; dd[1] = src[1];
}

// Q4_K: one thread per (row, super-block); ggml-semantics blocks are rewritten
// into the quant.c semantics with identical dequantized values:
//   scales: get_scale_min_k4 (cuda_ops.cu:684-692) -> quant.c:290-297 packing
//   nibbles: 32 B per 64 values (cuda_ops.cu:712-729) -> 16 B per 32 values
__global__ void repack_q4_k_kernel(uint8_t *__restrict__ out, const uint8_t *__restrict__ in,
                                   int rows, int nsb, int ggml) {
    using G = UnitGeom<GT_Q4_K>;
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)rows * nsb) return;
    int r = (int)(gid / nsb), s = (int)(gid % nsb);
    const uint8_t *src = in + (size_t)r * nsb * G::BLK_BYTES + (size_t)s * G::BLK_BYTES;
    int lr = r % TILE_ROWS;
    uint8_t *unit = out + ((size_t)(r / TILE_ROWS) * nsb + s) * G::UNIT_BYTES;
    uint8_t *head = unit + unit_head_off<GT_Q4_K>(lr);
    if (!ggml) {
        for (int i = 0; i < 16; i++) head[i] = src[i];
        for (int j = 0; j < 8; j++)
            for (int l = 0; l < 16; l++) unit[unit_plane_off<GT_Q4_K>(j, lr) + l] = src[16 + j * 16 + l];
        return;
    }
    uint8_t sc[8], mn[8];
    const uint8_t *q = src + 4;
    for (int j = 0; j < 8; j++) {
        if (j < 4) { sc[j] = q[j] & 63; mn[j] = q[j + 4] & 63; }
        else {
            sc[j] = (uint8_t)((q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4));
            mn[j] = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
        }
    }
    for (int i = 0; i < 4; i++) head[i] = src[i];
    for (int j = 0; j < 4; j++) {
        head[4 + j] = (uint8_t)(sc[j] | ((sc[j + 4] & 3) << 6));
        head[8 + j] = (uint8_t)(mn[j] | ((mn[j + 4] & 3) << 6));
        head[12 + j] = (uint8_t)((sc[j + 4] >> 2) | ((mn[j + 4] >> 2) << 4));
    }
    // value v of sub-block j, position l (0..31): ggml group g = j/2 holds it in
    // byte qs[g*32 + l], low nibble for even j, high nibble for odd j.
    const uint8_t *qs = src + 16;
    for (int j = 0; j < 8; j++) {
        int g = j >> 1, hi = j & 1;
        for (int l = 0; l < 16; l++) {
            uint8_t a = qs[g * 32 + l], b = qs[g * 32 + l + 16];
            uint8_t na = hi ? (a >> 4) : (a & 0x0f);
            uint8_t nb = hi ? (b >> 4) : (b & 0x0f);
            unit[unit_plane_off<GT_Q4_K>(j, lr) + l] = (uint8_t)(na | (nb << 4));
        }
    }
}

// Q6_K: one thread per (row, 128-value half); the half's bytes move as they
// are (quant.c:251-268 reads them in this order)
__global__ void repack_q6_k_kernel(uint8_t *__restrict__ out, const uint8_t *__restrict__ in, int rows, int nsb) {
    using G = UnitGeom<GT_Q6_K>;
    const int units = 2 * nsb;
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)rows * units) return;
    int r = (int)(gid / units), hf = (int)(gid % units);
    const uint8_t *src = in + (size_t)r * nsb * G::BLK_BYTES + (size_t)(hf >> 1) * G::BLK_BYTES;
    const int n = hf & 1, lr = r % TILE_ROWS;
    uint8_t *unit = out + ((size_t)(r / TILE_ROWS) * units + hf) * G::UNIT_BYTES;
    uint8_t *head = unit + unit_head_off<GT_Q6_K>(lr);
    head[0] = src[208];
    head[1] = src[209];
    for (int k = 0; k < 8; k++) head[2 + k] = src[192 + n * 8 + k];
    for (int p = 0; p < 4; p++)
        for (int l = 0; l < 16; l++) unit[unit_plane_off<GT_Q6_K>(p, lr) + l] = src[n * 64 + p * 16 + l];
    for (int p = 0; p < 2; p++)
        for (int l = 0; l < 16; l++) unit[unit_plane_off<GT_Q6_K>(4 + p, lr) + l] = src[128 + n * 32 + p * 16 + l];
}

// F16: one thread per (row, 8 values)
__global__ void repack_f16_kernel(uint8_t *__restrict__ out, const uint8_t *__restrict__ in, int rows, int cols) {
    using G = UnitGeom<GT_F16>;
    const int chunks = cols / 8, units = cols / G::VALS;
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)rows * chunks) return;
    int r = (int)(gid / chunks), c = (int)(gid % chunks);
    const int lr = r % TILE_ROWS, s = c / UNIT_PLANES, p = c % UNIT_PLANES;
    const uint4 v = *reinterpret_cast<const uint4 *>(in + ((size_t)r * cols + (size_t)c * 8) * 2);
    uint8_t *unit = out + ((size_t)(r / TILE_ROWS) * units + s) * G::UNIT_BYTES;
    *reinterpret_cast<uint4 *>(unit + unit_plane_off<GT_F16>(p, lr)) = v;
}

}  // namespace

bool holo_quant_shape_ok(int type, int rows, int cols) {
    if (rows <= 0 || cols <= 0) return false;
    if (type == GT_Q4_K || type == GT_Q6_K) return cols % 256 == 0;
    if (type == GT_F16) return cols % UnitGeom<GT_F16>::VALS == 0;
    if (type == GT_Q8_0 || type == GT_Q4_0) return cols % 32 == 0;
    return false;
}

extern "C" size_t cuda_quant_tiled_bytes(int ggml_type, int rows, int cols) {
    if (!holo_quant_shape_ok(ggml_type, rows, cols)) return 0;
    size_t nrb = (size_t)(rows + TILE_ROWS - 1) / TILE_ROWS;
    return nrb * (size_t)units_per_row(ggml_type, cols) * (size_t)unit_bytes(ggml_type);
}

bool holo_repack_to(void *dst, const void *dev_blocks, int ggml_type, int rows, int cols, int q4k_layout,
                    cudaStream_t st) {
    if (!holo_quant_shape_ok(ggml_type, rows, cols) || !dev_blocks || !dst) {
        holo_set_status(HOLO_E_ARG, "repack: unsupported type or shape");
        return false;
    }
    const size_t bytes = cuda_quant_tiled_bytes(ggml_type, rows, cols);
    cudaMemsetAsync(dst, 0, bytes, st);   // padding rows and blocks are zero
    const int units = units_per_row(ggml_type, cols);
    const int threads = 256;
    if (ggml_type == GT_Q8_0) {
        int nblk = cols / 32;
        int64_t n = (int64_t)rows * nblk;
        repack_q8_0_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, st>>>(
            (uint8_t *)dst, (const uint8_t *)dev_blocks, rows, nblk, units);
    } else if (ggml_type == GT_Q4_0) {
        int nblk = cols / 32;
        int64_t n = (int64_t)rows * nblk;
        repack_q4_0_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, st>>>(
            (uint8_t *)dst, (const uint8_t *)dev_blocks, rows, nblk, units);
    } else if (ggml_type == GT_Q4_K) {
        int nsb = cols / 256;
        int64_t n = (int64_t)rows * nsb;
        repack_q4_k_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, st>>>(
            (uint8_t *)dst, (const uint8_t *)dev_blocks, rows, nsb, q4k_layout == HOLO_Q4K_GGML);
    } else if (ggml_type == GT_Q6_K) {
        int nsb = cols / 256;
        int64_t n = (int64_t)rows * nsb * 2;
        repack_q6_k_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, st>>>(
            (uint8_t *)dst, (const uint8_t *)dev_blocks, rows, nsb);
    } else {
        if ((uintptr_t)dev_blocks % 16) {
            holo_set_status(HOLO_E_ARG, "repack: F16 rows must start 16-byte aligned");
            return false;
        }
        int64_t n = (int64_t)rows * (cols / 8);
        repack_f16_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, st>>>(
            (uint8_t *)dst, (const uint8_t *)dev_blocks, rows, cols);
    }
    return holo_check_launch("repack kernel");
}

WeightInfo holo_weight_info(int ggml_type, int rows, int cols, int q4k_layout) {
    WeightInfo wi;
    wi.type = ggml_type;
    wi.rows = rows;
    wi.cols = cols;
    wi.rows_padded = (rows + TILE_ROWS - 1) / TILE_ROWS * TILE_ROWS;
    wi.units = units_per_row(ggml_type, cols);
    wi.q4k_layout = q4k_layout;
    wi.bytes = cuda_quant_tiled_bytes(ggml_type, rows, cols);
    return wi;
}

extern "C" void *cuda_repack_quant(const void *dev_blocks, int ggml_type, int rows, int cols) {
    if (!holo_quant_shape_ok(ggml_type, rows, cols) || !dev_blocks) {
        holo_set_status(HOLO_E_ARG, "cuda_repack_quant: unsupported type or shape");
        return nullptr;
    }
    HoloDevice *D = holo_dev();
    if (!D) return nullptr;
    cudaStream_t st = holo_stream();
    size_t bytes = cuda_quant_tiled_bytes(ggml_type, rows, cols);
    void *out = nullptr;
    if (cudaMalloc(&out, bytes) != cudaSuccess) {
        cudaGetLastError();
        holo_set_status(HOLO_E_NOMEM, "cuda_repack_quant: allocation");
        return nullptr;
    }
    const int layout = holo_q4k_layout();
    if (!holo_repack_to(out, dev_blocks, ggml_type, rows, cols, layout, st)) {
        cudaFree(out);
        return nullptr;
    }
    holo_registry_add(out, holo_weight_info(ggml_type, rows, cols, layout));
    return out;
}

extern "C" void *cuda_upload_quant(const void *host_blocks, int ggml_type, int rows, int cols) {
    if (!holo_quant_shape_ok(ggml_type, rows, cols) || !host_blocks) {
        holo_set_status(HOLO_E_ARG, "cuda_upload_quant: unsupported type or shape");
        return nullptr;
    }
    if (!holo_dev()) return nullptr;
    cudaStream_t st = holo_stream();
    size_t raw = (size_t)rows * (size_t)gguf_row_bytes(ggml_type, cols);
    void *staging = nullptr;
    if (cudaMalloc(&staging, raw) != cudaSuccess) {
        cudaGetLastError();
        holo_set_status(HOLO_E_NOMEM, "cuda_upload_quant: staging allocation");
        return nullptr;
    }
    HOLO_CUDA_TRY(cudaMemcpyAsync(staging, host_blocks, raw, cudaMemcpyHostToDevice, st), "cuda_upload_quant: copy");
    void *out = cuda_repack_quant(staging, ggml_type, rows, cols);
    cudaStreamSynchronize(st);
    cudaFree(staging);
    return out;
}
