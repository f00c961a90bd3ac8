// synth.cu -- seeded synthetic model weights generated on the device.
//
// Values are N(0, std) from a counter-based generator (splitmix64 of
// (seed, element index), Box-Muller), so any element can be regenerated
// independently; quantized blocks use round-to-nearest quantizers that follow
// the host ones in holo_b200/synth.py (the reference has no f32 -> Q8_0 /
// Q4_0 / Q4_K quantizer).  Output is raw GGUF blocks, row-major, the layout
// the reference loader reads, so the same bytes can feed both the reference
// and cuda_repack_quant.  Not part of any parity contract: the oracle and the
// GPU always consume identical bytes.
#include "holo_common.cuh"

namespace {

// splitmix64 (Steele, Lea, Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014)
__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// element i of the N(0, std) stream `seed` (Box-Muller on two 24-bit uniforms)
__device__ __forceinline__ float synth_normal(uint64_t seed, uint64_t i, float std) {
    const uint64_t h = splitmix64(seed * 0x100000001B3ull + i);
    const float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = ((float)(h & 0xFFFFFFull) + 0.5f) * (1.0f / 16777216.0f);
    return std * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__device__ __forceinline__ uint16_t f16_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }
__device__ __forceinline__ float f16_round(float v) { return __half2float(__float2half_rn(v)); }

__global__ void synth_f32_kernel(float *out, int64_t n, uint64_t seed, float std) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = synth_normal(seed, (uint64_t)i, std);
}
__global__ void synth_f16_kernel(__half *out, int64_t n, uint64_t seed, float std) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __float2half_rn(synth_normal(seed, (uint64_t)i, std));
}

// Q8_0: d = fp16(amax/127), q = clip(rint(v / d), -127, 127)
__global__ void synth_q8_0_kernel(uint8_t *out, int64_t nblk, uint64_t seed, float std) {
    const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    float v[32], amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 32; ++k) {
        v[k] = synth_normal(seed, (uint64_t)b * 32 + k, std);
        amax = fmaxf(amax, fabsf(v[k]));
    }
    const float d = f16_round(amax / 127.0f);
    const float inv = d > 0.0f ? 1.0f / d : 0.0f;
    uint8_t *o = out + b * 34;
    const uint16_t db = f16_bits(amax / 127.0f);
    o[0] = (uint8_t)(db & 0xff);
    o[1] = (uint8_t)(db >> 8);
#pragma unroll
    for (int k = 0; k < 32; ++k) o[2 + k] = (uint8_t)(int8_t)max(-127, min(127, __float2int_rn(v[k] * inv)));
}

// Q4_0: d = fp16(m / -8) with m the value of largest magnitude,
// q = clip(rint(v / d + 8), 0, 15)
__global__ void synth_q4_0_kernel(uint8_t *out, int64_t nblk, uint64_t seed, float std) {
    const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    float v[32], mx = 0.0f;
#pragma unroll
    for (int k = 0; k < 32; ++k) {
        v[k] = synth_normal(seed, (uint64_t)b * 32 + k, std);
        if (fabsf(v[k]) > fabsf(mx)) mx = v[k];
    }
    const float d = f16_round(mx / -8.0f);
    const float inv = d != 0.0f ? 1.0f / d : 0.0f;
    uint8_t *o = out + b * 18;
    const uint16_t db = f16_bits(mx / -8.0f);
    o[0] = (uint8_t)(db & 0xff);
    o[1] = (uint8_t)(db >> 8);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int q0 = max(0, min(15, __float2int_rn(v[k] * inv + 8.0f)));
        const int q1 = max(0, min(15, __float2int_rn(v[k + 16] * inv + 8.0f)));
        o[2 + k] = (uint8_t)(q0 | (q1 << 4));
    }
}

// Q4_K: per 32-value sub-block, scale = (hi - lo)/15 and min = -lo (lo <= 0);
// d = fp16(max scale / 63), dmin = fp16(max min / 63); 6-bit codes
// rint(scale/d), rint(min/dmin); q = clip(rint((v + dmin*m) / (d*sc)), 0, 15);
// scales packed as quant.c:290-297 reads them.  Values are regenerated per
// pass instead of being held (256 per thread).
__global__ void synth_q4_k_kernel(uint8_t *out, int64_t nsb, uint64_t seed, float std) {
    const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nsb) return;
    float scale[8], mins[8], smax = 0.0f, mmax = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float lo = 0.0f, hi = -INFINITY;
        for (int k = 0; k < 32; ++k) {
            const float v = synth_normal(seed, (uint64_t)b * 256 + j * 32 + k, std);
            lo = fminf(lo, v);
            hi = fmaxf(hi, v);
        }
        scale[j] = (hi - lo) / 15.0f;
        mins[j] = -lo;
        smax = fmaxf(smax, scale[j]);
        mmax = fmaxf(mmax, mins[j]);
    }
    const float d = f16_round(smax / 63.0f), dmin = f16_round(mmax / 63.0f);
    uint8_t sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = (uint8_t)max(0, min(63, __float2int_rn(scale[j] / (d > 0.0f ? d : 1.0f))));
        mn[j] = (uint8_t)max(0, min(63, __float2int_rn(mins[j] / (dmin > 0.0f ? dmin : 1.0f))));
    }
    uint8_t *o = out + b * 144;
    const uint16_t db = f16_bits(smax / 63.0f), dmb = f16_bits(mmax / 63.0f);
    o[0] = (uint8_t)(db & 0xff);
    o[1] = (uint8_t)(db >> 8);
    o[2] = (uint8_t)(dmb & 0xff);
    o[3] = (uint8_t)(dmb >> 8);
    for (int j = 0; j < 4; ++j) {
        o[4 + j] = (uint8_t)(sc[j] | ((sc[j + 4] & 3) << 6));
        o[8 + j] = (uint8_t)(mn[j] | ((mn[j + 4] & 3) << 6));
        o[12 + j] = (uint8_t)((sc[j + 4] >> 2) | ((mn[j + 4] >> 2) << 4));
    }
    for (int j = 0; j < 8; ++j) {
        const float es = d * (float)sc[j], em = dmin * (float)mn[j];
        const float inv = es > 0.0f ? 1.0f / es : 0.0f;
        for (int k = 0; k < 16; ++k) {
            const float v0 = synth_normal(seed, (uint64_t)b * 256 + j * 32 + k, std);
            const float v1 = synth_normal(seed, (uint64_t)b * 256 + j * 32 + k + 16, std);
            const int q0 = max(0, min(15, __float2int_rn((v0 + em) * inv)));
            const int q1 = max(0, min(15, __float2int_rn((v1 + em) * inv)));
            o[16 + j * 16 + k] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

}  // namespace

extern "C" int cuda_synth_weights(void *dst, int ggml_type, int rows, int cols, unsigned long long seed,
                                  float std) {
    if (!dst || rows <= 0 || cols <= 0) {
        holo_set_status(HOLO_E_ARG, "cuda_synth_weights: bad arguments");
        return HOLO_E_ARG;
    }
    if (!holo_dev()) return cuda_last_status();
    cudaStream_t st = holo_stream();
    const int64_t n = (int64_t)rows * cols;
    const int threads = 256;
    switch (ggml_type) {
    case GT_F32:
        synth_f32_kernel<<<4096, threads, 0, st>>>((float *)dst, n, seed, std);
        break;
    case GT_F16:
        synth_f16_kernel<<<4096, threads, 0, st>>>((__half *)dst, n, seed, std);
        break;
    case GT_Q8_0:
    case GT_Q4_0:
        if (cols % 32) {
            holo_set_status(HOLO_E_ARG, "cuda_synth_weights: cols % 32");
            return HOLO_E_ARG;
        }
        if (ggml_type == GT_Q8_0)
            synth_q8_0_kernel<<<(unsigned)((n / 32 + threads - 1) / threads), threads, 0, st>>>((uint8_t *)dst, n / 32,
                                                                                          seed, std);
        else
            synth_q4_0_kernel<<<(unsigned)((n / 32 + threads - 1) / threads), threads, 0, st>>>((uint8_t *)dst, n / 32,
                                                                                          seed, std);
        break;
    case GT_Q4_K:
        if (cols % 256) {
            holo_set_status(HOLO_E_ARG, "cuda_synth_weights: cols % 256");
            return HOLO_E_ARG;
        }
        synth_q4_k_kernel<<<(unsigned)((n / 256 + threads - 1) / threads), threads, 0, st>>>((uint8_t *)dst, n / 256,
                                                                                         seed, std);
        break;
    default:
        holo_set_status(HOLO_E_ARG, "cuda_synth_weights: unsupported type");
        return HOLO_E_ARG;
    }
    return holo_check_launch("cuda_synth_weights") ? HOLO_OK : cuda_last_status();
}
