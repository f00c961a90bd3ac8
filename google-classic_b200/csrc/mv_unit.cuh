// mv_unit.cuh -- device building blocks of the unit-layout matvec, shared by
// the standalone kernel (matvec.cu) and the persistent decode step (step.cu):
// streaming loads, L2 prefetch and bulk copies, the per-warp unit fragment and
// its dot product with the activation in shared memory.
#pragma once
#include "holo_common.cuh"
#include "mv_device.cuh"

namespace holo_mv {

// L2 prefetch of a byte range (no data returns to the SM)
__device__ __forceinline__ void prefetch_l2_bulk(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(src), "r"(bytes) : "memory");
}

// 1-D bulk copy global -> shared (no multicast, no cache hint)
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}

// streaming loads: read once, not kept in L1
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ldg_stream2(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// What one warp loads for one unit (lane = row): eight 16-byte code planes and
// the row's head (Q4_K head / Q4_0 eight fp16 scales / Q8_0 four).
struct Frag {
    uint4 q[UNIT_PLANES];
    uint4 h;
};

template <int TYPE>
__device__ __forceinline__ void load_unit(Frag &f, const uint8_t *__restrict__ unit, int lane) {
    const uint8_t *row = unit + (size_t)TILE_ROWS * UnitGeom<TYPE>::HEAD_BYTES + lane * 16;
    constexpr int NPL = TYPE == GT_Q6_K ? UnitGeom<GT_Q6_K>::PLANES : UNIT_PLANES;
#pragma unroll
    for (int pl = 0; pl < NPL; ++pl) f.q[pl] = ldg_stream(row + pl * TILE_ROWS * 16);
    if constexpr (TYPE == GT_F16) {
        f.h = make_uint4(0u, 0u, 0u, 0u);
    } else if constexpr (TYPE == GT_Q8_0) {
        const uint2 h = ldg_stream2(unit + lane * 8);
        f.h = make_uint4(h.x, h.y, 0u, 0u);
    } else {
        f.h = ldg_stream(unit + lane * 16);
    }
}

// the same fragment from a unit staged in shared memory (16-byte rows: the
// 32 lanes of a plane read 512 contiguous bytes, no bank conflicts)
template <int TYPE>
__device__ __forceinline__ void load_unit_smem(Frag &f, const uint8_t *unit, int lane) {
    const uint8_t *row = unit + (size_t)TILE_ROWS * UnitGeom<TYPE>::HEAD_BYTES + lane * 16;
    constexpr int NPL = TYPE == GT_Q6_K ? UnitGeom<GT_Q6_K>::PLANES : UNIT_PLANES;
#pragma unroll
    for (int pl = 0; pl < NPL; ++pl) f.q[pl] = lds128(row + pl * TILE_ROWS * 16);
    if constexpr (TYPE == GT_F16) {
        f.h = make_uint4(0u, 0u, 0u, 0u);
    } else if constexpr (TYPE == GT_Q8_0) {
        const uint2 h = *reinterpret_cast<const uint2 *>(unit + lane * 8);
        f.h = make_uint4(h.x, h.y, 0u, 0u);
    } else {
        f.h = lds128(unit + lane * 16);
    }
}

// order this thread's (and, after a warp or CTA barrier, its peers') generic
// shared-memory accesses before later async-proxy (bulk copy) writes
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// signed byte k (0..15) of a head word set, as an exact float
__device__ __forceinline__ float sbyte_to_float_s(const uint4 &h, int k) {
    const uint32_t w = k < 4 ? h.x : k < 8 ? h.y : k < 12 ? h.z : h.w;
    return (float)(int8_t)(uint8_t)(w >> (8 * (k & 3)));
}

// fp16 scale k (0..7) of a head word set
__device__ __forceinline__ float head_half(const uint4 &h, int k) {
    const uint32_t w = k < 2 ? h.x : k < 4 ? h.y : k < 6 ? h.z : h.w;
    return half_bits_to_float((k & 1) ? (w >> 16) : (w & 0xffffu));
}

// this lane's (row's) contribution of one unit, added into acc; b0 = index of
// the unit's first 32-block in the activation vector
template <int TYPE, int ACT>
__device__ __forceinline__ void unit_dot(float &acc, const Frag &f, int b0, const uint8_t *__restrict__ aq,
                                         const float2 *__restrict__ ads, const float *__restrict__ xs,
                                         const float *__restrict__ xsum) {
    if constexpr (TYPE == GT_Q4_K) {
        const uint4 h = f.h;
        // d/16 is exact, so (d/16)*sc rounds like (d*sc)/16
        const float d = half_bits_to_float(h.x & 0xffffu) * (ACT == HOLO_ACT_Q8 ? 0.0625f : 1.0f);
        const float dmin = half_bits_to_float(h.x >> 16);
        const uint32_t sc_lo = h.y & 0x3F3F3F3Fu, m_lo = h.z & 0x3F3F3F3Fu;
        const uint32_t sc_hi = ((h.w & LO4) << 2) | ((h.y >> 6) & 0x03030303u);
        const uint32_t m_hi = (((h.w >> 4) & LO4) << 2) | ((h.z >> 6) & 0x03030303u);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float sc = d * ubyte_to_float(j < 4 ? sc_lo : sc_hi, j & 3);
            const float mn = dmin * ubyte_to_float(j < 4 ? m_lo : m_hi, j & 3);
            const int blk = b0 + j;
            if constexpr (ACT == HOLO_ACT_Q8) {
                const uint4 a0 = lds128(aq + (size_t)blk * 32), a1 = lds128(aq + (size_t)blk * 32 + 16);
                const float2 ds = ads[blk];
                const float f16 = int_to_float_exact(dot_nib16_q8_x16(f.q[j], a0, a1));
                acc += fmaf(sc, ds.x * f16, -mn * ds.y);
            } else {
                acc += fmaf(sc, dot_nib16_f32<true>(f.q[j], xs + (size_t)blk * 32), -mn * xsum[blk]);
            }
        }
    } else if constexpr (TYPE == GT_Q6_K) {
        // 32-block j of the half: values l = 0..15 from planes (j&1 ? 2 : 0)
        // and 4, l = 16..31 from planes (j&1 ? 3 : 1) and 5; low nibbles for
        // j < 2, high for j >= 2; high bits 2j..2j+1 of the qh byte; codes
        // u = nib | qh2 << 4 (0..63), value d * sc * (u - 32) with scale
        // 2j for l < 16 and 2j+1 above (quant.c:255-264)
        const float d = half_bits_to_float(f.h.x & 0xffffu);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int nsh = (j & 2) ? 4 : 0, hsh = 2 * j;
            const uint4 l0 = f.q[(j & 1) ? 2 : 0], l1 = f.q[(j & 1) ? 3 : 1], h0 = f.q[4], h1 = f.q[5];
            uint32_t u[8];
            u[0] = ((l0.x >> nsh) & LO4) | (((h0.x >> hsh) & 0x03030303u) << 4);
            u[1] = ((l0.y >> nsh) & LO4) | (((h0.y >> hsh) & 0x03030303u) << 4);
            u[2] = ((l0.z >> nsh) & LO4) | (((h0.z >> hsh) & 0x03030303u) << 4);
            u[3] = ((l0.w >> nsh) & LO4) | (((h0.w >> hsh) & 0x03030303u) << 4);
            u[4] = ((l1.x >> nsh) & LO4) | (((h1.x >> hsh) & 0x03030303u) << 4);
            u[5] = ((l1.y >> nsh) & LO4) | (((h1.y >> hsh) & 0x03030303u) << 4);
            u[6] = ((l1.z >> nsh) & LO4) | (((h1.z >> hsh) & 0x03030303u) << 4);
            u[7] = ((l1.w >> nsh) & LO4) | (((h1.w >> hsh) & 0x03030303u) << 4);
            const float w0 = d * sbyte_to_float_s(f.h, 2 + 2 * j), w1 = d * sbyte_to_float_s(f.h, 3 + 2 * j);
            const int blk = b0 + j;
            if constexpr (ACT == HOLO_ACT_Q8) {
                const uint4 a0 = lds128(aq + (size_t)blk * 32), a1 = lds128(aq + (size_t)blk * 32 + 16);
                int s0 = 0, s1 = 0, t0 = 0, t1 = 0;
                s0 = dp4a_us(u[0], a0.x, s0); s0 = dp4a_us(u[1], a0.y, s0);
                s0 = dp4a_us(u[2], a0.z, s0); s0 = dp4a_us(u[3], a0.w, s0);
                s1 = dp4a_us(u[4], a1.x, s1); s1 = dp4a_us(u[5], a1.y, s1);
                s1 = dp4a_us(u[6], a1.z, s1); s1 = dp4a_us(u[7], a1.w, s1);
                t0 = __dp4a((int)a0.x, 0x01010101, t0); t0 = __dp4a((int)a0.y, 0x01010101, t0);
                t0 = __dp4a((int)a0.z, 0x01010101, t0); t0 = __dp4a((int)a0.w, 0x01010101, t0);
                t1 = __dp4a((int)a1.x, 0x01010101, t1); t1 = __dp4a((int)a1.y, 0x01010101, t1);
                t1 = __dp4a((int)a1.z, 0x01010101, t1); t1 = __dp4a((int)a1.w, 0x01010101, t1);
                // sum (u-32)*q over each 16: exact integers (|.| < 2^15)
                const float i0 = int_to_float_exact(s0 - 32 * t0), i1 = int_to_float_exact(s1 - 32 * t1);
                acc += ads[blk].x * fmaf(w0, i0, w1 * i1);
            } else {
                const float *xb = xs + (size_t)blk * 32;
                float f0 = 0.0f, f1 = 0.0f;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float4 x0 = *reinterpret_cast<const float4 *>(xb + 4 * k);
                    const float4 x1 = *reinterpret_cast<const float4 *>(xb + 16 + 4 * k);
                    f0 = fmaf(ubyte_to_float(u[k], 0) - 32.0f, x0.x, f0);
                    f0 = fmaf(ubyte_to_float(u[k], 1) - 32.0f, x0.y, f0);
                    f0 = fmaf(ubyte_to_float(u[k], 2) - 32.0f, x0.z, f0);
                    f0 = fmaf(ubyte_to_float(u[k], 3) - 32.0f, x0.w, f0);
                    f1 = fmaf(ubyte_to_float(u[4 + k], 0) - 32.0f, x1.x, f1);
                    f1 = fmaf(ubyte_to_float(u[4 + k], 1) - 32.0f, x1.y, f1);
                    f1 = fmaf(ubyte_to_float(u[4 + k], 2) - 32.0f, x1.z, f1);
                    f1 = fmaf(ubyte_to_float(u[4 + k], 3) - 32.0f, x1.w, f1);
                }
                acc += fmaf(w0, f0, w1 * f1);
            }
        }
    } else if constexpr (TYPE == GT_F16) {
        // fp32 activation in both modes (x as staged, before any quantization)
#pragma unroll
        for (int pl = 0; pl < UNIT_PLANES; ++pl) {
            const float *xb = xs + (size_t)b0 * 32 + 8 * pl;
            const float4 x0 = *reinterpret_cast<const float4 *>(xb), x1 = *reinterpret_cast<const float4 *>(xb + 4);
            const uint4 q = f.q[pl];
            const float2 w0 = __half22float2(*reinterpret_cast<const __half2 *>(&q.x));
            const float2 w1 = __half22float2(*reinterpret_cast<const __half2 *>(&q.y));
            const float2 w2 = __half22float2(*reinterpret_cast<const __half2 *>(&q.z));
            const float2 w3 = __half22float2(*reinterpret_cast<const __half2 *>(&q.w));
            float t = w0.x * x0.x;
            t = fmaf(w0.y, x0.y, t); t = fmaf(w1.x, x0.z, t); t = fmaf(w1.y, x0.w, t);
            t = fmaf(w2.x, x1.x, t); t = fmaf(w2.y, x1.y, t); t = fmaf(w3.x, x1.z, t); t = fmaf(w3.y, x1.w, t);
            acc += t;
        }
    } else if constexpr (TYPE == GT_Q4_0) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float dw = head_half(f.h, j);
            const int blk = b0 + j;
            if constexpr (ACT == HOLO_ACT_Q8) {
                const uint4 a0 = lds128(aq + (size_t)blk * 32), a1 = lds128(aq + (size_t)blk * 32 + 16);
                const float2 ds = ads[blk];
                const float f16 = int_to_float_exact(dot_nib16_q8_x16(f.q[j], a0, a1));
                acc += dw * fmaf(ds.x * 0.0625f, f16, -8.0f * ds.y);
            } else {
                acc += dw * (dot_nib16_f32<true>(f.q[j], xs + (size_t)blk * 32) - 8.0f * xsum[blk]);
            }
        }
    } else {  // Q8_0: block j = planes 2j, 2j+1
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float dw = head_half(f.h, j);
            const int blk = b0 + j;
            if constexpr (ACT == HOLO_ACT_Q8) {
                const uint4 a0 = lds128(aq + (size_t)blk * 32), a1 = lds128(aq + (size_t)blk * 32 + 16);
                const int s = dot_i8x32_q8(f.q[2 * j], f.q[2 * j + 1], a0, a1);
                acc += (dw * ads[blk].x) * int_to_float_exact(s);
            } else {
                acc += dw * dot_i8x32_f32<true>(f.q[2 * j], f.q[2 * j + 1], xs + (size_t)blk * 32);
            }
        }
    }
}


// Activation prologue: x (already in shared memory at xst, zero-padded to
// nblk32p*32 values) -> optional RMSNorm with weights nw (rms_norm,
// src/ai/tensor.c:242-255: scale = 1/sqrt(sum(x^2)/n + eps), x*scale*w) ->
// HOLO_ACT_Q8: per-32-block codes aq and (d, d*asum) ads; HOLO_ACT_F32: block
// sums xsum (x normalised in place).  wsum: NT/32 floats of scratch.  Ends
// with a CTA barrier.
template <int ACT, bool NORM, int NT>
__device__ __forceinline__ void act_prologue(float *__restrict__ xst, const float *__restrict__ nw,
                                             uint8_t *__restrict__ aq, float2 *__restrict__ ads,
                                             float *__restrict__ xsum, float *__restrict__ wsum, int in_dim,
                                             int nblk32p, float eps) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float scale = 1.0f;
    if constexpr (NORM) {
        float ss = 0.0f;
        for (int i = tid * 4; i < in_dim; i += NT * 4) {
            const float4 v = *reinterpret_cast<const float4 *>(xst + i);
            ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) wsum[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < NT / 32; w++) tot += wsum[w];
        scale = 1.0f / sqrtf(tot / (float)in_dim + eps);
    }
    {
        // One thread per 32-value block (no shuffles): normalise it (NORM,
        // written back), then ACT_Q8 finds amax, d = amax/127, id = 1/d and
        // packs rint(x*id) clamped to [-127, 127] -- the arithmetic of
        // quantize_vals_q8, with the clamp applied before rounding, which gives
        // the same integers for every finite x*id -- and ACT_F32 takes the block
        // sum.  Thread l reads the eight 16-byte chunks of its block starting at
        // chunk (l + l/8) % 8, so every shared-memory wavefront hits distinct
        // banks (loads: 8 lanes, word stores: 32 lanes).
        for (int b = tid; b < nblk32p; b += NT) {
            float4 *xb = reinterpret_cast<float4 *>(xst + (size_t)b * 32);
            const int rot = tid + (tid >> 3);
            float amax = 0.0f, xsb = 0.0f;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int c = (k + rot) & 7;
                float4 v = xb[c];
                if constexpr (NORM) {
                    const float4 w4 = reinterpret_cast<const float4 *>(nw + (size_t)b * 32)[c];
                    v.x = (v.x * scale) * w4.x; v.y = (v.y * scale) * w4.y;
                    v.z = (v.z * scale) * w4.z; v.w = (v.w * scale) * w4.w;
                    xb[c] = v;
                }
                if constexpr (ACT == HOLO_ACT_Q8)
                    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
                else
                    xsb += (v.x + v.y) + (v.z + v.w);
            }
            if constexpr (ACT == HOLO_ACT_Q8) {
                const float d = __fdiv_rn(amax, 127.0f);
                const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                uint32_t *qb = reinterpret_cast<uint32_t *>(aq + (size_t)b * 32);
                int sum = 0;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int c = (k + rot) & 7;
                    const float4 v = xb[c];
                    // |clamped value| <= 127: the low byte of v + 1.5*2^23 is the
                    // two's-complement code
                    const uint32_t b0 = __float_as_uint(__fadd_rn(fminf(fmaxf(__fmul_rn(v.x, id), -127.0f), 127.0f), 12582912.0f));
                    const uint32_t b1 = __float_as_uint(__fadd_rn(fminf(fmaxf(__fmul_rn(v.y, id), -127.0f), 127.0f), 12582912.0f));
                    const uint32_t b2 = __float_as_uint(__fadd_rn(fminf(fmaxf(__fmul_rn(v.z, id), -127.0f), 127.0f), 12582912.0f));
                    const uint32_t b3 = __float_as_uint(__fadd_rn(fminf(fmaxf(__fmul_rn(v.w, id), -127.0f), 127.0f), 12582912.0f));
                    const uint32_t word = __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
                    qb[c] = word;
                    sum = __dp4a((int)word, 0x01010101, sum);
                }
                ads[b] = make_float2(d, d * (float)sum);
            } else {
                xsum[b] = xsb;
            }
        }
        __syncthreads();
    }

}

}  // namespace holo_mv
