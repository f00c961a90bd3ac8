// mv_device.cuh -- device arithmetic shared by the matvec kernels and the
// parity probes, so that the probes exercise exactly the code the kernels run.
#pragma once
#include "holo_common.cuh"

// ---------------------------------------------------------------------------
// Q8 activation quantization of one 32-element block (the library's own
// definition; the reference multiplies by fp32 activations):
//   amax = max|x|; d = amax/127; id = d ? 1/d : 0; q = rint(x*id); asum = sum q
// Each operation is correctly rounded, so results equal a C implementation
// built without contraction.  Packs q into 8 little-endian int8x4 words.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void quantize_vals_q8(const float v[32], uint32_t w[8], float &d_out, int &asum_out) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(v[i]));
    float d = __fdiv_rn(amax, 127.0f);
    float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int asum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        uint32_t word = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            int q = __float2int_rn(__fmul_rn(v[4 * i + k], id));
            q = max(-127, min(127, q));
            asum += q;
            word |= ((uint32_t)q & 0xffu) << (8 * k);
        }
        w[i] = word;
    }
    d_out = d;
    asum_out = asum;
}

__device__ __forceinline__ void quantize_block_q8(const float *__restrict__ xb, uint32_t w[8],
                                                  float &d_out, int &asum_out) {
    float v[32];
    const float4 *x4 = reinterpret_cast<const float4 *>(xb);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float4 t = __ldg(x4 + i);
        v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
    quantize_vals_q8(v, w, d_out, asum_out);
}

// ---------------------------------------------------------------------------
// Integer block dots.  `a0` holds activation positions 0..15 of the block,
// `a1` positions 16..31 (16 int8 each).
// ---------------------------------------------------------------------------
constexpr uint32_t LO4 = 0x0F0F0F0Fu;

// 16 bytes of 4-bit codes: low nibble of byte l -> position l, high -> l+16
// (src/ai/quant.c:303-307 for Q4_K, quant.c:142-150 for Q4_0).  Returns
// sum nib*qa (unsigned nibbles).
__device__ __forceinline__ int dot_nib16_q8(uint4 q, uint4 a0, uint4 a1) {
    int s = 0;
    s = __dp4a((int)(q.x & LO4), (int)a0.x, s);
    s = __dp4a((int)(q.y & LO4), (int)a0.y, s);
    s = __dp4a((int)(q.z & LO4), (int)a0.z, s);
    s = __dp4a((int)(q.w & LO4), (int)a0.w, s);
    s = __dp4a((int)((q.x >> 4) & LO4), (int)a1.x, s);
    s = __dp4a((int)((q.y >> 4) & LO4), (int)a1.y, s);
    s = __dp4a((int)((q.z >> 4) & LO4), (int)a1.z, s);
    s = __dp4a((int)((q.w >> 4) & LO4), (int)a1.w, s);
    return s;
}

// dp4a with unsigned bytes in a, signed bytes in b
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 16 * sum nib*qa, same layout as dot_nib16_q8; the high nibbles are used in
// place (byte = 16*nib) so no shift is needed; exact (|result| < 2^20).
__device__ __forceinline__ int dot_nib16_q8_x16(uint4 q, uint4 a0, uint4 a1) {
    constexpr uint32_t HI4 = 0xF0F0F0F0u;
    int lo = 0, hi = 0;
    lo = __dp4a((int)(q.x & LO4), (int)a0.x, lo);
    hi = dp4a_us(q.x & HI4, a1.x, hi);
    lo = __dp4a((int)(q.y & LO4), (int)a0.y, lo);
    hi = dp4a_us(q.y & HI4, a1.y, hi);
    lo = __dp4a((int)(q.z & LO4), (int)a0.z, lo);
    hi = dp4a_us(q.z & HI4, a1.z, hi);
    lo = __dp4a((int)(q.w & LO4), (int)a0.w, lo);
    hi = dp4a_us(q.w & HI4, a1.w, hi);
    return (lo << 4) + hi;
}

// 32 int8 codes (q0: positions 0..15, q1: 16..31) against 32 int8 activations
__device__ __forceinline__ int dot_i8x32_q8(uint4 q0, uint4 q1, uint4 a0, uint4 a1) {
    int s = 0;
    s = __dp4a((int)q0.x, (int)a0.x, s);
    s = __dp4a((int)q0.y, (int)a0.y, s);
    s = __dp4a((int)q0.z, (int)a0.z, s);
    s = __dp4a((int)q0.w, (int)a0.w, s);
    s = __dp4a((int)q1.x, (int)a1.x, s);
    s = __dp4a((int)q1.y, (int)a1.y, s);
    s = __dp4a((int)q1.z, (int)a1.z, s);
    s = __dp4a((int)q1.w, (int)a1.w, s);
    return s;
}

// ---------------------------------------------------------------------------
// fp32-activation block dots: sum code*x over one 32-element block, codes
// turned into exact floats through the 2^23 mantissa (no I2F).
// ---------------------------------------------------------------------------
// SMEM: xb points into shared memory (plain loads); else global (read-only path)
template <bool SMEM = false>
__device__ __forceinline__ float4 ld_x4(const float4 *p) {
    if constexpr (SMEM) return *p;
    else return __ldg(p);
}

template <bool SMEM = false>
__device__ __forceinline__ float dot_nib16_f32(uint4 q, const float *__restrict__ xb) {
    const float4 *x4 = reinterpret_cast<const float4 *>(xb);
    uint32_t lo[4] = {q.x & LO4, q.y & LO4, q.z & LO4, q.w & LO4};
    uint32_t hi[4] = {(q.x >> 4) & LO4, (q.y >> 4) & LO4, (q.z >> 4) & LO4, (q.w >> 4) & LO4};
    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float4 xl = ld_x4<SMEM>(x4 + i), xh = ld_x4<SMEM>(x4 + 4 + i);
        s0 = fmaf(ubyte_to_float(lo[i], 0), xl.x, s0);
        s1 = fmaf(ubyte_to_float(lo[i], 1), xl.y, s1);
        s0 = fmaf(ubyte_to_float(lo[i], 2), xl.z, s0);
        s1 = fmaf(ubyte_to_float(lo[i], 3), xl.w, s1);
        s0 = fmaf(ubyte_to_float(hi[i], 0), xh.x, s0);
        s1 = fmaf(ubyte_to_float(hi[i], 1), xh.y, s1);
        s0 = fmaf(ubyte_to_float(hi[i], 2), xh.z, s0);
        s1 = fmaf(ubyte_to_float(hi[i], 3), xh.w, s1);
    }
    return s0 + s1;
}

// signed byte k of w as an exact float (bias by 128 through the mantissa)
__device__ __forceinline__ float sbyte_to_float(uint32_t w_biased, int k) {
    return __int_as_float(__byte_perm(w_biased, 0x4B000000u, 0x7440u + k)) - 8388736.0f;
}

template <bool SMEM = false>
__device__ __forceinline__ float dot_i8x32_f32(uint4 q0, uint4 q1, const float *__restrict__ xb) {
    const float4 *x4 = reinterpret_cast<const float4 *>(xb);
    uint32_t w[8] = {q0.x ^ 0x80808080u, q0.y ^ 0x80808080u, q0.z ^ 0x80808080u, q0.w ^ 0x80808080u,
                     q1.x ^ 0x80808080u, q1.y ^ 0x80808080u, q1.z ^ 0x80808080u, q1.w ^ 0x80808080u};
    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float4 xv = ld_x4<SMEM>(x4 + i);
        s0 = fmaf(sbyte_to_float(w[i], 0), xv.x, s0);
        s1 = fmaf(sbyte_to_float(w[i], 1), xv.y, s1);
        s0 = fmaf(sbyte_to_float(w[i], 2), xv.z, s0);
        s1 = fmaf(sbyte_to_float(w[i], 3), xv.w, s1);
    }
    return s0 + s1;
}

// ---------------------------------------------------------------------------
// Q4_K header: fp16 d, fp16 dmin, 12 bytes of 6-bit scales/mins packed as in
// src/ai/quant.c:290-297.  Unpacks four scale codes per word.
// ---------------------------------------------------------------------------
struct Q4KHead {
    float d, dmin;
    uint32_t sc_lo, sc_hi, m_lo, m_hi;   // byte j of *_lo: index j, of *_hi: index j+4
};
__device__ __forceinline__ Q4KHead q4k_head(uint4 h) {
    Q4KHead r;
    r.d = half_bits_to_float(h.x & 0xffffu);
    r.dmin = half_bits_to_float(h.x >> 16);
    r.sc_lo = h.y & 0x3F3F3F3Fu;
    r.m_lo = h.z & 0x3F3F3F3Fu;
    r.sc_hi = ((h.w & LO4) << 2) | ((h.y >> 6) & 0x03030303u);
    r.m_hi = (((h.w >> 4) & LO4) << 2) | ((h.z >> 6) & 0x03030303u);
    return r;
}
__device__ __forceinline__ float q4k_scale(const Q4KHead &h, int j) {
    return ubyte_to_float(j < 4 ? h.sc_lo : h.sc_hi, j & 3);
}
__device__ __forceinline__ float q4k_min(const Q4KHead &h, int j) {
    return ubyte_to_float(j < 4 ? h.m_lo : h.m_hi, j & 3);
}

// ---------------------------------------------------------------------------
// RoPE angle of pair i at position pos (src/ai/llm.c:1139-1142):
//   freq = 1 / base^((2i)/hd), theta = pos * freq, in float32.
// pow, cos and sin are evaluated in double and rounded once to float, so the
// float32 values are the correctly rounded ones (what a correctly rounded
// libm returns); the float operations around them round as in the C code.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void rope_cos_sin(int pos, int i, int hd, float base, float &c, float &s) {
    const float ex = __fdiv_rn((float)(2 * i), (float)hd);
    const float pw = (float)pow((double)base, (double)ex);
    const float freq = __fdiv_rn(1.0f, pw);
    const float theta = __fmul_rn((float)pos, freq);
    double sd, cd;
    sincos((double)theta, &sd, &cd);
    c = (float)cd;
    s = (float)sd;
}
// (a, b) <- (a*c - b*s, a*s + b*c), each product and sum rounded separately
__device__ __forceinline__ void rope_rotate(float &a, float &b, float c, float s) {
    const float a0 = a, b0 = b;
    a = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(b0, s));
    b = __fadd_rn(__fmul_rn(a0, s), __fmul_rn(b0, c));
}

// ---------------------------------------------------------------------------
// Tiled-layout addressing (holo_common.cuh): the unit holding row r and
// position block b (32-value block for Q8_0/Q4_0, super-block for Q4_K).
// ---------------------------------------------------------------------------
template <int TYPE>
__device__ __forceinline__ const uint8_t *unit_ptr(const uint8_t *W, int units, int r, int s) {
    return W + ((size_t)(r / TILE_ROWS) * units + s) * UnitGeom<TYPE>::UNIT_BYTES;
}
