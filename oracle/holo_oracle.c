/*
 * holo_oracle.c -- CPU restatement of holo's quantized matvec (checker only).
 *
 * TEST INFRASTRUCTURE ONLY: see holo_oracle.h.  Nothing in the product library
 * links this file; tests/ compare the CUDA path against it, and it is itself
 * pinned against the reference's own C code compiled from source
 * (oracle/_ref, built by oracle/Makefile) and against committed fixtures in
 * tests/golden/.
 */
#include "holo_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef union { uint32_t u; float f; } bits32;

/* ---- fp16 ------------------------------------------------------------------ */

/* Exact widening of binary16, including subnormals, infinities and NaN
 * payloads: the value table of src/ai/quant.c:44-82. */
float ho_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp5 = (h >> 10) & 0x1fu;
    uint32_t frac = h & 0x3ffu;
    bits32 r;
    if (exp5 == 0x1fu) {
        r.u = sign | 0x7f800000u | (frac << 13);
    } else if (exp5 != 0) {
        r.u = sign | ((exp5 + 112u) << 23) | (frac << 13);
    } else if (frac == 0) {
        r.u = sign;
    } else {
        /* subnormal: frac * 2^-24, exact in binary32 */
        r.f = (float)frac * 5.9604644775390625e-8f;
        r.u |= sign;
    }
    return r.f;
}

uint16_t ho_f32_to_f16_rn(float f) {
    bits32 b; b.f = f;
    uint32_t sign = (b.u >> 16) & 0x8000u;
    uint32_t ax = b.u & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);   /* >= 65520 -> inf */
    if (ax < 0x38800000u) {                                     /* below 2^-14 */
        bits32 a; a.u = ax;
        uint32_t m = (uint32_t)rintf(a.f * 16777216.0f);        /* units of 2^-24 */
        return (uint16_t)(sign | m);
    }
    uint32_t e = (ax >> 23) - 112u;
    uint32_t m = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* ---- block geometry (src/ai/quant.h:43-120, quant.c:676-719) ------------------ */

int64_t ho_row_bytes(int type, int64_t cols) {
    switch (type) {
    case HO_TYPE_F32:  return cols * 4;
    case HO_TYPE_F16:  return cols * 2;
    case HO_TYPE_Q8_0: return (cols / 32) * 34;
    case HO_TYPE_Q4_0: return (cols / 32) * 18;
    case HO_TYPE_Q4_K: return (cols / 256) * 144;
    case HO_TYPE_Q6_K: return (cols / 256) * 210;
    default: return -1;
    }
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* 6-bit scale/min unpack of src/ai/quant.c:290-297 */
static void q4k_unpack_ref(const uint8_t *sp, uint8_t sc[8], uint8_t mn[8]) {
    for (int j = 0; j < 4; j++) {
        sc[j] = sp[j] & 0x3f;
        mn[j] = sp[j + 4] & 0x3f;
        sc[j + 4] = (uint8_t)(((sp[j + 8] & 0x0f) << 2) | (sp[j] >> 6));
        mn[j + 4] = (uint8_t)(((sp[j + 8] >> 4) << 2) | (sp[j + 4] >> 6));
    }
}

/* get_scale_min_k4 of src/ai/cuda_ops.cu:684-692 */
static void q4k_unpack_ggml(const uint8_t *q, uint8_t sc[8], uint8_t mn[8]) {
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            sc[j] = q[j] & 63;
            mn[j] = q[j + 4] & 63;
        } else {
            sc[j] = (uint8_t)((q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4));
            mn[j] = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
        }
    }
}

void ho_q4k_to_ref_layout(const void *src_block, void *dst_block, int src_layout) {
    const uint8_t *s = (const uint8_t *)src_block;
    uint8_t out[144];
    if (src_layout == HO_Q4K_REF) { memcpy(dst_block, s, 144); return; }
    uint8_t sc[8], mn[8], nib[256];
    q4k_unpack_ggml(s + 4, sc, mn);
    /* cuda_ops.cu:712-729: 32 bytes per 64 values, low nibbles first */
    for (int g = 0; g < 4; g++)
        for (int l = 0; l < 32; l++) {
            uint8_t byte = s[16 + g * 32 + l];
            nib[g * 64 + l] = byte & 0x0f;
            nib[g * 64 + 32 + l] = byte >> 4;
        }
    memcpy(out, s, 4);                           /* d, dmin */
    for (int j = 0; j < 4; j++) {                /* inverse of quant.c:290-297 */
        out[4 + j] = (uint8_t)(sc[j] | ((sc[j + 4] & 3) << 6));
        out[4 + j + 4] = (uint8_t)(mn[j] | ((mn[j + 4] & 3) << 6));
        out[4 + j + 8] = (uint8_t)((sc[j + 4] >> 2) | ((mn[j + 4] >> 2) << 4));
    }
    for (int j = 0; j < 8; j++)                  /* quant.c:303-307 placement */
        for (int l = 0; l < 16; l++)
            out[16 + j * 16 + l] = (uint8_t)(nib[j * 32 + l] | (nib[j * 32 + l + 16] << 4));
    memcpy(dst_block, out, 144);
}

/* ---- dequantization -------------------------------------------------------- */

void ho_dequant_row(int type, const void *row, float *y, int64_t cols, int q4k_layout) {
    const uint8_t *p = (const uint8_t *)row;
    switch (type) {
    case HO_TYPE_Q8_0:                                       /* quant.c:118-128 */
        for (int64_t b = 0; b < cols / 32; b++, p += 34) {
            float d = ho_f16_to_f32(rd16(p));
            for (int i = 0; i < 32; i++) y[b * 32 + i] = d * (float)(int8_t)p[2 + i];
        }
        break;
    case HO_TYPE_Q4_0:                                       /* quant.c:136-153 */
        for (int64_t b = 0; b < cols / 32; b++, p += 18) {
            float d = ho_f16_to_f32(rd16(p));
            for (int i = 0; i < 16; i++) {
                y[b * 32 + i] = d * (float)((p[2 + i] & 0x0f) - 8);
                y[b * 32 + i + 16] = d * (float)((p[2 + i] >> 4) - 8);
            }
        }
        break;
    case HO_TYPE_Q4_K:                                       /* quant.c:277-311 */
        for (int64_t s = 0; s < cols / 256; s++, p += 144) {
            uint8_t blk[144], sc[8], mn[8];
            ho_q4k_to_ref_layout(p, blk, q4k_layout);
            float d = ho_f16_to_f32(rd16(blk)), dmin = ho_f16_to_f32(rd16(blk + 2));
            q4k_unpack_ref(blk + 4, sc, mn);
            for (int j = 0; j < 8; j++) {
                float scale = d * (float)sc[j];
                float mval = dmin * (float)mn[j];
                for (int l = 0; l < 16; l++) {
                    uint8_t byte = blk[16 + j * 16 + l];
                    y[s * 256 + j * 32 + l] = scale * (float)(byte & 0x0f) - mval;
                    y[s * 256 + j * 32 + l + 16] = scale * (float)(byte >> 4) - mval;
                }
            }
        }
        break;
    case HO_TYPE_Q6_K:                                       /* quant.c:241-275 */
        for (int64_t s = 0; s < cols / 256; s++, p += 210) {
            float d = ho_f16_to_f32(rd16(p + 208));
            for (int n = 0; n < 2; n++) {
                const uint8_t *ql = p + n * 64, *qh = p + 128 + n * 32;
                const int8_t *sc = (const int8_t *)(p + 192) + n * 8;
                float *yy = y + s * 256 + n * 128;
                for (int l = 0; l < 32; l++) {
                    int is = l / 16;
                    int8_t q1 = (int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                    int8_t q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    int8_t q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    int8_t q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    yy[l] = d * sc[is + 0] * q1;
                    yy[l + 32] = d * sc[is + 2] * q2;
                    yy[l + 64] = d * sc[is + 4] * q3;
                    yy[l + 96] = d * sc[is + 6] * q4;
                }
            }
        }
        break;
    case HO_TYPE_F16:
        for (int64_t i = 0; i < cols; i++) y[i] = ho_f16_to_f32(rd16(p + 2 * i));
        break;
    case HO_TYPE_F32:
        memcpy(y, row, (size_t)cols * 4);
        break;
    default:
        memset(y, 0, (size_t)cols * 4);
    }
}

/* ---- fp32-activation matvec: the arithmetic of src/ai/llm.c:770-926 --------- */

/* llm.c:836-874: eight lane accumulators, lane i takes elements k+i of each
 * 8-group; each term is (q*x)*scale; then lanes i and i+4 are added and the
 * four sums are combined as (s0+s1)+(s2+s3). */
static float row_q8_0_f32(const uint8_t *row, const float *x, int cols) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < cols / 32; b++) {
        const uint8_t *blk = row + (int64_t)b * 34;
        float scale = ho_f16_to_f32(rd16(blk));
        for (int k = 0; k < 32; k += 8)
            for (int i = 0; i < 8; i++) {
                float prod = (float)(int8_t)blk[2 + k + i] * x[b * 32 + k + i];
                prod = prod * scale;
                acc[i] = acc[i] + prod;
            }
    }
    float s0 = acc[0] + acc[4], s1 = acc[1] + acc[5], s2 = acc[2] + acc[6], s3 = acc[3] + acc[7];
    return (s0 + s1) + (s2 + s3);
}

/* llm.c:893-915 */
static float row_q4_0_f32(const uint8_t *row, const float *x, int cols) {
    float sum = 0.0f;
    for (int b = 0; b < cols / 32; b++) {
        const uint8_t *blk = row + (int64_t)b * 18;
        float scale = ho_f16_to_f32(rd16(blk));
        for (int k = 0; k < 16; k++) {
            uint8_t byte = blk[2 + k];
            sum += scale * (float)((byte & 0x0f) - 8) * x[b * 32 + k];
            sum += scale * (float)((byte >> 4) - 8) * x[b * 32 + k + 16];
        }
    }
    return sum;
}

/* quant.c:541-580 */
static float row_q4_k_f32(const uint8_t *row, const float *x, int cols, int layout) {
    float sum = 0.0f;
    for (int s = 0; s < cols / 256; s++) {
        uint8_t blk[144], sc[8], mn[8];
        ho_q4k_to_ref_layout(row + (int64_t)s * 144, blk, layout);
        float d = ho_f16_to_f32(rd16(blk)), dmin = ho_f16_to_f32(rd16(blk + 2));
        q4k_unpack_ref(blk + 4, sc, mn);
        for (int j = 0; j < 8; j++) {
            float scale = d * (float)sc[j];
            float mval = dmin * (float)mn[j];
            const float *xb = x + s * 256 + j * 32;
            for (int l = 0; l < 16; l++) {
                uint8_t byte = blk[16 + j * 16 + l];
                sum += (scale * (float)(byte & 0x0f) - mval) * xb[l];
                sum += (scale * (float)(byte >> 4) - mval) * xb[l + 16];
            }
        }
    }
    return sum;
}

/* quant.c:582-601: each super-block dequantized (quant.c:241-275), then one
 * running sum over the values in order */
static float row_q6_k_f32(const uint8_t *row, const float *x, int cols) {
    float sum = 0.0f, tmp[256];
    for (int s = 0; s < cols / 256; s++) {
        ho_dequant_row(HO_TYPE_Q6_K, row + (int64_t)s * 210, tmp, 256, 0);
        for (int j = 0; j < 256; j++) sum += tmp[j] * x[s * 256 + j];
    }
    return sum;
}

/* llm.c:817-827 */
static float row_f16_f32(const uint8_t *row, const float *x, int cols) {
    float sum = 0.0f;
    for (int j = 0; j < cols; j++) sum += ho_f16_to_f32(rd16(row + 2 * j)) * x[j];
    return sum;
}

void ho_matvec_f32act(int type, const void *W, const float *x, float *y,
                      int rows, int cols, int q4k_layout, int nthreads) {
    const uint8_t *base = (const uint8_t *)W;
    int64_t rb = ho_row_bytes(type, cols);
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (int r = 0; r < rows; r++) {
        const uint8_t *row = base + (int64_t)r * rb;
        float v;
        switch (type) {
        case HO_TYPE_Q8_0: v = row_q8_0_f32(row, x, cols); break;
        case HO_TYPE_Q4_0: v = row_q4_0_f32(row, x, cols); break;
        case HO_TYPE_Q4_K: v = row_q4_k_f32(row, x, cols, q4k_layout); break;
        case HO_TYPE_Q6_K: v = row_q6_k_f32(row, x, cols); break;
        case HO_TYPE_F16:  v = row_f16_f32(row, x, cols); break;
        default: v = 0.0f;
        }
        y[r] = v;
    }
}

/* ---- Q8 activations (no reference code: the build's own definition) -------- */

void ho_quantize_act_q8(const float *x, int64_t n, int8_t *q, float *d, int32_t *asum) {
    for (int64_t b = 0; b < n / 32; b++) {
        const float *xb = x + b * 32;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) {
            float a = fabsf(xb[i]);
            if (a > amax) amax = a;
        }
        float db = amax / 127.0f;
        float id = db != 0.0f ? 1.0f / db : 0.0f;
        int32_t s = 0;
        for (int i = 0; i < 32; i++) {
            float v = xb[i] * id;
            int qi = (int)rintf(v);
            if (qi > 127) qi = 127;
            if (qi < -127) qi = -127;
            q[b * 32 + i] = (int8_t)qi;
            s += qi;
        }
        d[b] = db;
        asum[b] = s;
    }
}

void ho_matvec_q8act(int type, const void *W, const int8_t *q, const float *d,
                     const int32_t *asum, float *y, int rows, int cols,
                     int q4k_layout, int32_t *isums, int nthreads) {
    const uint8_t *base = (const uint8_t *)W;
    int64_t rb = ho_row_bytes(type, cols);
    int nblk = cols / 32;
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (int r = 0; r < rows; r++) {
        const uint8_t *row = base + (int64_t)r * rb;
        int32_t *is_row = isums ? isums + (int64_t)r * nblk : NULL;
        float acc = 0.0f;
        if (type == HO_TYPE_Q8_0 || type == HO_TYPE_Q4_0) {
            for (int b = 0; b < nblk; b++) {
                const uint8_t *blk = row + (int64_t)b * (type == HO_TYPE_Q8_0 ? 34 : 18);
                const int8_t *qa = q + b * 32;
                int32_t s = 0;
                if (type == HO_TYPE_Q8_0) {
                    for (int i = 0; i < 32; i++) s += (int32_t)(int8_t)blk[2 + i] * qa[i];
                } else {
                    for (int i = 0; i < 16; i++) {
                        s += ((blk[2 + i] & 0x0f) - 8) * qa[i];
                        s += ((blk[2 + i] >> 4) - 8) * qa[i + 16];
                    }
                }
                if (is_row) is_row[b] = s;
                float dw = ho_f16_to_f32(rd16(blk));
                acc += (dw * d[b]) * (float)s;
            }
        } else if (type == HO_TYPE_Q4_K) {
            for (int sb = 0; sb < cols / 256; sb++) {
                uint8_t blk[144], sc[8], mn[8];
                ho_q4k_to_ref_layout(row + (int64_t)sb * 144, blk, q4k_layout);
                float dd = ho_f16_to_f32(rd16(blk)), dmin = ho_f16_to_f32(rd16(blk + 2));
                q4k_unpack_ref(blk + 4, sc, mn);
                for (int j = 0; j < 8; j++) {
                    int b = sb * 8 + j;
                    const int8_t *qa = q + b * 32;
                    int32_t s = 0;
                    for (int l = 0; l < 16; l++) {
                        uint8_t byte = blk[16 + j * 16 + l];
                        s += (byte & 0x0f) * qa[l];
                        s += (byte >> 4) * qa[l + 16];
                    }
                    if (is_row) is_row[b] = s;
                    float t = (dd * (float)sc[j]) * (float)s - (dmin * (float)mn[j]) * (float)asum[b];
                    acc += d[b] * t;
                }
            }
        } else if (type == HO_TYPE_Q6_K) {
            /* the value layout of quant.c:241-275; per 16 values (one scale)
             * the integer sum of code * q, then d_a * (w0 * s0 + w1 * s1) per
             * 32-block with w = d * scale (the build's own definition) */
            for (int sb = 0; sb < cols / 256; sb++) {
                const uint8_t *blk = row + (int64_t)sb * 210;
                float dd = ho_f16_to_f32(rd16(blk + 208));
                for (int n = 0; n < 2; n++) {
                    const uint8_t *ql = blk + n * 64, *qh = blk + 128 + n * 32;
                    const int8_t *sc = (const int8_t *)(blk + 192) + n * 8;
                    for (int j = 0; j < 4; j++) {
                        int b = sb * 8 + n * 4 + j;
                        const int8_t *qa = q + b * 32;
                        int32_t s2[2] = {0, 0};
                        for (int l = 0; l < 32; l++) {
                            int byte = (j & 1) ? ql[l + 32] : ql[l];
                            int nib = (j & 2) ? (byte >> 4) : (byte & 0xF);
                            int code = (nib | (((qh[l] >> (2 * j)) & 3) << 4)) - 32;
                            s2[l / 16] += code * qa[l];
                        }
                        if (is_row) is_row[b] = s2[0] + s2[1];
                        float w0 = dd * (float)sc[2 * j], w1 = dd * (float)sc[2 * j + 1];
                        acc += d[b] * (w0 * (float)s2[0] + w1 * (float)s2[1]);
                    }
                }
            }
        }
        y[r] = acc;
    }
}

/* ---- tokenizer ----------------------------------------------------------------- */

/* The byte-level string the reference assigns to byte b (llm.c:116-147):
 * printable ASCII 33..126 is itself; bytes 161 and 166..172 have none; every
 * other byte, counted in increasing order, is code point 256 + its rank,
 * written as two UTF-8 bytes.  Returns the string length (0: none). */
static int ho_byte_string(int b, char out[3]) {
    if (b >= 33 && b <= 126) { out[0] = (char)b; out[1] = 0; return 1; }
    if (b == 161 || (b >= 166 && b <= 172)) { out[0] = 0; return 0; }
    int rank = 0;
    for (int i = 0; i < b; i++)
        if (!(i >= 33 && i <= 126) && !(i == 161 || (i >= 166 && i <= 172))) rank++;
    int cp = 256 + rank;
    out[0] = (char)(0xC0 | (cp >> 6));
    out[1] = (char)(0x80 | (cp & 0x3F));
    out[2] = 0;
    return 2;
}

/* first vocabulary index whose string equals s, or -1 */
static int ho_find_exact(const char *const *vocab, int vocab_size, const char *s) {
    for (int i = 0; i < vocab_size; i++)
        if (vocab[i] && strcmp(vocab[i], s) == 0) return i;
    return -1;
}

int ho_tokenize(const char *const *vocab, int vocab_size, int bos, int unk, const char *text,
                int *tokens, int max_tokens, int add_bos) {
    int n = 0;
    if (add_bos && n < max_tokens) tokens[n++] = bos;
    const char *p = text;
    while (*p && n < max_tokens) {
        /* longest vocabulary string that prefixes p; the first of that length */
        size_t best_len = 0;
        int best = unk;
        for (int i = 0; i < vocab_size; i++) {
            if (!vocab[i]) continue;
            size_t len = strlen(vocab[i]);
            if (len > best_len && strncmp(p, vocab[i], len) == 0) { best_len = len; best = i; }
        }
        if (best_len > 0) { tokens[n++] = best; p += best_len; continue; }
        /* one byte: <0xNN>, else the byte-level string, else unk */
        unsigned char b = (unsigned char)*p;
        char hex[8], bs[3];
        snprintf(hex, sizeof hex, "<0x%02X>", b);
        int id = ho_find_exact(vocab, vocab_size, hex);
        if (id < 0 && ho_byte_string(b, bs) > 0) id = ho_find_exact(vocab, vocab_size, bs);
        tokens[n++] = id >= 0 ? id : unk;
        p++;
    }
    return n;
}
