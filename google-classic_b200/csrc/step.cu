// step.cu -- one decode step (one token) as a single persistent kernel.
//
// The step of decode.cu as phases of one cooperative launch, one 256-thread
// CTA per SM:
//
//   embed | per layer: QKV (RMSNorm fused) | RoPE + KV append + attention |
//   Wo (+x) | W1/W3 (RMSNorm, SwiGLU) | W2 (+x) | output matrix (RMSNorm) |
//   sampler (CTA 0)
//
// The reference's sequence is the same as in decode.cu (src/ai/llm.c:1015-1269,
// 1281-1328).  What the single kernel buys over one launch per op:
//   * no launch, drain or grid barrier between ops: the vectors between
//     phases are LL vectors (step.cuh), so a CTA starts a phase as soon as the
//     elements it reads carry the producing phase's epoch;
//   * every matvec phase gives each CTA whole row-blocks, so outputs are final
//     in the CTA (no split-K fix-up, no atomics);
//   * an L2 prefetch table keeps ~32 MB of upcoming weights requested from
//     HBM at all times (cp.async.bulk.prefetch.L2, split over the CTAs), so HBM
//     streams while the phases compute from L2.
// Sharded over several GPUs (one process each), the phases store their
// slices into every rank's LL copies over NVLink; nothing else changes.
// Every wait (LL polls, bulk copies) is bounded; a CTA that gives up records
// HOLO_E_TIMEOUT, waits elsewhere see the status and give up too, and later
// launches return at once.
#include "holo_common.cuh"
#include "mv_device.cuh"
#include "mv_unit.cuh"
#include "step.cuh"

#include <algorithm>
#include <cfloat>
#include <type_traits>

namespace {

using namespace holo_mv;
using namespace holo_dec;

// The layers kernel runs 8 warps a CTA with each warp's next weight units in
// a register ring (255 registers a thread): its phases are short, and the
// register path starts computing soonest.  The output kernel, one long
// matvec, runs 16 warps with the weight units staged in shared memory by bulk
// copies (128 registers a thread, twice the warps to hide latency).
constexpr int LY_WARPS = 8;
constexpr int LY_THREADS = LY_WARPS * 32;
constexpr int OUT_WARPS = 16;
constexpr int OUT_THREADS = OUT_WARPS * 32;
constexpr int MAX_WARPS = 16;
constexpr int ST_RING = 3;                         // register ring: units loading per warp
constexpr int ST_MAX_DEPTH = 3;                    // shared-memory slots per warp, at most
constexpr int ST_HD = 128;                         // head_dim of this kernel
constexpr unsigned long long ST_WAIT_NS = 1000000000ull;
constexpr size_t ST_PERSIST = 2048;                // bytes of the persistent shared region

// shared memory kept across phases (start of the dynamic allocation)
struct StepPersist {
    float2 rope[ST_HD / 2];    // (cos, sin) of the RoPE pairs at pos
    uint64_t mbar;             // bulk-copy completion (norm weights)
    uint64_t slot[MAX_WARPS * ST_MAX_DEPTH];  // weight slot k of warp w: [w * ST_MAX_DEPTH + k]
    unsigned long long launch; // launch index (barrier targets)
    int ok;
    int pos;
};
static_assert(sizeof(StepPersist) <= ST_PERSIST, "persistent region");

template <int T> __device__ __forceinline__ int units_of(int cols) {
    return (cols + UnitGeom<T>::VALS - 1) / UnitGeom<T>::VALS;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}

// ---------------------------------------------------------------------------
// LL words (step.cuh): float in the low half, epoch in the high half.  The
// accesses are volatile (never served from L1) and 8 or 16 bytes wide; every
// 8-byte word is written and read whole.
// ---------------------------------------------------------------------------
__device__ __forceinline__ StepWord ll_word(float v, unsigned e) {
    return ((StepWord)e << 32) | __float_as_uint(v);
}
__device__ __forceinline__ float ll_val(StepWord w) { return __uint_as_float((unsigned)w); }
__device__ __forceinline__ bool ll_ok(StepWord w, unsigned e) { return (unsigned)(w >> 32) == e; }
__device__ __forceinline__ void ll_st(StepWord *p, float v, unsigned e) {
    asm volatile("st.volatile.global.u64 [%0], %1;" :: "l"(p), "l"(ll_word(v, e)) : "memory");
}
__device__ __forceinline__ void ll_st2(StepWord *p, float a, float b, unsigned e) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" :: "l"(p), "l"(ll_word(a, e)), "l"(ll_word(b, e))
                 : "memory");
}
__device__ __forceinline__ StepWord ll_ld(const StepWord *p) {
    StepWord v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ll_ld2(const StepWord *p, StepWord &a, StepWord &b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// bookkeeping of one poll loop: false once ST_WAIT_NS has passed (status set)
// or another CTA has already recorded an error
struct Poll {
    unsigned it = 0;
    unsigned long long t0 = 0;
    __device__ __forceinline__ bool again(int *status) {
        if ((++it & 31u) != 0) return true;
        if (*reinterpret_cast<volatile int *>(status) != 0) return false;
        const unsigned long long t = holo_globaltimer();
        if (t0 == 0) {
            t0 = t;
        } else if (t - t0 > ST_WAIT_NS) {
            atomicExch(status, HOLO_E_TIMEOUT);
            return false;
        }
        return true;
    }
};

// dst[0..n) <- the values of src[0..n) once every word holds epoch e (n even,
// src 16-byte aligned; dst shared or global).  Each thread keeps LL_BATCH
// 16-byte loads in flight and re-polls the batch until all are current.
constexpr int LL_BATCH = 8;
template <int NT>
__device__ bool ll_gather(float *dst, const StepWord *src, int n, unsigned e, int *status) {
    const int npair = n >> 1;
    for (int base = threadIdx.x; base < npair; base += NT * LL_BATCH) {
        StepWord w[2 * LL_BATCH];
        Poll poll;
        for (;;) {
#pragma unroll
            for (int k = 0; k < LL_BATCH; ++k) {
                const int i = base + k * NT;
                if (i < npair) ll_ld2(src + 2 * i, w[2 * k], w[2 * k + 1]);
                else w[2 * k] = w[2 * k + 1] = (StepWord)e << 32;
            }
            bool ready = true;
#pragma unroll
            for (int k = 0; k < 2 * LL_BATCH; ++k) ready &= ll_ok(w[k], e);
            if (ready) break;
            if (!poll.again(status)) return false;
        }
#pragma unroll
        for (int k = 0; k < LL_BATCH; ++k) {
            const int i = base + k * NT;
            if (i < npair) *reinterpret_cast<float2 *>(dst + 2 * i) = make_float2(ll_val(w[2 * k]), ll_val(w[2 * k + 1]));
        }
    }
    return true;
}

// one value (a word already known to be written, or nearly)
__device__ __forceinline__ bool ll_get(const StepWord *p, unsigned e, int *status, float &v) {
    Poll poll;
    for (;;) {
        const StepWord w = ll_ld(p);
        if (ll_ok(w, e)) {
            v = ll_val(w);
            return true;
        }
        if (!poll.again(status)) return false;
    }
}

// 16 consecutive values (16-byte aligned) into registers
__device__ __forceinline__ bool ll_get16(const StepWord *p, unsigned e, int *status, float (&o)[16]) {
    Poll poll;
    for (;;) {
        StepWord w[16];
#pragma unroll
        for (int k = 0; k < 8; ++k) ll_ld2(p + 2 * k, w[2 * k], w[2 * k + 1]);
        bool ready = true;
#pragma unroll
        for (int k = 0; k < 16; ++k) ready &= ll_ok(w[k], e);
        if (ready) {
#pragma unroll
            for (int k = 0; k < 16; ++k) o[k] = ll_val(w[k]);
            return true;
        }
        if (!poll.again(status)) return false;
    }
}

// epoch of phase ph of the step that launch number `launch` runs: phase 0
// embedding, 1 .. 5L the layers' phases, 5L + 1 the output matrix (never 0:
// the buffers start zeroed)
__device__ __forceinline__ unsigned step_epoch(const StepArgs &a, unsigned long long launch, int ph) {
    return (unsigned)(launch * (unsigned long long)step_phases(a.n_layers) + (unsigned long long)ph + 1ull);
}

// this CTA's share of the phase's L2 prefetch ranges (warp 0, 32 KB requests)
__device__ void step_prefetch(const StepArgs &a, int phase) {
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    const StepPrefetch *pf = a.prefetch + (size_t)phase * STEP_PF_MAX;
    constexpr unsigned long long CH = 32768;
    for (int k = 0; k < STEP_PF_MAX; ++k) {
        const unsigned long long n = pf[k].bytes;
        if (n == 0) continue;
        const unsigned long long c = blockIdx.x, G = a.grid;
        const unsigned long long b0 = (n * c / G) & ~15ull;
        const unsigned long long b1 = c + 1 == G ? n : ((n * (c + 1) / G) & ~15ull);
        for (unsigned long long o = b0 + (unsigned long long)lane * CH; o < b1; o += 32 * CH)
            prefetch_l2_bulk(pf[k].ptr + o, (uint32_t)(b1 - o < CH ? b1 - o : CH));
    }
}

__device__ __forceinline__ size_t align128(size_t v) { return (v + 127) & ~(size_t)127; }

// ---------------------------------------------------------------------------
// matvec phase: rows x in_dim unit-layout weight, whole row-blocks per CTA
// ---------------------------------------------------------------------------
// x: LL input vector (epoch ex); epi: 0 store, 1 y = residual + W.x (residual
// an LL vector of epoch er), 2 SwiGLU over rows interleaved by 16; norm_w
// non-NULL: RMSNorm of x first.  rows: this rank's rows of W; output row j
// goes to element yoff + j of ydst[0..ncopy) (every rank's copy) with epoch
// ey.  One instance per weight type and kernel: the kernel calls it from a
// single site (separate inlined copies per phase exhaust the register file).
//
// NW warps; warp w takes the CTA's units w, w + NW, ...  SMEMW false: each
// warp keeps its next ST_RING units in registers.  SMEMW true: warp w owns
// a.mv_depth shared-memory slots that its lane 0 fills by 1-D bulk copies
// and refills with the warp's next unit once the warp has folded the current
// one; spar holds the warp's slot parities across phases.
template <int TYPE, int ACT, int NW, bool SMEMW>
__device__ __forceinline__ bool step_mv(const StepArgs &a, StepPersist &P, uint8_t *sm, unsigned &mb_par,
                        unsigned &spar, const uint8_t *__restrict__ W, int rows, int in_dim, const StepWord *x,
                        unsigned ex, StepWord *const *ydst, int ncopy, int yoff, unsigned ey,
                        const StepWord *residual, unsigned er, const float *norm_w, int epi) {
    constexpr int NT = NW * 32;
    const bool norm = norm_w != nullptr;
    constexpr int BLKS32 = UnitGeom<TYPE>::BLKS32;
    constexpr size_t UB = UnitGeom<TYPE>::UNIT_BYTES;
    const int D = SMEMW ? a.mv_depth : 0;
    const int units = units_of<TYPE>(in_dim), nblk32p = units * BLKS32;
    const int nrb = (rows + TILE_ROWS - 1) / TILE_ROWS;
    const int G = a.grid, c = blockIdx.x;
    const int rb0 = (int)((long long)nrb * c / G), rb1 = (int)((long long)nrb * (c + 1) / G);
    if (rb0 >= rb1) return true;
    const int nloc = rb1 - rb0;
    const int u0 = rb0 * units, n = (rb1 - rb0) * units;   // this CTA's units [u0, u0 + n)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    uint8_t *ring = sm;                                    // SMEMW: [NW * D] slots of UB bytes
    size_t o = SMEMW ? align128((size_t)NW * D * UB) : 0;
    float *red = reinterpret_cast<float *>(sm + o);
    o += align128((size_t)nloc * NW * 32 * sizeof(float));
    uint8_t *aq = sm + o;
    float2 *ads = reinterpret_cast<float2 *>(sm + o + (size_t)nblk32p * 32);
    float *xst, *xsum = nullptr;
    if constexpr (ACT == HOLO_ACT_Q8) {
        o += align128((size_t)nblk32p * 40);
        xst = reinterpret_cast<float *>(sm + o);
        o += (size_t)nblk32p * 128;
    } else {
        xst = reinterpret_cast<float *>(sm + o);
        xsum = xst + (size_t)nblk32p * 32;
        o += align128((size_t)nblk32p * 132);
    }
    float *nw = reinterpret_cast<float *>(sm + o);
    if (norm) o += (size_t)nblk32p * 128;
    float *wsum = reinterpret_cast<float *>(sm + o);

    // the warp's first units (registers or slots), and the norm weights,
    // requested while the activations are polled
    Frag ring_r[SMEMW ? 1 : ST_RING];
    uint64_t pol = 0;
    if constexpr (SMEMW) {
        pol = l2_policy_evict_first();
        if (lane == 0) {
            for (int k = 0; k < D; ++k) {
                const int i = warp + k * NW;
                if (i < n) {
                    uint64_t *fb = &P.slot[warp * ST_MAX_DEPTH + k];
                    mbar_arrive_expect_tx(fb, (uint32_t)UB);
                    bulk_g2s(ring + (size_t)(warp * D + k) * UB, W + (size_t)(u0 + i) * UB, (uint32_t)UB, fb, pol);
                }
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < ST_RING; ++k) {
            const int i = warp + k * NW;
            if (i < n) load_unit<TYPE>(ring_r[k], W + (size_t)(u0 + i) * UB, lane);
        }
    }
    const uint32_t xbytes = (uint32_t)in_dim * 4u;
    if (norm && tid == 0) {
        mbar_arrive_expect_tx(&P.mbar, xbytes);
        bulk_copy_g2s(nw, norm_w, xbytes, &P.mbar);
    }
    // the residual of the warp's first row-block, requested now (it was
    // written phases ago) rather than on the epilogue's critical path
    StepWord rw = 0;
    if (epi == 1 && warp < nloc && (rb0 + warp) * TILE_ROWS + lane < rows)
        rw = ll_ld(residual + yoff + (rb0 + warp) * TILE_ROWS + lane);
    for (int i = in_dim + tid; i < nblk32p * 32; i += NT) {
        xst[i] = 0.0f;
        if (norm) nw[i] = 0.0f;
    }
    for (int i = tid; i < nloc * NW * 32; i += NT) red[i] = 0.0f;
    bool ok = ll_gather<NT>(xst, x, in_dim, ex, a.status);
    if (norm) {
        ok = mbar_wait_bounded(&P.mbar, mb_par, a.status, HOLO_E_TIMEOUT) && ok;
        mb_par ^= 1u;
    }
    ok = __syncthreads_and(ok) != 0;
    if (ok) {
        if (norm) act_prologue<ACT, true, NT>(xst, nw, aq, ads, xsum, wsum, in_dim, nblk32p, a.eps);
        else act_prologue<ACT, false, NT>(xst, nw, aq, ads, xsum, wsum, in_dim, nblk32p, a.eps);
    }
    const float *xs = xst;

    // unit u0 + i, i = warp, warp + NW, ...: row-block rb, unit s of its row
    int rb = (u0 + warp) / units, s = u0 + warp - rb * units;
    const int dq = NW / units, dr = NW - dq * units;
    int cur_rb = rb;
    float acc = 0.0f;
    bool wok = ok;   // a failed slot wait skips the warp's remaining units
    if constexpr (SMEMW) {
        int k = 0, i = warp;
        for (; wok && i < n; i += NW) {
            uint64_t *fb = &P.slot[warp * ST_MAX_DEPTH + k];
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(fb, (spar >> k) & 1u, a.status, HOLO_E_TIMEOUT))) {
                wok = false;
                break;
            }
            spar ^= 1u << k;
            Frag f;
            load_unit_smem<TYPE>(f, ring + (size_t)(warp * D + k) * UB, lane);
            if (rb != cur_rb) {
                red[((cur_rb - rb0) * NW + warp) * 32 + lane] = acc;
                acc = 0.0f;
                cur_rb = rb;
            }
            unit_dot<TYPE, ACT>(acc, f, s * BLKS32, aq, ads, xs, xsum);
            // the slot's next unit: the fold above consumed every lane's
            // reads of the slot, and the proxy fence orders them before the
            // bulk copy's writes
            __syncwarp();
            const int inext = i + D * NW;
            if (lane == 0 && inext < n) {
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(fb, (uint32_t)UB);
                bulk_g2s(ring + (size_t)(warp * D + k) * UB, W + (size_t)(u0 + inext) * UB, (uint32_t)UB, fb, pol);
            }
            s += dr;
            rb += dq;
            if (s >= units) { s -= units; ++rb; }
            k = k + 1 == D ? 0 : k + 1;
        }
        if (!wok) {
            // the warp's copies still in flight (at most D, from unit i on)
            // land before the slots are given up (bounded)
            for (int t = 0; t < D && i < n; ++t, i += NW) {
                if (mbar_wait_bounded(&P.slot[warp * ST_MAX_DEPTH + k], (spar >> k) & 1u, nullptr, 0))
                    spar ^= 1u << k;
                k = k + 1 == D ? 0 : k + 1;
            }
            ok = false;
        }
    } else {
        for (int ib = warp; ok && ib < n; ib += ST_RING * NW) {
#pragma unroll
            for (int k = 0; k < ST_RING; ++k) {
                const int i = ib + k * NW;
                if (i >= n) break;
                if (rb != cur_rb) {
                    red[((cur_rb - rb0) * NW + warp) * 32 + lane] = acc;
                    acc = 0.0f;
                    cur_rb = rb;
                }
                unit_dot<TYPE, ACT>(acc, ring_r[k], s * BLKS32, aq, ads, xs, xsum);
                const int inext = i + ST_RING * NW;
                if (inext < n) load_unit<TYPE>(ring_r[k], W + (size_t)(u0 + inext) * UB, lane);
                s += dr;
                rb += dq;
                if (s >= units) { s -= units; ++rb; }
            }
        }
    }
    if (warp < n) red[((cur_rb - rb0) * NW + warp) * 32 + lane] = acc;
    const bool cta_ok = __syncthreads_and(ok) != 0;
    for (int l = warp; cta_ok && l < nloc; l += NW) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) v += red[(l * NW + w) * 32 + lane];
        const int rbl = rb0 + l;
        if (epi == 2) {   // SwiGLU over rows interleaved by 16
            const float u = __shfl_down_sync(0xffffffffu, v, 16);
            const int r = rbl * 16 + lane;
            if (lane < 16 && r < (rows >> 1)) {
                const float y = (v / (1.0f + expf(-v))) * u;
                for (int c2 = 0; c2 < ncopy; ++c2) ll_st(ydst[c2] + yoff + r, y, ey);
            }
        } else {
            const int row = rbl * TILE_ROWS + lane;
            if (row < rows) {
                if (epi == 1) {
                    float r;
                    if (l == warp && ll_ok(rw, er)) r = ll_val(rw);
                    else ok = ll_get(residual + yoff + row, er, a.status, r) && ok;
                    v += r;
                }
                for (int c2 = 0; c2 < ncopy; ++c2) ll_st(ydst[c2] + yoff + row, v, ey);
            }
        }
    }
    // the slots and the reduction scratch are the next phase's
    return __syncthreads_and(ok) != 0;
}

// ---------------------------------------------------------------------------
// attention phase: one warp per (head, 64-position split); 8-lane groups
// hold 16 dims each, a warp folds four positions at a time
// ---------------------------------------------------------------------------
template <typename KV> __device__ __forceinline__ KV to_kv_st(float v);
template <> __device__ __forceinline__ float to_kv_st<float>(float v) { return v; }
template <> __device__ __forceinline__ __half to_kv_st<__half>(float v) { return __float2half_rn(v); }
__device__ __forceinline__ float kv_f(float v) { return v; }
__device__ __forceinline__ float kv_f(__half v) { return __half2float(v); }

// RoPE of the 16 dims a lane holds (dims 16*l8 ..), rounding as rope_rotate.
// Rotate-half: lanes l8 < 4 hold pair firsts (dims i), lanes l8 >= 4 the
// seconds (dims i + 64).  Adjacent pairs (2i, 2i+1) lie within the lane.
__device__ __forceinline__ void rope16(float (&v)[16], int l8, const StepPersist &P, int mode) {
    if (mode == HOLO_ROPE_ADJACENT) {
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            const float2 cs = P.rope[8 * l8 + j / 2];
            const float a = v[j], b = v[j + 1];
            v[j] = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
            v[j + 1] = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const float other = __shfl_xor_sync(0xffffffffu, v[j], 4);
        const int i = 16 * (l8 & 3) + j;
        const float c = P.rope[i].x, s = P.rope[i].y;
        if (l8 < 4) v[j] = __fsub_rn(__fmul_rn(v[j], c), __fmul_rn(other, s));
        else v[j] = __fadd_rn(__fmul_rn(other, s), __fmul_rn(v[j], c));
    }
}

// positions a CTA folds per iteration: 8 warps x 4 groups of 8 lanes
constexpr int ATT_SLOTS = LY_WARPS * 4;
// the CTA count the attention splits are sized for (one per SM of a B200)
constexpr int ATT_SPLIT_CTAS = 148;

// partial (m, l, acc[HD]) of one (head, split): header at 0, 1; acc at 4..
// (stride HD + 4 floats keeps every acc row 16-byte aligned)
constexpr int ATT_STRIDE = ST_HD + 4;

// raw K or V elements of one lane (16 dims) as loaded, converted when used
template <typename KV> struct KvRaw;
template <> struct KvRaw<__half> {
    uint4 r[2];
    __device__ __forceinline__ void load(const __half *p) {
        r[0] = *reinterpret_cast<const uint4 *>(p);
        r[1] = *reinterpret_cast<const uint4 *>(p + 8);
    }
    __device__ __forceinline__ float at(int j) const {
        const __half2 h2 = reinterpret_cast<const __half2 *>(&r[j >> 3])[(j & 7) >> 1];
        return (j & 1) ? __high2float(h2) : __low2float(h2);
    }
};
template <> struct KvRaw<float> {
    float4 r[4];
    __device__ __forceinline__ void load(const float *p) {
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] = *reinterpret_cast<const float4 *>(p + 4 * i);
    }
    __device__ __forceinline__ float at(int j) const {
        const float4 v = r[j >> 2];
        return (j & 3) == 0 ? v.x : (j & 3) == 1 ? v.y : (j & 3) == 2 ? v.z : v.w;
    }
};

// Attention of one position (llm.c:1173-1213 per head): an item is (local
// head h, split sp) and takes one CTA; its 32 position slots (warp w, group g)
// fold positions p0 + slot, p0 + 32 + slot, ... with an online softmax, the
// next position's K and V in flight while the current one is folded.  Groups
// merge by shuffles, warps through shared memory; with several splits the
// last CTA of a head (acq_rel counter) merges the split partials.  The
// current position's K and V come from the QKV output (rotated and rounded
// as the cache stores them); the head's first query head of its KV group
// also writes them to the cache.
// q, k, v: the LL QKV output of epoch eq; the output goes to every rank's
// attention vector with epoch eo.  False on a time-out.
template <typename KV>
__device__ __forceinline__ bool step_attn(const StepArgs &a, const StepPersist &P, uint8_t *sm, int layer, int pos,
                                       unsigned eq, unsigned eo) {
    constexpr int HD = ST_HD;
    const int kv_len = pos + 1, nh = a.n_heads;
    // A head's positions are cut into splits of whole slot iterations, about
    // ATT_SPLIT_CTAS / (all heads of the model) of them: a function of kv_len
    // and the model alone, so every world size (and grid) folds a head's
    // positions in the same splits and merges them in the same order -- a
    // sharded step's attention output is bit-identical to one GPU's.
    const int per_head = max(1, ATT_SPLIT_CTAS / a.n_heads_g);
    int per_split = (kv_len + per_head - 1) / per_head;
    per_split = (per_split + ATT_SLOTS - 1) / ATT_SLOTS * ATT_SLOTS;
    const int nsp = (kv_len + per_split - 1) / per_split;
    const int items = nh * nsp;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 3, l8 = lane & 7;
    const int slot = warp * 4 + g;
    const int q_dim = nh * HD, kv_dim = a.n_kv_heads * HD, group = nh / a.n_kv_heads;
    KV *kc = reinterpret_cast<KV *>(a.kc) + (size_t)layer * a.max_seq * kv_dim;
    KV *vc = reinterpret_cast<KV *>(a.vc) + (size_t)layer * a.max_seq * kv_dim;
    const float sqrt_hd = sqrtf((float)HD);
    float *wpart = reinterpret_cast<float *>(sm);                  // [LY_WARPS][ATT_STRIDE]
    for (int it = blockIdx.x; it < items; it += a.grid) {
        const int h = it % nh, sp = it / nh, kvh = h / group;
        const int p0 = sp * per_split, p1 = min(kv_len, p0 + per_split);
        // (waits are CTA-uniform: every warp leaves together on a time-out)
        float qf[16];
        if (!__syncthreads_and(ll_get16(a.qkv + (size_t)h * HD + 16 * l8, eq, a.status, qf))) return false;
        rope16(qf, l8, P, a.rope_mode);
        // the current position: its warp takes k and v from the QKV output,
        // rotated and rounded as the cache stores them, into shared memory
        const int pslot = (pos - p0) % ATT_SLOTS;
        const bool pos_warp = pos >= p0 && pos < p1 && pslot / 4 == warp;
        float *kps = wpart + LY_WARPS * ATT_STRIDE, *vps = kps + HD;
        {
            float kp[16], vp[16];
            bool got = true;
            if (pos_warp)
                got = ll_get16(a.qkv + q_dim + (size_t)kvh * HD + 16 * l8, eq, a.status, kp) &&
                      ll_get16(a.qkv + q_dim + kv_dim + (size_t)kvh * HD + 16 * l8, eq, a.status, vp);
            if (!__syncthreads_and(got)) return false;
            if (pos_warp) {
                rope16(kp, l8, P, a.rope_mode);
                if (g == pslot % 4) {
                    const bool writer = h % group == 0;   // one writer per KV head
                    KV *kd = kc + (size_t)pos * kv_dim + (size_t)kvh * HD + 16 * l8;
                    KV *vd = vc + (size_t)pos * kv_dim + (size_t)kvh * HD + 16 * l8;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const KV kq = to_kv_st<KV>(kp[j]), vq = to_kv_st<KV>(vp[j]);
                        kps[16 * l8 + j] = kv_f(kq);
                        vps[16 * l8 + j] = kv_f(vq);
                        if (writer) { kd[j] = kq; vd[j] = vq; }
                    }
                }
                __syncwarp();
            }
        }
        float m = -FLT_MAX, l = 0.0f, acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
        const size_t koff = (size_t)kvh * HD + 16 * l8;
        KvRaw<KV> kn, vn;   // the next position's, in flight
        int p = p0 + slot;
        if (p < p1 && p != pos) {
            kn.load(kc + (size_t)p * kv_dim + koff);
            vn.load(vc + (size_t)p * kv_dim + koff);
        }
        for (; p - slot < p1; p += ATT_SLOTS) {
            const bool live = p < p1, here = p == pos;
            const KvRaw<KV> kr = kn, vr = vn;
            const int pn = p + ATT_SLOTS;
            if (pn < p1 && pn != pos) {
                kn.load(kc + (size_t)pn * kv_dim + koff);
                vn.load(vc + (size_t)pn * kv_dim + koff);
            }
            float dot = 0.0f;
            if (live) {
#pragma unroll
                for (int j = 0; j < 16; ++j) dot = fmaf(qf[j], here ? kps[16 * l8 + j] : kr.at(j), dot);
            }
            dot += __shfl_xor_sync(0xffffffffu, dot, 1);
            dot += __shfl_xor_sync(0xffffffffu, dot, 2);
            dot += __shfl_xor_sync(0xffffffffu, dot, 4);
            if (live) {
                const float sc = __fdiv_rn(dot, sqrt_hd);     // score / sqrtf(hd), llm.c:1187
                const float mn = fmaxf(m, sc);
                const float corr = __expf(m - mn), e = __expf(sc - mn);
                l = fmaf(l, corr, e);
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[j] = fmaf(acc[j], corr, e * (here ? vps[16 * l8 + j] : vr.at(j)));
                m = mn;
            }
        }
        // the four groups of the warp
#pragma unroll
        for (int off = 8; off <= 16; off <<= 1) {
            const float om = __shfl_xor_sync(0xffffffffu, m, off), ol = __shfl_xor_sync(0xffffffffu, l, off);
            const float M = fmaxf(m, om);
            const float ca = l > 0.0f ? __expf(m - M) : 0.0f, cb = ol > 0.0f ? __expf(om - M) : 0.0f;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float oa = __shfl_xor_sync(0xffffffffu, acc[j], off);
                acc[j] = acc[j] * ca + oa * cb;
            }
            l = l * ca + ol * cb;
            m = M;
        }
        // the warps of the CTA: warp 0 merges, one float4 of dims a lane
        float *wp = wpart + warp * ATT_STRIDE;
        if (g == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<float4 *>(wp + 4 + 16 * l8 + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
        }
        if (lane == 0) { wp[0] = m; wp[1] = l; }
        __syncthreads();
        if (warp == 0) {
            float M = -FLT_MAX;
#pragma unroll
            for (int w = 0; w < LY_WARPS; ++w)
                if (wpart[w * ATT_STRIDE + 1] > 0.0f) M = fmaxf(M, wpart[w * ATT_STRIDE]);
            float L = 0.0f;
            float4 o4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int w = 0; w < LY_WARPS; ++w) {
                const float lw = wpart[w * ATT_STRIDE + 1];
                const float s = lw > 0.0f ? __expf(wpart[w * ATT_STRIDE] - M) : 0.0f;
                L = fmaf(lw, s, L);
                const float4 v = *reinterpret_cast<const float4 *>(wpart + w * ATT_STRIDE + 4 + 4 * lane);
                o4.x = fmaf(v.x, s, o4.x); o4.y = fmaf(v.y, s, o4.y);
                o4.z = fmaf(v.z, s, o4.z); o4.w = fmaf(v.w, s, o4.w);
            }
            bool out = nsp == 1;
            if (!out) {
                float *part = a.att_part + ((size_t)h * a.max_splits + sp) * ATT_STRIDE;
                reinterpret_cast<float4 *>(part + 4)[lane] = o4;
                if (lane == 0) { part[0] = M; part[1] = L; }
                __syncwarp();
                int last = 0;
                if (lane == 0) {
                    // acq_rel: publishes this split's partial, and the last
                    // arrival sees every other split's
                    int prev;
                    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(prev) : "l"(a.att_cnt + h) : "memory");
                    last = prev == nsp - 1;
                }
                out = __shfl_sync(0xffffffffu, last, 0);
                if (out) {
                    // the splits' partials, in split order (dec_attn_merge_kernel's arithmetic)
                    const float *ph = a.att_part + (size_t)h * a.max_splits * ATT_STRIDE;
                    M = -FLT_MAX;
                    for (int s0 = 0; s0 < nsp; s0 += 32) {
                        const int s2 = s0 + lane;
                        if (s2 < nsp) {
                            const float2 ml = __ldcg(reinterpret_cast<const float2 *>(ph + (size_t)s2 * ATT_STRIDE));
                            if (ml.y > 0.0f) M = fmaxf(M, ml.x);
                        }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
                    L = 0.0f;
                    o4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    for (int s0 = 0; s0 < nsp; s0 += 32) {
                        const int s2 = s0 + lane;
                        float w = 0.0f;
                        if (s2 < nsp) {
                            const float2 ml = __ldcg(reinterpret_cast<const float2 *>(ph + (size_t)s2 * ATT_STRIDE));
                            if (ml.y > 0.0f) { w = __expf(ml.x - M); L = fmaf(ml.y, w, L); }
                        }
                        const int n = min(32, nsp - s0);
#pragma unroll 8
                        for (int j = 0; j < n; ++j) {
                            const float wj = __shfl_sync(0xffffffffu, w, j);
                            const float4 v = __ldcg(reinterpret_cast<const float4 *>(ph + (size_t)(s0 + j) * ATT_STRIDE + 4) + lane);
                            o4.x = fmaf(v.x, wj, o4.x); o4.y = fmaf(v.y, wj, o4.y);
                            o4.z = fmaf(v.z, wj, o4.z); o4.w = fmaf(v.w, wj, o4.w);
                        }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
                    if (lane == 0) a.att_cnt[h] = 0;
                }
            }
            if (out) {
                const float inv = 1.0f / L;
                for (int c = 0; c < a.world; ++c) {
                    StepWord *dst = a.patt[c] + (size_t)(a.h0 + h) * HD + 4 * lane;
                    ll_st2(dst, o4.x * inv, o4.y * inv, eo);
                    ll_st2(dst + 2, o4.z * inv, o4.w * inv, eo);
                }
            }
        }
        __syncthreads();   // wpart is the next item's
    }
    return true;
}

// ---------------------------------------------------------------------------
// the kernels: the layers (embed + 5 phases per layer), then the output
// matrix and the sampler.  Two kernels because a second weight type in one
// kernel (a Q8_0 output matrix after Q4_K layers) doubles the live registers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool step_begin(const StepArgs &a, StepPersist &P, const unsigned long long *launches) {
    if (threadIdx.x == 0) {
        P.launch = ld_acquire_u64(launches);
        P.pos = __ldcg(a.pos);
        P.ok = __ldcg(a.status) == 0;
        mbar_init(&P.mbar, 1);
        for (int k = 0; k < MAX_WARPS * ST_MAX_DEPTH; ++k) mbar_init(&P.slot[k], 1);
        fence_barrier_init();
    }
    __syncthreads();
    return P.ok != 0;   // an earlier launch failed: do nothing
}

__device__ __forceinline__ void step_end(unsigned long long *launches, const StepPersist &P) {
    __syncthreads();
    if (blockIdx.x == 0 && threadIdx.x == 0) st_release_u64(launches, P.launch + 1);
}

template <int LT, int ACT, bool KVF16>
__global__ void __launch_bounds__(LY_THREADS, 1) dec_step_kernel(const StepArgs a) {
    using KV = typename std::conditional<KVF16, __half, float>::type;
    extern __shared__ __align__(128) uint8_t smem[];
    StepPersist &P = *reinterpret_cast<StepPersist *>(smem);
    uint8_t *sm = smem + ST_PERSIST;
    unsigned long long *launches = a.bar + 1;
    if (!step_begin(a, P, launches)) return;
    const int tid = threadIdx.x, pos = P.pos;
    const int q_dim = a.n_heads * ST_HD, kv_dim = a.n_kv_heads * ST_HD;
    if (tid < ST_HD / 2) {
        float c, s;
        rope_cos_sin(pos, tid, ST_HD, a.rope_base, c, s);
        P.rope[tid] = make_float2(c, s);
    }
    __syncthreads();
    unsigned mb_par = 0, spar = 0;
    StepWord *const x = a.px[a.rank];

    // embed: x = emb[seq[pos]] (every rank, whole vector, own copy)
    step_prefetch(a, 0);
    {
        const unsigned e0 = step_epoch(a, P.launch, 0);
        const int tok = __ldcg(a.seq + pos);
        for (int i = blockIdx.x * LY_THREADS + tid; i < a.dim; i += a.grid * LY_THREADS) {
            float v = 0.0f;
            if (tok >= 0 && tok < a.vocab)
                v = a.emb_f16 ? __half2float(reinterpret_cast<const __half *>(a.emb)[(size_t)tok * a.dim + i])
                              : reinterpret_cast<const float *>(a.emb)[(size_t)tok * a.dim + i];
            ll_st(x + i, v, e0);
        }
    }

    // layers: 5 phases each, one matvec call site; each phase polls its inputs
    const int last = 5 * a.n_layers;
    const size_t kv_es = KVF16 ? 2 : 4;
    for (int ph = 1; ph <= last; ++ph) {
        step_prefetch(a, ph);
        const int l = (ph - 1) / 5, k = (ph - 1) % 5;
        const unsigned ein = step_epoch(a, P.launch, ph - 1), eout = step_epoch(a, P.launch, ph);
        if (k == 0 && pos > 0 && tid < 32) {
            // the layer's cached K and V rows (positions 0..pos-1) into L2 for
            // the attention phase that follows
            const unsigned long long n = (unsigned long long)pos * kv_dim * kv_es;
            const unsigned long long c = blockIdx.x, G = a.grid, CH = 32768;
            const unsigned long long b0 = (n * c / G) & ~15ull, b1 = c + 1 == G ? n : ((n * (c + 1) / G) & ~15ull);
            const uint8_t *kb = reinterpret_cast<const uint8_t *>(a.kc) + (size_t)l * a.max_seq * kv_dim * kv_es;
            const uint8_t *vb = reinterpret_cast<const uint8_t *>(a.vc) + (size_t)l * a.max_seq * kv_dim * kv_es;
            for (unsigned long long o = b0 + (unsigned long long)tid * CH; o < b1; o += 32 * CH) {
                const uint32_t len = (uint32_t)(b1 - o < CH ? b1 - o : CH);
                prefetch_l2_bulk(kb + o, len);
                prefetch_l2_bulk(vb + o, len);
            }
        }
        bool ok;
        if (k == 1) {
            ok = step_attn<KV>(a, P, sm, l, pos, ein, eout);
            __syncthreads();   // the attention scratch is the next phase's
        } else {
            const StepLayer &L = a.layers[l];
            const uint8_t *W = k == 0 ? L.wqkv : k == 2 ? L.wo : k == 3 ? L.w13 : L.w2;
            // local rows: QKV of the local heads, a dim slice, a ffn slice (x2 interleaved)
            const int rows = k == 0 ? q_dim + 2 * kv_dim : k == 3 ? 2 * a.ffn_loc : a.dim_loc;
            const int in_dim = k == 2 ? a.n_heads_g * ST_HD : k == 4 ? a.ffn : a.dim;
            const StepWord *xin = k == 2 ? a.patt[a.rank] : k == 4 ? a.ph[a.rank] : x;
            StepWord *const *ydst = k == 0 ? &a.qkv : k == 3 ? a.ph : a.px;
            const int ncopy = k == 0 ? 1 : a.world;
            const int yoff = k == 0 ? 0 : k == 3 ? a.f0 : a.d0;
            // the residual x: written by the phase before the attention (Wo)
            // or by Wo (W2)
            const unsigned er = step_epoch(a, P.launch, k == 2 ? ph - 3 : ph - 2);
            const float *nw = k == 0 ? L.attn_norm : k == 3 ? L.ffn_norm : nullptr;
            const int epi = k == 3 ? 2 : (k == 2 || k == 4) ? 1 : 0;
            ok = step_mv<LT, ACT, LY_WARPS, false>(a, P, sm, mb_par, spar, W, rows, in_dim, xin, ein, ydst, ncopy, yoff, eout, x, er, nw,
                                  epi);
        }
        if (!__syncthreads_or(!ok)) continue;
        return;
    }
    step_end(launches, P);
}

// output matrix (RMSNorm fused; skipped for prompt positions of a
// generation), then on CTA 0 the logits gathered into the plain buffer, the
// sampler and the next position
template <int OT, int ACT>
__global__ void __launch_bounds__(OUT_THREADS, 1) dec_out_kernel(const StepArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    StepPersist &P = *reinterpret_cast<StepPersist *>(smem);
    uint8_t *sm = smem + ST_PERSIST;
    unsigned long long *launches = a.bar + 3;
    if (!step_begin(a, P, launches)) return;
    const int tid = threadIdx.x, pos = P.pos;
    unsigned mb_par = 0, spar = 0;
    const int ph = step_phases(a.n_layers) - 1;
    step_prefetch(a, ph);
    const unsigned ein = step_epoch(a, P.launch, ph - 1), eout = step_epoch(a, P.launch, ph);
    const bool need = !a.sa.gen || pos >= a.sa.n_prompt - 1;
    if (need && !step_mv<OT, ACT, OUT_WARPS, true>(a, P, sm, mb_par, spar, a.out_w, a.vocab_loc, a.dim, a.px[a.rank], ein, a.plog,
                                  a.world, a.v0, eout, nullptr, 0, a.final_norm, 0))
        return;
    if (blockIdx.x == 0) {
        if (need && !__syncthreads_and(ll_gather<OUT_THREADS>(a.logits, a.plog[a.rank], a.vocab, eout, a.status)))
            return;
        if (a.sample && need) {
            SampleSmem &S = *reinterpret_cast<SampleSmem *>(sm);
            const int gi = a.sa.gen ? pos - (a.sa.n_prompt - 1) : 0;
            const int nhist = __ldcg(a.nhist);
            const int token = sample_body(S, a.logits, a.probs, a.kept_idx, a.kept_p, a.hist, nhist,
                                          __ldcg(a.rvals + gi), a.status, a.sa);
            if (token >= 0 && tid == 0) {
                *a.last = token;
                if (a.sa.gen) {
                    a.seq[pos + 1] = token;
                    a.hist[nhist] = token;
                    *a.nhist = nhist + 1;
                    a.out_tokens[gi] = token;
                }
            }
        }
        if (tid == 0) *a.pos = pos + 1;
    }
    step_end(launches, P);
}

// shared memory of a matvec phase (the layout of step_mv) of nw warps with
// `depth` shared-memory slots a warp (0: the register ring)
size_t mv_smem(const StepArgs &a, int act, int type, int rows, int in_dim, bool norm, int nw, int depth) {
    const int vals = type == GT_Q8_0 ? 128 : 256, b32 = type == GT_Q8_0 ? 4 : 8;
    const size_t ub = type == GT_Q8_0 ? 4352 : 4608;
    const int units = (in_dim + vals - 1) / vals, nblk32p = units * b32;
    const int nrb = (rows + 31) / 32, nloc = (nrb + a.grid - 1) / a.grid;
    auto al = [](size_t v) { return (v + 127) & ~(size_t)127; };
    size_t o = (depth ? al((size_t)nw * depth * ub) : 0) + al((size_t)nloc * nw * 32 * 4);
    if (act == HOLO_ACT_Q8) o += al((size_t)nblk32p * 40) + (size_t)nblk32p * 128;
    else o += al((size_t)nblk32p * 132);
    if (norm) o += (size_t)nblk32p * 128;
    return o + nw * 4;
}

size_t layer_smem(const StepArgs &a, int lt, int act) {
    const int q_dim = a.n_heads * ST_HD, kv_dim = a.n_kv_heads * ST_HD;
    size_t m = mv_smem(a, act, lt, q_dim + 2 * kv_dim, a.dim, true, LY_WARPS, 0);
    m = std::max(m, mv_smem(a, act, lt, a.dim_loc, a.n_heads_g * ST_HD, false, LY_WARPS, 0));
    m = std::max(m, mv_smem(a, act, lt, 2 * a.ffn_loc, a.dim, true, LY_WARPS, 0));
    m = std::max(m, mv_smem(a, act, lt, a.dim_loc, a.ffn, false, LY_WARPS, 0));
    m = std::max(m, (size_t)(LY_WARPS * ATT_STRIDE + 2 * ST_HD) * sizeof(float));   // attention scratch
    return ST_PERSIST + m;
}

size_t out_smem(const StepArgs &a, int act, int depth) {
    size_t m = mv_smem(a, act, a.out_type, a.vocab_loc, a.dim, true, OUT_WARPS, depth);
    if (a.sample) m = std::max(m, sizeof(SampleSmem));
    return ST_PERSIST + m;
}

constexpr size_t ST_SMEM_MAX = 227 * 1024;

template <typename K>
bool coop_launch(K kern, const StepArgs &a, size_t smem, int threads, cudaStream_t st) {
    if (smem > ST_SMEM_MAX) {
        holo_set_status(HOLO_E_UNSUPPORTED, "decode step: shared memory");
        return false;
    }
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ST_SMEM_MAX) != cudaSuccess)
        return holo_check_launch("decode step: attributes");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;   // all CTAs resident: the grid barriers need it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, a) != cudaSuccess) return holo_check_launch("decode step launch");
    return holo_check_launch("decode step launch");
}

template <int LT>
bool launch_layers(const StepArgs &a, int act, int kv_f16, cudaStream_t st) {
    const size_t smem = layer_smem(a, LT, act);
    if (act == HOLO_ACT_Q8)
        return kv_f16 ? coop_launch(dec_step_kernel<LT, HOLO_ACT_Q8, true>, a, smem, LY_THREADS, st)
                      : coop_launch(dec_step_kernel<LT, HOLO_ACT_Q8, false>, a, smem, LY_THREADS, st);
    return kv_f16 ? coop_launch(dec_step_kernel<LT, HOLO_ACT_F32, true>, a, smem, LY_THREADS, st)
                  : coop_launch(dec_step_kernel<LT, HOLO_ACT_F32, false>, a, smem, LY_THREADS, st);
}

template <int OT>
bool launch_out(const StepArgs &args, int act, cudaStream_t st) {
    StepArgs a = args;
    // the deepest slot pipeline that fits
    a.mv_depth = 0;
    for (int d = ST_MAX_DEPTH; d >= 1 && a.mv_depth == 0; --d)
        if (out_smem(a, act, d) <= ST_SMEM_MAX) a.mv_depth = d;
    if (a.mv_depth == 0) {
        holo_set_status(HOLO_E_UNSUPPORTED, "decode step: shared memory");
        return false;
    }
    const size_t smem = out_smem(a, act, a.mv_depth);
    return act == HOLO_ACT_Q8 ? coop_launch(dec_out_kernel<OT, HOLO_ACT_Q8>, a, smem, OUT_THREADS, st)
                              : coop_launch(dec_out_kernel<OT, HOLO_ACT_F32>, a, smem, OUT_THREADS, st);
}

}  // namespace

bool holo_step_launch(const StepArgs &a, int layer_type, int act, int kv_f16, cudaStream_t st) {
    bool ok;
    switch (layer_type) {
    case GT_Q8_0: ok = launch_layers<GT_Q8_0>(a, act, kv_f16, st); break;
    case GT_Q4_0: ok = launch_layers<GT_Q4_0>(a, act, kv_f16, st); break;
    case GT_Q4_K: ok = launch_layers<GT_Q4_K>(a, act, kv_f16, st); break;
    default:
        holo_set_status(HOLO_E_ARG, "decode step: layer type");
        return false;
    }
    if (!ok) return false;
    switch (a.out_type) {
    case GT_Q8_0: return launch_out<GT_Q8_0>(a, act, st);
    case GT_Q4_0: return launch_out<GT_Q4_0>(a, act, st);
    case GT_Q4_K: return launch_out<GT_Q4_K>(a, act, st);
    default:
        holo_set_status(HOLO_E_ARG, "decode step: output type");
        return false;
    }
}
