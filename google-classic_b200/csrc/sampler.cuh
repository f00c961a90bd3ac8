// sampler.cuh -- the device sampler (llm_sample, src/ai/llm.c:1281-1328 and
// src/ai/tensor.c:460-667), run by one CTA: shared by the graph step
// (decode.cu) and the persistent step kernel (step.cu).
#pragma once
#include "holo_common.cuh"

#include <cfloat>

namespace holo_dec {

// ---------------------------------------------------------------------------
// sampler: llm_sample (llm.c:1281-1328) on the device, one 1024-thread CTA.
//  1. temperature: logits *= 1/T when T > 0 and T != 1 (tensor.c:636-642)
//  2. repetition penalty over the last repeat_last_n history tokens, once per
//     occurrence: /= penalty if positive, *= penalty otherwise (tensor.c:644-657)
//  3. greedy (T == 0): the first index of the largest penalised logit
//  4. softmax; 5. top-k (keep p >= the k-th largest p, renormalise);
//  6. top-p (sort descending, keep through the first cumulative sum > p,
//     renormalise); 7. draw: first index whose cumulative sum exceeds r.
// The sums of the renormalisations and the draw run in the reference's order
// (index order; descending order for top-p).  Two steps differ in rounding
// only: exp is evaluated in double and rounded once, and the softmax
// denominator is summed as a tree.
// ---------------------------------------------------------------------------
constexpr int SM_THREADS = 1024;
constexpr int SM_SORT_MAX = 4096;           // top-p candidates sorted in shared memory
constexpr int SM_VOCAB_SMEM = 36864;        // vocabularies up to this size are sampled in shared memory

struct SampleArgs {
    int vocab;
    int use_temp;          // T > 0 and T != 1
    float tscale;          // 1/T
    int greedy;            // T == 0
    float penalty;
    int last_n;
    int top_k;
    float top_p;
    int gen;               // 1: generation step (skip during the prompt, append the token)
    int n_prompt;
};

__device__ __forceinline__ void block_reduce_max_first(float &v, int &idx, float *sv, int *si) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
    }
    if (lane == 0) { sv[warp] = v; si[warp] = idx; }
    __syncthreads();
    if (warp == 0) {
        v = lane < (int)(blockDim.x >> 5) ? sv[lane] : -FLT_MAX;
        idx = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
        }
        if (lane == 0) { sv[0] = v; si[0] = idx; }
    }
    __syncthreads();
    v = sv[0];
    idx = si[0];
    __syncthreads();
}

__device__ __forceinline__ float block_sum(float v, float *sv) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sv[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (int)(blockDim.x >> 5) ? sv[lane] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) sv[0] = v;
    }
    __syncthreads();
    v = sv[0];
    __syncthreads();
    return v;
}

// Shared state of the sampler (static shared memory of the kernel that runs it).
struct SampleSmem {
    int ncand;
    float sv[32];
    int si[32];
    unsigned hist256[256];
    unsigned prefix;
    int krem;
    float scale;
    int ncut;
    int token;
    float cand_p[SM_SORT_MAX];   // candidates (index order), then the top-p sort
    int cand_i[SM_SORT_MAX];
    float sort_p[SM_SORT_MAX];   // also the per-warp digit histograms of the top-k selection
    int sort_j[SM_SORT_MAX];
    float work[SM_VOCAB_SMEM];   // the logits, then the probabilities (small vocabularies)
};
// per-warp histograms of the radix selection: 32 warps x 256 digits
static_assert(2 * SM_SORT_MAX >= 32 * 256, "digit histograms fit the sort buffers");

// a slot in a shared list for each lane with pred (one atomic a warp); the
// whole warp calls it; -1 for the others
__device__ __forceinline__ int warp_slot(int *counter, bool pred) {
    const unsigned bal = __ballot_sync(0xffffffffu, pred);
    if (!bal) return -1;
    const int lane = threadIdx.x & 31;
    int base = 0;
    if (lane == __ffs(bal) - 1) base = atomicAdd(counter, __popc(bal));
    base = __shfl_sync(0xffffffffu, base, __ffs(bal) - 1);
    return pred ? base + __popc(bal & ((1u << lane) - 1u)) : -1;
}

// warp 0: the digit at `shift` of the k-th largest key among those counted in
// S.hist256 (keys matching S.prefix so far); updates S.prefix and S.krem
// (out of line: the sampler runs once a launch, so each inlined copy of its
// code would be fetched cold into the instruction cache)
static __device__ __noinline__ void radix_digit(SampleSmem &S, int shift, int lane) {
    // lane l owns digits 255-8l .. 248-8l (descending); find the digit where
    // the count of larger-or-equal digits reaches krem
    unsigned cnt[8], tot = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) { cnt[k] = S.hist256[255 - 8 * lane - k]; tot += cnt[k]; }
    unsigned incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    const int krem = S.krem;
    const unsigned before = incl - tot;
    if ((int)before < krem && (int)incl >= krem) {
        unsigned cum = before;
        for (int k = 0; k < 8; ++k) {
            if ((int)(cum + cnt[k]) >= krem) {
                S.prefix |= (unsigned)(255 - 8 * lane - k) << shift;
                S.krem = krem - (int)cum;
                break;
            }
            cum += cnt[k];
        }
    }
}


// The sampler body, run by one CTA of any size (a multiple of 32, <= 1024).
// The logits are copied into a work array -- shared memory for vocabularies
// up to SM_VOCAB_SMEM, else the global `probs` buffer -- and every step runs
// there; the logits themselves are left as they are.  Candidates (the top-k
// set, or every index when top-k is off) live in shared memory when they fit,
// so the reference's sequential sums read shared memory.  Returns the token
// (all threads), -1 when top-p needs more candidates than fit.
static __device__ int sample_body(SampleSmem &S, const float *__restrict__ logits, float *__restrict__ probs,
                           int *__restrict__ kept_idx, float *__restrict__ kept_p, const int *__restrict__ hist,
                           int nhist, float r, int *__restrict__ status, const SampleArgs &a) {
    const int V = a.vocab, tid = threadIdx.x, NT = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5;
    float *work = V <= SM_VOCAB_SMEM ? S.work : probs;
    // 1. copy (eight loads in flight per thread) with the temperature applied
    //    (logits * (1/T) when T > 0 and T != 1, tensor.c:636-642)
    {
        const float ts = a.use_temp ? a.tscale : 1.0f;
        for (int i0 = 0; i0 < V; i0 += 8 * NT) {
            float v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int i = i0 + k * NT + tid;
                v[k] = i < V ? __ldcg(logits + i) : 0.0f;   // written by other CTAs: bypass L1
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int i = i0 + k * NT + tid;
                if (i < V) work[i] = a.use_temp ? v[k] * ts : v[k];
            }
        }
    }
    __syncthreads();
    // 2. repetition penalty, once per occurrence (tensor.c:644-657).  Applying
    //    the same operation c times does not depend on the order of the
    //    occurrences, so the first occurrence of each token applies all c.
    if (a.penalty != 1.0f && nhist > 0) {
        const int start = nhist > a.last_n ? nhist - a.last_n : 0;
        // the window of the history in shared memory (cand_i is free here)
        const bool staged = nhist - start <= SM_SORT_MAX;
        const int *hw = staged ? S.cand_i : hist + start;
        if (staged) {
            for (int t = tid; t < nhist - start; t += NT) S.cand_i[t] = __ldcg(hist + start + t);
            __syncthreads();
        }
        for (int t = start + tid; t < nhist; t += NT) {
            const int tok = staged ? hw[t - start] : __ldcg(hw + (t - start));
            // occurrences of tok in the window (itself included), and whether
            // this is the first; no early exit, so the loop pipelines
            bool first = true;
            int c = 0;
            if (staged) {
#pragma unroll 8
                for (int u = 0; u < nhist - start; ++u) {
                    const bool eq = hw[u] == tok;
                    c += eq;
                    first = first && !(eq && u < t - start);
                }
            } else {
                for (int u = 0; u < nhist - start; ++u) {
                    const bool eq = __ldcg(hw + u) == tok;
                    c += eq;
                    first = first && !(eq && u < t - start);
                }
            }
            if (first && tok >= 0 && tok < V) {
                float v = work[tok];
                for (int k = 0; k < c; ++k) v = v > 0.0f ? __fdiv_rn(v, a.penalty) : v * a.penalty;
                work[tok] = v;
            }
        }
        __syncthreads();
    }
    // every pass over the vocabulary is strided (coalesced); where the
    // reference's index order matters, candidates are put back in index order
    if (a.greedy) {
        float bv = -FLT_MAX;
        int bi = 0x7fffffff;
        for (int i = tid; i < V; i += NT)
            if (work[i] > bv || bi == 0x7fffffff) { bv = work[i]; bi = i; }
        block_reduce_max_first(bv, bi, S.sv, S.si);
        return bi;
    }
    // 4. softmax
    float mx = -FLT_MAX;
    int mi = 0;
    for (int i = tid; i < V; i += NT) mx = fmaxf(mx, work[i]);
    block_reduce_max_first(mx, mi, S.sv, S.si);
    float part = 0.0f;
    for (int i = tid; i < V; i += NT) {
        const float e = (float)exp((double)(work[i] - mx));
        work[i] = e;
        part += e;
    }
    const float sum_e = block_sum(part, S.sv);
    const float scale = __fdiv_rn(1.0f, sum_e);

    // 5. top-k: the k-th largest probability by radix selection on its bits
    //    (probabilities are >= 0, so their bit patterns order like the
    //    values).  Digit counts go to one histogram per warp (most
    //    probabilities share a few exponents: one histogram would serialise
    //    the CTA's atomics on one or two bins), summed per digit afterwards.
    //    The first digit is counted in the pass that scales the
    //    probabilities; then the keys at or above the selected top byte --
    //    the candidates and the rest of the boundary byte, usually a few
    //    hundred -- are compacted, and the later digits are counted over
    //    them alone.  A boundary byte too crowded to compact falls back to
    //    passes over the vocabulary.
    float thr = 0.0f;
    const bool topk = a.top_k > 0 && a.top_k < V;
    unsigned *wh = reinterpret_cast<unsigned *>(S.sort_p);   // [warps][256]
    const int nw = NT >> 5;
    if (topk) {
        for (int b = tid; b < nw * 256; b += NT) wh[b] = 0u;
        if (tid == 0) { S.prefix = 0u; S.krem = a.top_k; S.ncut = 0; S.ncand = 0; }
        __syncthreads();
    }
    {
        unsigned *mine = wh + warp * 256;
        for (int i = tid; i < V; i += NT) {
            const float p = work[i] * scale;
            work[i] = p;
            if (topk) atomicAdd(&mine[__float_as_uint(p) >> 24], 1u);
        }
        __syncthreads();
    }
    bool have_cands = false;   // candidates already collected (compacted path)
    if (topk) {
        for (int b = tid; b < 256; b += NT) {
            unsigned c = 0u;
            for (int w = 0; w < nw; ++w) c += wh[w * 256 + b];
            S.hist256[b] = c;
        }
        __syncthreads();
        if (warp == 0) radix_digit(S, 24, lane);
        __syncthreads();
        // compact the keys whose top byte is at least the selected one
        const unsigned top = S.prefix >> 24;
        for (int i0 = 0; i0 < V; i0 += NT) {
            const int i = i0 + tid;
            const float p = i < V ? work[i] : 0.0f;
            const int slot = warp_slot(&S.ncut, i < V && (__float_as_uint(p) >> 24) >= top);
            if (slot >= 0 && slot < SM_SORT_MAX) { S.sort_p[slot] = p; S.sort_j[slot] = i; }
        }
        __syncthreads();
        const int nc = S.ncut;
        unsigned mask = 0xFF000000u;
        if (nc <= SM_SORT_MAX) {
            for (int shift = 16; shift >= 0; shift -= 8) {
                for (int b = tid; b < 256; b += NT) S.hist256[b] = 0u;
                __syncthreads();
                const unsigned prefix = S.prefix;
                for (int j = tid; j < nc; j += NT) {
                    const unsigned key = __float_as_uint(S.sort_p[j]);
                    if ((key & mask) == prefix) atomicAdd(&S.hist256[(key >> shift) & 255u], 1u);
                }
                __syncthreads();
                if (warp == 0) radix_digit(S, shift, lane);
                mask |= 255u << shift;
                __syncthreads();
            }
            thr = __uint_as_float(S.prefix);
            // the candidates: the compacted keys at or above the threshold
            for (int j0 = 0; j0 < nc; j0 += NT) {
                const int j = j0 + tid;
                const float p = j < nc ? S.sort_p[j] : 0.0f;
                const int slot = warp_slot(&S.ncand, j < nc && p >= thr);
                if (slot >= 0) {
                    S.cand_i[slot] = S.sort_j[j];
                    S.cand_p[slot] = p;
                }
            }
            __syncthreads();
            have_cands = true;
        } else {
            for (int shift = 16; shift >= 0; shift -= 8) {
                for (int b = tid; b < nw * 256; b += NT) wh[b] = 0u;
                __syncthreads();
                const unsigned prefix = S.prefix;
                unsigned *mine = wh + warp * 256;
                for (int i = tid; i < V; i += NT) {
                    const unsigned key = __float_as_uint(work[i]);
                    if ((key & mask) == prefix) atomicAdd(&mine[(key >> shift) & 255u], 1u);
                }
                __syncthreads();
                for (int b = tid; b < 256; b += NT) {
                    unsigned c = 0u;
                    for (int w = 0; w < nw; ++w) c += wh[w * 256 + b];
                    S.hist256[b] = c;
                }
                __syncthreads();
                if (warp == 0) radix_digit(S, shift, lane);
                mask |= 255u << shift;
                __syncthreads();
            }
            thr = __uint_as_float(S.prefix);
        }
    }
    // candidates (p >= thr; every index without top-k), in index order
    if (!have_cands) {
        if (tid == 0) S.ncand = 0;
        __syncthreads();
        for (int i0 = 0; i0 < V; i0 += NT) {
            const int i = i0 + tid;
            const float p = i < V ? work[i] : 0.0f;
            const int slot = warp_slot(&S.ncand, i < V && p >= thr);
            if (slot >= 0 && slot < SM_SORT_MAX) { S.cand_i[slot] = i; S.cand_p[slot] = p; }
        }
        __syncthreads();
    }
    const int nk = S.ncand;
    if (nk <= 64) {
        // a few candidates (top-k): warp 0 finishes alone.  Orders come from
        // ranks (a pass over the candidates in shared memory, broadcast
        // reads), not sorting networks: candidate e (lanes e and e-32) has
        // index rank ri and, after the top-k renormalisation, rank rp in
        // (descending p, ascending index) order.
        if (warp == 0) {
            float *ap = S.sort_p, *bp = S.cand_p;   // by index rank, by p rank
            int *ai = S.sort_j;
            float p[2];
            int ix[2], ri[2] = {0, 0}, rp[2] = {0, 0};
            bool live[2];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int e = lane + 32 * q;
                live[q] = e < nk;
                p[q] = live[q] ? S.cand_p[e] : 0.0f;
                ix[q] = live[q] ? S.cand_i[e] : 0x7fffffff;
            }
            for (int j = 0; j < nk; ++j) {
                const int ij = S.cand_i[j];
#pragma unroll
                for (int q = 0; q < 2; ++q) ri[q] += ij < ix[q];
            }
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 2; ++q)
                if (live[q]) { ap[ri[q]] = p[q]; ai[ri[q]] = ix[q]; }
            __syncwarp();
            if (topk) {   // renormalise: sequential sum in index order
                float sc = 0.0f;
                if (lane == 0) {
                    float sum = 0.0f;
                    for (int j = 0; j < nk; ++j) sum += ap[j];
                    sc = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 1.0f;
                }
                sc = __shfl_sync(0xffffffffu, sc, 0);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    p[q] = p[q] * sc;
                    if (live[q]) ap[ri[q]] = p[q];
                }
                __syncwarp();
            }
            if (a.top_p > 0.0f && a.top_p < 1.0f) {
                // cut at the first cumulative sum above top_p in descending
                // order (ties: lower index first), renormalise
                for (int j = 0; j < nk; ++j) {
                    const float pj = ap[j];
#pragma unroll
                    for (int q = 0; q < 2; ++q) rp[q] += pj > p[q] || (pj == p[q] && j < ri[q]);
                }
#pragma unroll
                for (int q = 0; q < 2; ++q)
                    if (live[q]) bp[rp[q]] = p[q];
                __syncwarp();
                int cut = nk;
                if (lane == 0) {
                    float cum = 0.0f;
                    for (int j = 0; j < nk; ++j) {
                        cum += bp[j];
                        if (cum > a.top_p) { cut = j + 1; break; }
                    }
                }
                cut = __shfl_sync(0xffffffffu, cut, 0);
#pragma unroll
                for (int q = 0; q < 2; ++q)
                    if (live[q] && rp[q] >= cut) { p[q] = 0.0f; ap[ri[q]] = 0.0f; }
                __syncwarp();
                float sc = 0.0f;
                if (lane == 0) {
                    float sum = 0.0f;
                    for (int j = 0; j < nk; ++j) sum += ap[j];
                    sc = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 1.0f;
                }
                sc = __shfl_sync(0xffffffffu, sc, 0);
#pragma unroll
                for (int q = 0; q < 2; ++q)
                    if (live[q]) ap[ri[q]] = p[q] * sc;
                __syncwarp();
            }
            // 7. draw over the candidates in index order
            if (lane == 0) {
                float cum = 0.0f;
                int tok = V - 1;
                for (int j = 0; j < nk; ++j) {
                    cum += ap[j];
                    if (r < cum) { tok = ai[j]; break; }
                }
                S.token = tok;
            }
        }
        __syncthreads();
        return S.token;
    }
    const bool in_smem = nk <= SM_SORT_MAX;
    float *cp = S.cand_p;
    int *ci = S.cand_i;
    if (in_smem) {
        // bitonic sort of the candidates by index
        int n2 = 1;
        while (n2 < nk) n2 <<= 1;
        for (int j = nk + tid; j < n2; j += NT) { ci[j] = 0x7fffffff; cp[j] = 0.0f; }
        __syncthreads();
        for (int k = 2; k <= n2; k <<= 1)
            for (int jj = k >> 1; jj > 0; jj >>= 1) {
                for (int t = tid; t < n2; t += NT) {
                    const int u = t ^ jj;
                    if (u > t) {
                        const bool up = (t & k) == 0;
                        const int it = ci[t], iu = ci[u];
                        if (up ? it > iu : it < iu) {
                            ci[t] = iu; ci[u] = it;
                            const float pt = cp[t];
                            cp[t] = cp[u]; cp[u] = pt;
                        }
                    }
                }
                __syncthreads();
            }
    } else {
        // more candidates than shared memory holds (top-k off): ordered
        // compaction into global memory, NT indices at a time
        cp = kept_p;
        ci = kept_idx;
        int base = 0;
        for (int k0 = 0; k0 < V; k0 += NT) {
            const int i = k0 + tid;
            const bool pred = i < V && work[i] >= thr;
            const unsigned bal = __ballot_sync(0xffffffffu, pred);
            if (lane == 0) S.si[warp] = __popc(bal);
            __syncthreads();
            int woff = 0, tot = 0;
            for (int w = 0; w < (NT >> 5); ++w) {
                if (w < warp) woff += S.si[w];
                tot += S.si[w];
            }
            if (pred) {
                const int o = base + woff + __popc(bal & ((1u << lane) - 1u));
                ci[o] = i;
                cp[o] = work[i];
            }
            base += tot;
            __syncthreads();
        }
    }
    __syncthreads();
    if (topk) {
        if (tid == 0) {
            float sum = 0.0f;
            for (int j = 0; j < nk; ++j) sum += cp[j];
            S.scale = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 1.0f;
        }
        __syncthreads();
        for (int j = tid; j < nk; j += NT) cp[j] = cp[j] * S.scale;
        __syncthreads();
    }

    // 6. top-p over the candidates, sorted descending in shared memory
    if (a.top_p > 0.0f && a.top_p < 1.0f) {
        if (nk > SM_SORT_MAX) {
            if (tid == 0) atomicExch(status, HOLO_E_UNSUPPORTED);
            return -1;
        }
        int n2 = 1;
        while (n2 < nk) n2 <<= 1;
        for (int j = tid; j < n2; j += NT) {
            S.sort_p[j] = j < nk ? cp[j] : -1.0f;
            S.sort_j[j] = j < nk ? j : 0x7fffffff;
        }
        __syncthreads();
        // bitonic sort: descending probability, ties by ascending candidate
        for (int k = 2; k <= n2; k <<= 1) {
            for (int jj = k >> 1; jj > 0; jj >>= 1) {
                for (int t = tid; t < n2; t += NT) {
                    const int u = t ^ jj;
                    if (u > t) {
                        const bool desc = (t & k) == 0;
                        const float pt = S.sort_p[t], pu = S.sort_p[u];
                        const int it = S.sort_j[t], iu = S.sort_j[u];
                        const bool t_first = pt > pu || (pt == pu && it < iu);
                        if (desc ? !t_first : t_first) {
                            S.sort_p[t] = pu; S.sort_p[u] = pt;
                            S.sort_j[t] = iu; S.sort_j[u] = it;
                        }
                    }
                }
                __syncthreads();
            }
        }
        if (tid == 0) {
            float cum = 0.0f;
            int cut = nk;
            for (int j = 0; j < nk; ++j) {
                cum += S.sort_p[j];
                if (cum > a.top_p) { cut = j + 1; break; }
            }
            S.ncut = cut;
        }
        __syncthreads();
        for (int j = tid; j < nk; j += NT)
            if (j >= S.ncut) cp[S.sort_j[j]] = 0.0f;
        __syncthreads();
        if (tid == 0) {
            float sum = 0.0f;
            for (int j = 0; j < nk; ++j) sum += cp[j];
            S.scale = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 1.0f;
        }
        __syncthreads();
        for (int j = tid; j < nk; j += NT) cp[j] = cp[j] * S.scale;
        __syncthreads();
    }

    // 7. draw (sample_prob, tensor.c:473-482) over the candidates in index order
    if (tid == 0) {
        float cum = 0.0f;
        int tok = V - 1;
        for (int j = 0; j < nk; ++j) {
            cum += cp[j];
            if (r < cum) { tok = ci[j]; break; }
        }
        S.token = tok;
    }
    __syncthreads();
    return S.token;
}

}  // namespace holo_dec
