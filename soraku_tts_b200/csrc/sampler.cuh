// Fused CFG + mask + temperature + top-k + top-p + draw for one request, run
// by one 256-thread CTA.  Restates soraku_inference/model.py:579-595 and
// _sample_logits (model.py:686-708) with an explicit Philox uniform in place
// of torch.multinomial:
//
//   merged = u + s * (c - u)                     (model.py:581; IEEE ops, no FMA)
//   BOS, PAD (and EOS when masked) -> -inf        (model.py:582-584)
//   temperature <= 0 -> first maximal index       (model.py:694-695)
//   f = merged / temperature (+0.0 folds -0 into +0)
//   top-k: cutoff = k-th largest f (duplicates counted); keep f >= cutoff
//   candidates ordered by (f descending, index ascending)
//   e_j = exp(f_j - f_0) with the exp below
//   top-p: S1 = sequential sum of e_j; cum = sequential sum of e_j / S1;
//          keep the prefix up to and including the first j with cum > p
//   draw: S2 = sequential sum of kept e_j; first kept j whose sequential
//         running sum of e_j exceeds u * S2 (else the last kept j with e_j > 0)
//
// Every float operation below rounds once, in the order written (explicit
// __f*_rn intrinsics stop the compiler from contracting), so the result is
// identical to the C restatement in the oracle for the same logits and u.
//
// Top-k selection: one 2048-bin histogram pass over the top 11 bits of an
// order-preserving integer key of the merged logit m finds the bin holding
// the k-th largest m (f = m / T is non-decreasing in m, so the top-k by f
// lies at or above it); every element at or above the bin below that one is
// divided by T, compacted (typically ~k + a few dozen) and rank-sorted
// exactly by (key of f, index).  With top-k off every element is a candidate
// (slow path, O(V^2 / 256) compares).
#pragma once

#include "common.cuh"

namespace skb {

constexpr int SAMPLER_THREADS = 256;
constexpr int SAMPLER_VMAX = 4096;
constexpr int SAMPLER_BINS = 2048;
constexpr int DEPTH_VMAX_SMALL = 2304;


// ---------------------------------------------------------------- exp
// Cody-Waite reduction + degree-7 Taylor polynomial (W. J. Cody and W. Waite,
// "Software Manual for the Elementary Functions", 1980); results below 2^-126
// flush to zero.  Same operations as orc_exp in the oracle.
__device__ __forceinline__ float skb_exp(float x) {
    const float LOG2E = 1.44269502162933349609375f;
    const float LN2_HI = 0.693145751953125f;
    const float LN2_LO = 1.428606765330187045e-06f;
    if (x != x) return x;
    if (x == -INFINITY) return 0.0f;
    if (x < -104.0f) return 0.0f;
    if (x > 88.7f) return INFINITY;
    const float t = __fmul_rn(x, LOG2E);
    const float n = rintf(t);
    float r = __fmaf_rn(-n, LN2_HI, x);
    r = __fmaf_rn(-n, LN2_LO, r);
    float p = 1.984126984126984e-04f;
    p = __fmaf_rn(p, r, 1.388888888888889e-03f);
    p = __fmaf_rn(p, r, 8.333333333333333e-03f);
    p = __fmaf_rn(p, r, 4.166666666666667e-02f);
    p = __fmaf_rn(p, r, 1.666666666666667e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = (int)n;
    if (ni < -126) return 0.0f;
    if (ni > 127) return INFINITY;
    const float scale = __int_as_float((ni + 127) << 23);
    const float y = __fmul_rn(p, scale);
    if (y < 1.17549435e-38f) return 0.0f;
    return y;
}

// -------------------------------------------------------------- philox
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11).
__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int round = 0; round < 10; ++round) {
        if (round > 0) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint32_t lo0 = 0xD2511F53u * c[0];
        const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]);
        const uint32_t lo1 = 0xCD9E8D57u * c[2];
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]);
        const uint32_t n0 = hi1 ^ c[1] ^ k0;
        const uint32_t n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0;
        c[1] = lo1;
        c[2] = n2;
        c[3] = lo0;
    }
}

__device__ __forceinline__ float philox_uniform(uint64_t seed, uint32_t request, uint32_t frame,
                                                uint32_t q) {
    uint32_t c[4] = {q, frame, request, 0u};
    philox4x32_10(c, (uint32_t)(seed & 0xffffffffu), (uint32_t)(seed >> 32));
    return __fmul_rn((float)(c[0] >> 8), 1.0f / 16777216.0f);
}

// Order-preserving key: a < b (as floats, no NaN) <=> key(a) < key(b).
__device__ __forceinline__ uint32_t ord_key(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct SampleJob {
    const float* cond;    // [V]
    const float* uncond;  // [V] or nullptr
    int V;
    float cfg_scale, temperature, top_p;
    int top_k, mask_eos, bos, pad, eos;
    float u;
    unsigned long long* ts;  // optional debug stage stamps (slots 6..11 of a kernel timeline)
};

// Block-wide exclusive scan of one int per thread (256 threads).
template <class Sync>
__device__ __forceinline__ int block_exclusive_scan(int v, int* tmp /* [8] */, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(FULL, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) tmp[warp] = x;
    Sync::sync();
    int wprefix = 0, tot = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const int t = tmp[w];
        if (w < warp) wprefix += t;
        tot += t;
    }
    Sync::sync();
    *total = tot;
    return wprefix + x - v;
}

// Shared memory a sampler with vocabulary capacity VMAX needs.
// [sorted keys: VMAX u64][candidates, then e and running sums: VMAX u64]
// [histogram][scalars][e / S1: VMAX floats]
template <int VMAX>
constexpr size_t sampler_smem_bytes() {
    return (size_t)VMAX * 20 + SAMPLER_BINS * 4 + 256;
}
constexpr size_t SAMPLER_SMEM = sampler_smem_bytes<SAMPLER_VMAX>();

// Returns the drawn code (same value in every thread).  smem:
// sampler_smem_bytes<VMAX>() bytes of shared memory, 16-byte aligned.
// Requires V <= VMAX and exactly 256 participating threads (0..255).
template <class Sync = BlockSync, int VMAX = SAMPLER_VMAX>
static __device__ int sample_one(const SampleJob& J, unsigned char* smem, int* n_kept_out = nullptr) {
    constexpr int NPT = (VMAX + SAMPLER_THREADS - 1) / SAMPLER_THREADS;  // logits per thread
    unsigned long long* sorted = reinterpret_cast<unsigned long long*>(smem);
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem + (size_t)VMAX * 8);
    float* e = reinterpret_cast<float*>(smem + (size_t)VMAX * 8);
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem + (size_t)VMAX * 16);
    int* sc = reinterpret_cast<int*>(smem + (size_t)VMAX * 16 + SAMPLER_BINS * 4);
    // sc[0..7] scan tmp, sc[8] count, sc[9] bin, sc[10] n_keep_topk, sc[11] keep, sc[12] pick,
    // sc[16..] reduction scratch
    float* scf = reinterpret_cast<float*>(sc + 16);

    const int tid = threadIdx.x;
    const int V = J.V;
    const bool greedy = !(J.temperature > 0.0f);

    // All of this thread's logits are requested before any is used (one L2
    // round trip, not one per element); f stays in registers.
    float cv[NPT], uv[NPT], fv[NPT];
#pragma unroll
    for (int k = 0; k < NPT; ++k) {
        const int i = tid + k * SAMPLER_THREADS;
        cv[k] = i < V ? __ldcg(J.cond + i) : 0.f;
        uv[k] = (i < V && J.uncond != nullptr) ? __ldcg(J.uncond + i) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < NPT; ++k) {
        const int i = tid + k * SAMPLER_THREADS;
        float m = cv[k];
        if (J.uncond != nullptr) m = __fadd_rn(uv[k], __fmul_rn(J.cfg_scale, __fsub_rn(cv[k], uv[k])));
        if (i == J.bos || i == J.pad || (J.mask_eos && i == J.eos) || i >= V) m = -INFINITY;
        fv[k] = m;  // merged logit; divided by the temperature once it is a candidate
    }

    if (tid == 0 && J.ts) stamp_max(J.ts + 6);
    if (greedy) {
        // first maximal index
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int k = 0; k < NPT; ++k) {
            const int i = tid + k * SAMPLER_THREADS;
            if (i < V && (fv[k] > bv || (fv[k] == bv && i < bi))) {
                bv = fv[k];
                bi = i;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(FULL, bv, o);
            const int oi = __shfl_xor_sync(FULL, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if ((tid & 31) == 0) {
            scf[tid >> 5] = bv;
            sc[8 + (tid >> 5) + 16] = bi;
        }
        Sync::sync();
        if (tid == 0) {
            float b = scf[0];
            int idx = sc[8 + 16];
            for (int w = 1; w < 8; ++w) {
                const float v = scf[w];
                const int ii = sc[8 + w + 16];
                if (v > b || (v == b && ii < idx)) {
                    b = v;
                    idx = ii;
                }
            }
            sc[12] = idx;
            sc[11] = 1;
        }
        Sync::sync();
        if (n_kept_out) *n_kept_out = 1;
        const int code = sc[12];
        Sync::sync();
        return code;
    }

    const bool topk_on = J.top_k > 0 && J.top_k < V;
    uint32_t low_key = 0;
    if (topk_on) {
        for (int b = tid; b < SAMPLER_BINS; b += SAMPLER_THREADS) hist[b] = 0;
        Sync::sync();
#pragma unroll
        for (int k = 0; k < NPT; ++k)
            if (tid + k * SAMPLER_THREADS < V) atomicAdd(&hist[ord_key(fv[k]) >> 21], 1u);
        Sync::sync();
        // (the histogram is over the merged logits m: f = m / T + 0 is
        // non-decreasing in m for T > 0, so the top-k by f lies in the bins
        // of m at or above the k-th largest m's bin -- up to a rounding tie
        // at the bin's lower edge, checked after the sort)
        // thread t owns descending bins 2047-8t .. 2040-8t
        int s = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) s += (int)hist[SAMPLER_BINS - 1 - (tid * 8 + j)];
        int total;
        const int before = block_exclusive_scan<Sync>(s, sc, &total);
        if (before < J.top_k && J.top_k <= before + s) {
            int acc = before;
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
                const int b = SAMPLER_BINS - 1 - (tid * 8 + j);
                const int h = (int)hist[b];
                if (acc + h >= J.top_k) {
                    sc[9] = b;
                    break;
                }
                acc += h;
            }
        }
        Sync::sync();
        low_key = (uint32_t)sc[9] << 21;
    }
    if (tid == 0 && J.ts) stamp_max(J.ts + 7);
    // compaction of every element at or above the cutoff bin (f = m / T is
    // formed only for these): slots come from a block scan of per-thread
    // counts, the exact rank sort by (key of f, -index) fixes the order.  If
    // the largest float below the bin, divided by T, could still reach the
    // k-th largest f (a rounding tie at the bin edge), the bin below is added
    // and the step repeats, so the top-k set is exact.
    int C = 0;
    for (int pass = 0; pass < 3; ++pass) {
        int mine = 0;
#pragma unroll
        for (int k = 0; k < NPT; ++k)
            mine += (tid + k * SAMPLER_THREADS < V && ord_key(fv[k]) >= low_key) ? 1 : 0;
        int slot = block_exclusive_scan<Sync>(mine, sc, &C);
        // (m, index) first; the divisions then run one per thread, not once
        // per loop slot in every warp that holds a candidate there
#pragma unroll
        for (int k = 0; k < NPT; ++k) {
            const int i = tid + k * SAMPLER_THREADS;
            if (i < V && ord_key(fv[k]) >= low_key)
                cand[slot++] = ((unsigned long long)__float_as_uint(fv[k]) << 32) |
                               (unsigned long long)(0xffffffffu - (uint32_t)i);
        }
        Sync::sync();
        for (int j = tid; j < C; j += SAMPLER_THREADS) {
            const unsigned long long c = cand[j];
            const float f = __fadd_rn(__fdiv_rn(__uint_as_float((uint32_t)(c >> 32)), J.temperature), 0.0f);
            cand[j] = ((unsigned long long)ord_key(f) << 32) | (c & 0xffffffffull);  // +0.0 folds -0 into +0
        }
        Sync::sync();
        // exact rank sort, descending by (key, -index)
        if (C & 1) {
            if (tid == 0) cand[C] = 0ull;  // pad to pairs: key 0 ranks below every candidate
            Sync::sync();
        }
        for (int i = tid; i < C; i += SAMPLER_THREADS) {
            const unsigned long long ki = cand[i];
            const ulonglong2* c2 = reinterpret_cast<const ulonglong2*>(cand);
            int rank = 0;
#pragma unroll 4
            for (int j = 0; j < (C + 1) / 2; ++j) {
                const ulonglong2 p = c2[j];
                rank += (p.x > ki) ? 1 : 0;
                rank += (p.y > ki) ? 1 : 0;
            }
            sorted[rank] = ki;
        }
        Sync::sync();
        if (!topk_on || low_key == 0) break;
        const float below = key_float(low_key - 1u);  // largest value below the bin
        const float bound = __fadd_rn(__fdiv_rn(below, J.temperature), 0.0f);
        const float cutoff = key_float((uint32_t)(sorted[J.top_k - 1] >> 32));
        if (bound < cutoff) break;  // no element below the bin can tie or pass the cutoff
        // one bin lower (quarter of an octave); a third pass takes every element
        low_key = (pass == 0 && low_key >= (1u << 21)) ? low_key - (1u << 21) : 0u;
    }
    if (tid == 0 && J.ts) stamp_max(J.ts + 8);
    // top-k: keep the sorted prefix with f >= cutoff (ties kept); its end is the
    // one position where f >= cutoff is followed by f < cutoff (or the end)
    int n = C;
    if (topk_on) {
        const float cutoff = key_float((uint32_t)(sorted[J.top_k - 1] >> 32));
        for (int i = tid; i < C; i += SAMPLER_THREADS) {
            const bool in = !(key_float((uint32_t)(sorted[i] >> 32)) < cutoff);
            const bool next_out = (i + 1 == C) || (key_float((uint32_t)(sorted[i + 1] >> 32)) < cutoff);
            if (in && next_out) sc[10] = i + 1;
        }
        Sync::sync();
        n = sc[10];
    }
    // e_j, zero-padded to a multiple of 32 (adding +0 to a running sum of
    // non-negative terms changes nothing, so the sequential passes below run
    // whole 32-element chunks without per-element tests)
    const int npad = (n + 31) & ~31;
    const float top = key_float((uint32_t)(sorted[0] >> 32));
    for (int j = tid; j < npad; j += SAMPLER_THREADS)
        e[j] = j < n ? skb_exp(__fsub_rn(key_float((uint32_t)(sorted[j] >> 32)), top)) : 0.0f;
    Sync::sync();
    if (tid == 0 && J.ts) stamp_max(J.ts + 9);
    // Sequential FP32 sums in candidate order, as the oracle does.  One pass
    // (thread 0) forms the running sums P_j = e_0 + ... + e_j in order: the
    // oracle's S1 is P_{n-1}, its S2 is P_{keep-1} and its draw compares the
    // same running sums, so those need no pass of their own.  Each chunk's 32
    // terms are loaded first, then added as one dependent chain.
    float* P = e + VMAX;  // running sums
    if (tid == 0) {
        float run = 0.0f;
        for (int j0 = 0; j0 < npad; j0 += 32) {
            float v[32];
#pragma unroll
            for (int t = 0; t < 32; t += 4) {
                const float4 q = *reinterpret_cast<const float4*>(e + j0 + t);
                v[t] = q.x;
                v[t + 1] = q.y;
                v[t + 2] = q.z;
                v[t + 3] = q.w;
            }
#pragma unroll
            for (int t = 0; t < 32; ++t) {
                run = __fadd_rn(run, v[t]);
                v[t] = run;
            }
#pragma unroll
            for (int t = 0; t < 32; t += 4)
                *reinterpret_cast<float4*>(P + j0 + t) = make_float4(v[t], v[t + 1], v[t + 2], v[t + 3]);
        }
        sc[11] = n;
    }
    Sync::sync();
    const bool topp_on = J.top_p > 0.0f && J.top_p < 1.0f;
    if (topp_on) {
        const float s1 = P[n - 1];
        // e_j / S1 in parallel (zero-padded), then its sequential running sum
        // (thread 0); the prefix is kept up to and including the first j with
        // cum > p
        float* pj = reinterpret_cast<float*>(smem + (size_t)VMAX * 16 + SAMPLER_BINS * 4 + 256);
        for (int j = tid; j < npad; j += SAMPLER_THREADS) pj[j] = j < n ? __fdiv_rn(e[j], s1) : 0.0f;
        Sync::sync();
        if (tid == 0) {
            int keep = n;
            float cum = 0.0f;
            for (int j0 = 0; j0 < npad && keep == n; j0 += 32) {
                float v[32];
#pragma unroll
                for (int t = 0; t < 32; t += 4) {
                    const float4 q = *reinterpret_cast<const float4*>(pj + j0 + t);
                    v[t] = q.x;
                    v[t + 1] = q.y;
                    v[t + 2] = q.z;
                    v[t + 3] = q.w;
                }
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    cum = __fadd_rn(cum, v[t]);
                    v[t] = cum;
                }
                // cum is non-decreasing: the first crossing is the number of
                // chunk entries not above p
                int below = 0;
#pragma unroll
                for (int t = 0; t < 32; ++t) below += (v[t] > J.top_p) ? 0 : 1;
                if (below < 32 && j0 + below < n) keep = j0 + below + 1;
            }
            sc[11] = keep;
        }
        Sync::sync();
    }
    // draw: t = u * S2; the first kept j whose running sum exceeds t (else the
    // last kept j with e_j > 0), found by a block-wide minimum / maximum
    {
        const int keep = sc[11];
        const float t = __fmul_rn(J.u, P[keep - 1]);
        int first = 0x7fffffff, lastpos = -1;
        for (int j = tid; j < keep; j += SAMPLER_THREADS) {
            if (P[j] > t && j < first) first = j;
            if (e[j] > 0.0f) lastpos = j;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            first = min(first, __shfl_xor_sync(FULL, first, o));
            lastpos = max(lastpos, __shfl_xor_sync(FULL, lastpos, o));
        }
        if ((tid & 31) == 0) {
            sc[16 + (tid >> 5)] = first;
            sc[24 + (tid >> 5)] = lastpos;
        }
        Sync::sync();
        if (tid == 0) {
            int f = 0x7fffffff, lp = -1;
            for (int w = 0; w < SAMPLER_THREADS / 32; ++w) {
                f = min(f, sc[16 + w]);
                lp = max(lp, sc[24 + w]);
            }
            const int pick = f != 0x7fffffff ? f : (lp >= 0 ? lp : 0);
            sc[12] = (int)(0xffffffffu - (uint32_t)(sorted[pick] & 0xffffffffull));
        }
    }
    Sync::sync();
    if (n_kept_out) *n_kept_out = sc[11];
    const int code = sc[12];
    Sync::sync();
    return code;
}

}  // namespace skb
