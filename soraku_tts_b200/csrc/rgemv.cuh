// Ring-streamed FP32 decode GEMV: out[m, u] = epilogue(sum_k xn[m, k] * W[row(u), k])
// for M <= 4 activation rows, W row-major [N, K] (nn.Linear layout).
//
// One CTA is 8 consumer warps + 1 producer warp.  CTA c owns the contiguous
// units [c*NU/G, (c+1)*NU/G); a unit is one output row, or for SwiGLU one
// (gate row i, up row i) pair.  Lane 0 of the producer warp streams the
// slice's weight rows through a ring of shared-memory slots with 1-D bulk
// copies (TMA engine, no tensor map, no multicast), one full/empty mbarrier
// pair per slot.  Weights never depend on an earlier kernel, so the first
// ring-full of copies is issued before the programmatic-dependent-launch wait
// and overlaps the predecessor's tail.
//
// Consumer warp w takes units w, w+8, w+16, ...: a unit's whole K-row is one
// warp's dot product (lane l reads float4 columns l, l+32, ...), finished by
// warp shuffles and released back to the producer with one mbarrier arrive, so
// no CTA-wide barrier follows the prologue.  Shared memory stays under half of
// an SM: the next kernel's CTA is resident at the same time and fills its own
// ring while this one finishes.
//
// Prologue: warp w loads float4 columns q = w, w+8, ... of every activation
// row into shared memory with its partial sums of squares; after a barrier per
// norm, every warp reads the normalised rows from shared memory (or, for
// K <= 1024 and M <= 2, keeps them in registers).
//
// Memory-bound: 4 bytes of weight per 2*M flops, no tensor cores (FP32 parity
// with the reference's native path is required).
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace skb {

constexpr int RG_CWARPS = 8;                      // consumer warps
constexpr int RG_THREADS = 32 * (RG_CWARPS + 1);  // + the producer warp
constexpr int RG_SLOT = 24 * 1024;                // ring slot bytes
constexpr int RG_MAX_SLOTS = 5;
constexpr int RG_HEAD = 256;                      // mbarriers + flags
// Dynamic shared memory per CTA: at most this much, so that two CTAs (of this
// kernel and its neighbour in the frame) fit in one SM's 228 KB.  Inner size
// 3072 (the trunk down projection, a 12 KB row) gets room for a fourth slot:
// its whole slice (7 rows at bs1) is then staged before the wait, and its
// neighbours (gate/up, QKV: 104 KB each) still fit beside it.
constexpr size_t RG_SMEM_BUDGET = 112 * 1024;
constexpr size_t RG_SMEM_BUDGET_K3072 = 121 * 1024;
// SwiGLU at inner size 1024 (the trunk gate/up, 170 KB of weights per CTA at
// batch 1) gets a fifth slot: its neighbours -- the O projection (3 slots: a
// ring is never deeper than a CTA's chunk count) and the down projection
// (96 KB) -- still fit beside it in one SM.
constexpr size_t RG_SMEM_BUDGET_SWIGLU = 129 * 1024;
constexpr size_t RG_SMEM_MAX = RG_SMEM_BUDGET_SWIGLU;
constexpr int RG_EPI_MAX = 256;  // staged residual / bias values per CTA

struct RgHead {
    uint64_t full[RG_MAX_SLOTS];
    uint64_t empty[RG_MAX_SLOTS];
    unsigned issued;   // chunks the producer has issued
    int producer_done;
};

__device__ __forceinline__ void named_sync_consumers() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Issues the bulk copies of units [b0, b1) into slot `dst`.
__device__ __forceinline__ void rg_issue(const GemvArgs& a, bool swiglu, int upc, int b0, int b1, float* dst,
                                         uint64_t* bar) {
    const uint32_t rowb = (uint32_t)a.K * 4u;
    if (swiglu) {
        const uint32_t bytes = (uint32_t)(b1 - b0) * rowb;
        mbar_expect_tx(bar, 2u * bytes);
        bulk_g2s(dst, a.w0 + (size_t)b0 * a.K, bytes, bar);
        bulk_g2s(dst + (size_t)upc * a.K, a.w1 + (size_t)b0 * a.K, bytes, bar);
        return;
    }
    mbar_expect_tx(bar, (uint32_t)(b1 - b0) * rowb);
    // contiguous runs inside the segments [0, seg1) w0, [seg1, seg2) w1, [seg2, N) w2
    int r = b0;
    while (r < b1) {
        const float* src;
        int end;
        if (r < a.seg1) {
            src = a.w0 + (size_t)r * a.K;
            end = min(b1, a.seg1);
        } else if (r < a.seg2) {
            src = a.w1 + (size_t)(r - a.seg1) * a.K;
            end = min(b1, a.seg2);
        } else {
            src = a.w2 + (size_t)(r - a.seg2) * a.K;
            end = b1;
        }
        bulk_g2s(dst + (size_t)(r - b0) * a.K, src, (uint32_t)(end - r) * rowb, bar);
        r = end;
    }
}

// Units per CTA the K-split mode holds in registers.
constexpr int RG_KS_UNITS = 8;

// KQ: float4 columns per lane (K <= 128 * KQ).  XR: activations in registers.
// KS (K-split, for K > 1024 without SwiGLU, at most RG_KS_UNITS units per
// CTA): warp w takes float4 columns lane + 32q, q = w, w+8, ..., of every
// unit -- the same columns its prologue normalised, so the activations stay
// in its registers and no warp reads them from shared memory -- and the 8
// warps' partial sums meet in shared memory once, after the last chunk.
// rsm: the kernel's dynamic shared memory.  Returns false in the producer
// warp (which is done once it has issued every copy), true in the consumer
// warps once this CTA's outputs are stored.
template <int M, int KQ, int XM, int EM, bool XR, bool KS>
__device__ __forceinline__ bool rgemv_body(const GemvArgs& a, const int slots, unsigned char* rsm) {
    constexpr bool SW = (EM == E_SWIGLU);
    static_assert(!KS || (!SW && !XR && M * RG_KS_UNITS <= 32), "K-split: no SwiGLU, <= 32 partial sums");
    constexpr int KP4 = KQ * 32;  // padded float4 columns per activation row
    constexpr size_t XB = KS ? 0 : (size_t)M * KP4 * 16;  // staged activations
    RgHead& hd = *reinterpret_cast<RgHead*>(rsm);
    float4* xs = reinterpret_cast<float4*>(rsm + RG_HEAD);  // [M][KP4] (not with KS)
    float* ring = reinterpret_cast<float*>(rsm + RG_HEAD + XB);
    __shared__ float red[2][RG_CWARPS][M];
    __shared__ float epi[RG_EPI_MAX];  // this CTA's residuals or bias values

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int NU = SW ? a.N / 2 : a.N;
    const int u0 = (int)((long long)blockIdx.x * NU / G);
    const int u1 = (int)((long long)(blockIdx.x + 1) * NU / G);
    const int ub = (SW ? 2 : 1) * a.K * 4;
    const int upc = RG_SLOT / ub;  // units per chunk (the host checks >= 1)
    const int nch = (u1 - u0 + upc - 1) / upc;
    const int S = slots;
    const int K4 = a.K >> 2;

    if (threadIdx.x == 0) {
        stamp_min(a.ts);
        for (int s = 0; s < S; ++s) {
            mbar_init(&hd.full[s], 1);
            mbar_init(&hd.empty[s], RG_CWARPS);
        }
        hd.issued = 0;
        hd.producer_done = 0;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == RG_CWARPS) {
        // ------------------------------------------------------- producer
        if (lane == 0) {
            for (int c = 0; c < nch; ++c) {
                const int s = c % S;
                if (c >= S && !mbar_wait(&hd.empty[s], (uint32_t)((c / S) - 1) & 1u, a.err)) break;
                const int b0 = u0 + c * upc;
                rg_issue(a, SW, upc, b0, min(b0 + upc, u1), ring + (size_t)s * (RG_SLOT / 4), &hd.full[s]);
                *(volatile unsigned*)&hd.issued = (unsigned)(c + 1);
                if (c == S - 1) prefetch_share_from(a.pf, blockIdx.x, G);
            }
            if (nch < S) prefetch_share_from(a.pf, blockIdx.x, G);
            __threadfence_block();
            *(volatile int*)&hd.producer_done = 1;
        }
        return false;
    }

    // ----------------------------------------------------------- consumers
    // Latency matters here: every global round trip after the wait is on the
    // critical path, and under a full HBM stream one costs about a
    // microsecond.  So the norm weights and the bias (weights: no predecessor
    // writes them) are read before the wait, and the activations, the addend
    // rows and the residuals are all requested in one round trip after it.
    constexpr int QW = (KQ + RG_CWARPS - 1) / RG_CWARPS;  // own float4 columns per lane
    constexpr bool NORM = (XM != X_PLAIN);
    constexpr bool ADD = (XM == X_ADD_RMSNORM || XM == X_NORM_ADD_NORM);
    const int tid = threadIdx.x;
    const int nunits = u1 - u0;
    const bool stage_epi = (EM == E_RESID || EM == E_BIAS) && nunits * M <= RG_EPI_MAX;
    float4 nwv[QW], nw2v[QW];
#pragma unroll
    for (int qi = 0; qi < QW; ++qi) {
        const int q = warp + RG_CWARPS * qi, c4 = lane + 32 * q;
        const bool valid = q < KQ && c4 < K4;
        nwv[qi] = (NORM && valid) ? __ldg(reinterpret_cast<const float4*>(a.nw) + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
        nw2v[qi] = (XM == X_NORM_ADD_NORM && valid) ? __ldg(reinterpret_cast<const float4*>(a.nw2) + c4)
                                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (EM == E_BIAS && stage_epi)
        for (int t = tid; t < nunits; t += 32 * RG_CWARPS) epi[t] = __ldg(a.bias + u0 + t);

    pdl_wait();
    if (tid == 0) stamp_wait(a.ts);
    if (a.inc != nullptr && blockIdx.x == 0 && tid < a.n_inc) atomicAdd(a.inc + tid, 1);

    float4 xo[M][QW], x2o[ADD ? M : 1][QW];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int qi = 0; qi < QW; ++qi) {
            const int q = warp + RG_CWARPS * qi, c4 = lane + 32 * q;
            const bool valid = q < KQ && c4 < K4;
            xo[m][qi] = valid ? ld_cg4(reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx) + c4)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
            if (ADD)
                x2o[ADD ? m : 0][qi] =
                    valid ? ld_cg4(reinterpret_cast<const float4*>(a.x2 + (size_t)(m / a.x2_div) * a.ldx2) + c4)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    float rv = 0.f;
    if (EM == E_RESID && stage_epi && tid < nunits * M)
        rv = __ldcg(a.resid + (size_t)(tid / nunits) * a.ldr + u0 + tid % nunits);

    // norms: partial sums of squares of the own columns -> red, one barrier,
    // every warp adds the 8 partials in warp order
    auto add4 = [](float4 v, float4 p) { return make_float4(v.x + p.x, v.y + p.y, v.z + p.z, v.w + p.w); };
    auto sq4 = [](float4 v) { return v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w; };
    auto scale4 = [](float4 w, float4 v, float inv) {
        return make_float4(w.x * (v.x * inv), w.y * (v.y * inv), w.z * (v.z * inv), w.w * (v.w * inv));
    };
    auto inv_rms = [&](float (&ss)[M], int slot, float eps, float (&inv)[M]) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float t = warp_sum(ss[m]);
            if (lane == 0) red[slot][warp][m] = t;
        }
        named_sync_consumers();
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < RG_CWARPS; ++w) tot += red[slot][w][m];
            inv[m] = rsqrtf(tot / (float)a.K + eps);
        }
    };
    if (XM == X_NORM_ADD_NORM) {
        float ss[M], inv[M];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            ss[m] = 0.f;
#pragma unroll
            for (int qi = 0; qi < QW; ++qi) ss[m] += sq4(xo[m][qi]);
        }
        inv_rms(ss, 0, a.neps2, inv);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            ss[m] = 0.f;
#pragma unroll
            for (int qi = 0; qi < QW; ++qi) {
                const int q = warp + RG_CWARPS * qi, c4 = lane + 32 * q;
                const float4 h = scale4(nw2v[qi], xo[m][qi], inv[m]);
                if (a.hout != nullptr && blockIdx.x == 0 && q < KQ && c4 < K4)
                    reinterpret_cast<float4*>(a.hout + (size_t)m * a.K)[c4] = h;
                xo[m][qi] = add4(h, x2o[ADD ? m : 0][qi]);
                ss[m] += sq4(xo[m][qi]);
            }
        }
        inv_rms(ss, 1, a.neps, inv);
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
            for (int qi = 0; qi < QW; ++qi) xo[m][qi] = scale4(nwv[qi], xo[m][qi], inv[m]);
    } else if (NORM) {
        float ss[M], inv[M];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            ss[m] = 0.f;
#pragma unroll
            for (int qi = 0; qi < QW; ++qi) {
                if (ADD) xo[m][qi] = add4(xo[m][qi], x2o[ADD ? m : 0][qi]);
                ss[m] += sq4(xo[m][qi]);
            }
        }
        inv_rms(ss, 0, a.neps, inv);
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
            for (int qi = 0; qi < QW; ++qi) xo[m][qi] = scale4(nwv[qi], xo[m][qi], inv[m]);
    }
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int qi = 0; qi < QW; ++qi) {
            const int q = warp + RG_CWARPS * qi, c4 = lane + 32 * q;
            if (q < KQ) {
                if (!KS) xs[m * KP4 + c4] = xo[m][qi];
                if (NORM && a.xout != nullptr && blockIdx.x == 0 && c4 < K4)
                    reinterpret_cast<float4*>(a.xout + (size_t)m * a.K)[c4] = xo[m][qi];
            }
        }
    if (EM == E_RESID && stage_epi && tid < nunits * M) epi[tid] = rv;
    // This CTA's reads of predecessor data are done: let the next kernel
    // launch now (its weight burst no longer delays the round trip above).
    pdl_trigger();
    named_sync_consumers();
    if (tid == 0 && a.ts) stamp_max(a.ts + 4);
    float4 xv[XR ? M : 1][XR ? KQ : 1];
    if (XR) {
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
            for (int q = 0; q < KQ; ++q) xv[XR ? m : 0][XR ? q : 0] = xs[m * KP4 + lane + 32 * q];
    }

    bool ok = true;
    unsigned long long t_first = 0, t_last = 0;  // debug: first / last chunk ready in this CTA
    if constexpr (KS) {
        // ------------------------------------------- units, K split over warps
        constexpr int NVK = RG_KS_UNITS * M;  // (unit, row) partial sums per lane
        constexpr int SHK = 5 - Log2<NVK>::value;
        __shared__ float kpart[RG_CWARPS][NVK];
        float acc[NVK];
#pragma unroll
        for (int v = 0; v < NVK; ++v) acc[v] = 0.f;
        for (int c = 0; c < nch; ++c) {
            const int s = c % S;
            if (!mbar_wait(&hd.full[s], (uint32_t)(c / S) & 1u, a.err)) {
                ok = false;
                break;
            }
            if (c == 0 && a.ts) t_first = globaltimer_ns();
            if (c == nch - 1 && a.ts) t_last = globaltimer_ns();
            const float* slot = ring + (size_t)s * (RG_SLOT / 4);
            const int jb = c * upc;
#pragma unroll
            for (int jj = 0; jj < RG_KS_UNITS; ++jj) {
                // unit jj of this CTA, when it lies in chunk c
                if (jj >= jb && jj < jb + upc && jj < nunits) {
                    const float4* w = reinterpret_cast<const float4*>(slot + (size_t)(jj - jb) * a.K);
#pragma unroll
                    for (int qi = 0; qi < QW; ++qi) {
                        const int c4 = lane + 32 * (warp + RG_CWARPS * qi);
                        if (warp + RG_CWARPS * qi < KQ && c4 < K4) {
                            const float4 wv = w[c4];
#pragma unroll
                            for (int m = 0; m < M; ++m) {
                                float t = acc[jj * M + m];
                                t = fmaf(wv.x, xo[m][qi].x, t);
                                t = fmaf(wv.y, xo[m][qi].y, t);
                                t = fmaf(wv.z, xo[m][qi].z, t);
                                t = fmaf(wv.w, xo[m][qi].w, t);
                                acc[jj * M + m] = t;
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&hd.empty[s]);
        }
        // warp totals of every (unit, row), then the sum over warps in warp order
        const float res = butterfly_reduce<NVK>(acc, lane);
        if ((lane & ((1 << SHK) - 1)) == 0) kpart[warp][lane >> SHK] = res;
        named_sync_consumers();
        if (tid < nunits * M) {
            const int j = tid / M, m = tid - j * M;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < RG_CWARPS; ++w) v += kpart[w][j * M + m];
            const int n = u0 + j;
            if (EM == E_RESID) v += stage_epi ? epi[m * nunits + j] : __ldcg(a.resid + (size_t)m * a.ldr + n);
            if (EM == E_BIAS) v += stage_epi ? epi[j] : __ldg(a.bias + n);
            a.out[(size_t)m * a.ldo + n] = v;
        }
    } else {
    // ------------------------------------------------------------ units
    constexpr int NVR = SW ? 2 * M : M;
    constexpr int NV = NVR <= 1 ? 1 : (NVR <= 2 ? 2 : (NVR <= 4 ? 4 : 8));
    constexpr int SH = 5 - Log2<NV>::value;  // lane l holds value index l >> SH
    // Every consumer warp visits every chunk in order and arrives once on its
    // slot's empty barrier, so no warp can wait on a slot's phase r+1 before
    // it has seen phase r complete (mbarrier parity would alias them).
    for (int c = 0; c < nch; ++c) {
        const int s = c % S;
        if (!mbar_wait(&hd.full[s], (uint32_t)(c / S) & 1u, a.err)) {
            ok = false;
            break;
        }
        if (c == 0 && a.ts) t_first = globaltimer_ns();
        if (c == nch - 1 && a.ts) t_last = globaltimer_ns();
        const float* slot = ring + (size_t)s * (RG_SLOT / 4);
        const int jb = c * upc, je = min(jb + upc, u1 - u0);
        for (int j = jb + ((warp - jb) % RG_CWARPS + RG_CWARPS) % RG_CWARPS; j < je; j += RG_CWARPS) {
            const int i = j - jb;
            const float4* wg = reinterpret_cast<const float4*>(slot + (size_t)i * a.K);
            const float4* wu = reinterpret_cast<const float4*>(slot + (size_t)(upc + i) * a.K);
            float acc[NV];
#pragma unroll
            for (int v = 0; v < NV; ++v) acc[v] = 0.f;
#pragma unroll
            for (int q = 0; q < KQ; ++q) {
                const int c4 = lane + 32 * q;
                if (c4 < K4) {
                    const float4 g = wg[c4];
                    float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (SW) u = wu[c4];
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        const float4 x = XR ? xv[XR ? m : 0][XR ? q : 0] : xs[m * KP4 + c4];
                        float t = acc[m];
                        t = fmaf(g.x, x.x, t);
                        t = fmaf(g.y, x.y, t);
                        t = fmaf(g.z, x.z, t);
                        t = fmaf(g.w, x.w, t);
                        acc[m] = t;
                        if (SW) {
                            float t2 = acc[M + m];
                            t2 = fmaf(u.x, x.x, t2);
                            t2 = fmaf(u.y, x.y, t2);
                            t2 = fmaf(u.z, x.z, t2);
                            t2 = fmaf(u.w, x.w, t2);
                            acc[M + m] = t2;
                        }
                    }
                }
            }
            const float res = (NV == 1) ? warp_sum(acc[0]) : butterfly_reduce<NV>(acc, lane);
            const int vi = lane >> SH;
            const bool lead = (lane & ((1 << SH) - 1)) == 0 && vi < M;
            const int n = u0 + j;
            if (SW) {
                const float up = __shfl_down_sync(FULL, res, M << SH);
                if (lead) a.out[(size_t)vi * a.ldo + n] = silu(res) * up;
            } else if (lead) {
                float v = res;
                if (EM == E_RESID) v += stage_epi ? epi[vi * nunits + j] : __ldcg(a.resid + (size_t)vi * a.ldr + n);
                if (EM == E_BIAS) v += stage_epi ? epi[j] : __ldg(a.bias + n);
                a.out[(size_t)vi * a.ldo + n] = v;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&hd.empty[s]);
    }
    }
    if (a.ts) {
        const unsigned long long t_done = globaltimer_ns();  // this warp's units are stored
        named_sync_consumers();
        if (tid == 0) {
            stamp_max(a.ts + 3);
            atomicMax(a.ts + 5, t_first);
            atomicMax(a.ts + 7, t_last);
        }
        if (lane == 0) atomicMax(a.ts + 6, t_done);
    }
    if (!ok && lane == 0) {
        // a copy never arrived: let the producer stop, then wait (bounded) for
        // every copy it issued before this CTA's shared memory is released
        const uint64_t t0 = globaltimer_ns();
        while (!*(volatile int*)&hd.producer_done && globaltimer_ns() - t0 < 2000000000ull) {
        }
        // chunks before the last S issued have completed (their slots were reused)
        const unsigned issued = *(volatile unsigned*)&hd.issued;
        const unsigned first = issued > (unsigned)S ? issued - (unsigned)S : 0u;
        for (unsigned k = first; k < issued; ++k) mbar_wait(&hd.full[k % S], (k / S) & 1u, nullptr);
    }
    return true;
}

template <int M, int KQ, int XM, int EM, bool XR, bool KS>
__global__ void __maxnreg__(112) rgemv_kernel(const GemvArgs a, const int slots) {
    extern __shared__ __align__(128) unsigned char rsm[];
    rgemv_body<M, KQ, XM, EM, XR, KS>(a, slots, rsm);
}

// ------------------------------------------------------------------ host
struct RgPlan {
    int grid = 0, slots = 0, kq = 0;
    bool xr = false, ks = false;
    size_t smem = 0;
};

// Launch shape for N logical rows of K on at most `want` CTAs; slots = 0 if
// the shape is not supported (K not a multiple of 4, K > 3072, or a unit
// larger than a ring slot).
inline RgPlan rgemv_plan(int N, int K, int M, int EM, int want) {
    RgPlan p;
    if (K <= 0 || (K & 3) != 0 || K > 3072 || N <= 0) return p;
    const int unit_bytes = (EM == E_SWIGLU ? 2 : 1) * K * 4;
    if (unit_bytes > RG_SLOT) return p;
    p.kq = K <= 1024 ? 8 : (K <= 2048 ? 16 : 24);
    p.xr = (p.kq == 8 && M <= 2);
    const int NU0 = (EM == E_SWIGLU) ? N / 2 : N;
    const int G0 = want < NU0 ? (want < 1 ? 1 : want) : NU0;
    p.ks = p.kq > 8 && EM != E_SWIGLU && (NU0 + G0 - 1) / G0 <= RG_KS_UNITS && M * RG_KS_UNITS <= 32;
    const size_t xbytes = p.ks ? 0 : (size_t)M * p.kq * 128 * 4;
    const size_t budget = p.kq == 24 ? RG_SMEM_BUDGET_K3072
                                     : (EM == E_SWIGLU && p.kq == 8 ? RG_SMEM_BUDGET_SWIGLU : RG_SMEM_BUDGET);
    const size_t avail = budget > RG_HEAD + xbytes + 2 * RG_SLOT ? budget - RG_HEAD - xbytes : 2 * RG_SLOT;
    p.slots = (int)(avail / RG_SLOT);
    if (p.slots > RG_MAX_SLOTS) p.slots = RG_MAX_SLOTS;
    if (p.slots < 2) p.slots = 2;
    // no deeper than the chunks of the largest CTA slice: unused slots would
    // only keep a neighbouring kernel's CTA off the SM
    const int units = (NU0 + G0 - 1) / G0, upc = RG_SLOT / unit_bytes;
    const int nch = (units + upc - 1) / upc;
    if (p.slots > nch) p.slots = nch < 1 ? 1 : nch;
    p.smem = RG_HEAD + xbytes + (size_t)p.slots * RG_SLOT;
    const int NU = (EM == E_SWIGLU) ? N / 2 : N;
    p.grid = want < NU ? want : NU;
    if (p.grid < 1) p.grid = 1;
    return p;
}

}  // namespace skb
