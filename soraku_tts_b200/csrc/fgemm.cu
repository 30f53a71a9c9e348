// FP32 FFMA GEMM for few rows (T <= 32): out[m][n] = epilogue(sum_k X[m][k] W(n)[k]).
//
// Between the ring GEMV (<= 4 rows) and the tensor-core GEMM: a 3xTF32
// k-stage of 32 costs the tcgen05 kernels about 0.65 us per CTA whatever the
// row count, so 16 rows pay as much as 128, while 16 rows need only 16 FMA per
// weight, well inside the SMs' FP32 rate.
//
// One CTA per SM: 8 consumer warps + 1 producer warp.  CTA c owns at most 32
// contiguous units of one weight segment (a unit is an output row, or a
// (gate, up) row pair for SwiGLU); segments get CTAs in proportion to their
// rows.  Lane l of every warp works on units pl, pl + NP (two per lane up to
// 16 rows, so each activation load feeds twice the FMAs; one at 32) over
// float4 columns kl, kl+KL, ... (pl = l % NP, kl = l / NP, NP = the CTA's
// unit groups rounded up to a power of two, KL = 32 / NP), and warp w covers
// the w-th eighth of each K-chunk (1024, 512 or 256 columns).  Activation
// loads are the same 16-byte words for all units (broadcasts); a lane's
// weight rows are its own.  The producer
// warp fills a ring of K-chunks with TMA copies (no multicast):
//   * activations: one 2-D box of 256 columns x MT rows per 256 columns
//     (rows past T arrive as zeros);
//   * weights, more than 16 units per CTA: one 2-D box of 32 columns x BR
//     rows (BR = the largest unit count of a CTA) per 32 columns, with the
//     128-byte swizzle, which puts the 8 rows a quarter-warp reads in 8
//     different bank groups;
//   * weights, at most 16 units: one 1-D copy per row and chunk into rows
//     padded by max(1, 8/NP) 16-byte words (the same conflict-free spread).
// Weight copies of the first chunks are issued before the programmatic-
// dependent-launch wait (weights do not depend on the previous kernel).
// After the last chunk, partial sums meet over the KL lanes of a unit
// (shuffles) and over the 8 warps (shared memory, in warp order), and
// threads (row, unit) apply the epilogue (store / residual / bias / SwiGLU).
#include <cudaTypedefs.h>

#include "ops.cuh"
#include "trunk.cuh"
#include "trunk_api.cuh"

namespace skb {

namespace {

constexpr int FG_CW = 8;                      // consumer warps
constexpr int FG_THREADS = 32 * (FG_CW + 1);  // + the producer warp
constexpr int FG_KC_MIN = 256;                // K-chunk (floats): 1024, 512 or 256
constexpr int FG_XBOX = 256;                  // activation box width (floats)
constexpr int FG_MAX_UNITS = 32;
constexpr int FG_MAX_SLOTS = 6;
constexpr int FG_HEAD = 256;                  // mbarriers + flags
constexpr size_t FG_SMEM = 214 * 1024;        // dynamic shared memory per CTA
constexpr size_t FG_RING = FG_SMEM - 1024 - FG_HEAD;  // after the 1024-byte alignment slack
constexpr uint64_t FG_WAIT_NS = 2000000000ull;

struct FgHead {
    uint64_t full[FG_MAX_SLOTS];
    uint64_t empty[FG_MAX_SLOTS];
    unsigned issued;  // chunks the producer issued
    int producer_done;
};
static_assert(sizeof(FgHead) <= FG_HEAD, "head");

// Launch plan, the same for every CTA (computed on the host).
struct FgPlan {
    int nseg;        // weight segments (1 for SwiGLU)
    int seg0[4];     // first unit of each segment, seg0[nseg] = NU
    int gseg[4];     // first CTA of each segment, gseg[nseg] = grid
    int boxed;       // weights as 2-D swizzled boxes
    int br;          // units per CTA at most (box rows)
    int bstride;     // box stride, floats (br rounded up to 8 rows of 32)
    int u;           // units per lane (2 up to 16 rows, else 1)
    int kl;          // lanes per unit group (KL)
    int rs;          // padded weight row stride, floats (row copies)
    int kc;          // K-chunk, floats
    int wfloats;     // weight floats of a chunk
    int slot;        // slot stride, floats (a multiple of 256: 1024-byte aligned)
    int slots;       // ring depth
};

// Tensor maps: activations, then weight segments (or gate, up).
struct FgMaps {
    CUtensorMap x, w[3];
};

__device__ __forceinline__ void fg_tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ bool fg_wait(uint64_t* bar, uint32_t parity, int* err) {
    return mbar_wait_limit(bar, parity, err, FG_WAIT_NS);
}
__device__ __forceinline__ int fg_sync_and(int v) {
    int r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.and.pred q, 1, 256, p;\n selp.s32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"(v)
        : "memory");
    return r;
}
__device__ __forceinline__ void fg_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ void fg_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// MT: the row capacity (T <= MT); SW: SwiGLU pairs; U: units per lane.
template <int MT, bool SW, int U>
__global__ void __launch_bounds__(FG_THREADS, 1)
    fgemm_kernel(const GemmArgs a, const FgPlan p, const __grid_constant__ FgMaps tm) {
    extern __shared__ __align__(128) unsigned char fg_raw[];
    unsigned char* base = fg_raw + ((1024u - (smem_u32(fg_raw) & 1023u)) & 1023u);
    FgHead& hd = *reinterpret_cast<FgHead*>(base + FG_RING);
    float* ring = reinterpret_cast<float*>(base);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // this CTA's units [u0, u1) of segment sg
    int sg = 0;
    while (sg + 1 < p.nseg && (int)blockIdx.x >= p.gseg[sg + 1]) ++sg;
    const int gs = p.gseg[sg + 1] - p.gseg[sg], j = blockIdx.x - p.gseg[sg];
    const int len = p.seg0[sg + 1] - p.seg0[sg];
    const int u0 = p.seg0[sg] + (int)((long long)j * len / gs);
    const int u1 = p.seg0[sg] + (int)((long long)(j + 1) * len / gs);
    const int nu = u1 - u0, r0 = u0 - p.seg0[sg];  // r0: first row within the segment
    const int nch = a.K / p.kc;
    const int S = p.slots;
    const int nwb = p.kc / 32;         // weight boxes per matrix and chunk
    const int nxb = p.kc / FG_XBOX;    // activation boxes per chunk

    if (tid == 0) {
        stamp_min(a.ts);
        for (int s = 0; s < S; ++s) {
            mbar_init(&hd.full[s], 1);
            mbar_init(&hd.empty[s], FG_CW);
        }
        hd.issued = 0;
        hd.producer_done = 0;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == FG_CW) {
        // ------------------------------------------------------- producer
        // lane 0 arms a chunk's barrier with its bytes, then the 32 lanes
        // issue its copies
        const uint32_t xbytes = (uint32_t)nxb * MT * FG_XBOX * 4u;
        const uint32_t wbytes = p.boxed ? (uint32_t)(SW ? 2 : 1) * nwb * p.br * 128u
                                        : (uint32_t)(SW ? 2 : 1) * nu * p.kc * 4u;
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm.x)) : "memory");
            if (p.boxed) {
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm.w[SW ? 0 : sg]))
                             : "memory");
                if (SW) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm.w[1])) : "memory");
            }
        }
        const float* seg_w = SW ? a.w0 : (sg == 0 ? a.w0 : (sg == 1 ? a.w1 : a.w2));
        auto issue_w = [&](int c, int s) {
            float* slot = ring + (size_t)s * p.slot;
            if (p.boxed) {
                for (int i = lane; i < (SW ? 2 : 1) * nwb; i += 32) {
                    const int mat = i / nwb, b = i - mat * nwb;
                    fg_tma_2d(smem_u32(slot + (size_t)i * p.bstride), &tm.w[SW ? mat : sg], c * p.kc + 32 * b, r0,
                              &hd.full[s]);
                }
            } else {
                for (int r = lane; r < (SW ? 2 : 1) * nu; r += 32) {
                    const bool up = SW && r >= nu;
                    const int u = up ? r - nu : r;
                    const float* src = (up ? a.w1 : seg_w) + (size_t)(r0 + u) * a.K + (size_t)c * p.kc;
                    bulk_g2s(slot + (size_t)((up ? p.br : 0) + u) * p.rs, src, (uint32_t)p.kc * 4u, &hd.full[s]);
                }
            }
        };
        auto issue_x = [&](int c, int s) {
            float* xs = ring + (size_t)s * p.slot + p.wfloats;
            for (int i = lane; i < nxb; i += 32)
                fg_tma_2d(smem_u32(xs + (size_t)i * MT * FG_XBOX), &tm.x, c * p.kc + FG_XBOX * i, 0, &hd.full[s]);
        };
        const int first = S < nch ? S : nch;
        for (int c = 0; c < first; ++c) {  // weights of the first chunks before the wait
            if (lane == 0) mbar_expect_tx(&hd.full[c], wbytes + xbytes);
            __syncwarp();
            issue_w(c, c);
        }
        pdl_wait();
        if (lane == 0) stamp_wait(a.ts);
        for (int c = 0; c < first; ++c) issue_x(c, c);
        pdl_trigger();
        if (lane == 0) *(volatile unsigned*)&hd.issued = (unsigned)first;
        for (int c = first; c < nch; ++c) {
            const int s = c % S;
            bool good = true;
            if (lane == 0 && !fg_wait(&hd.empty[s], (uint32_t)((c / S) - 1) & 1u, a.err)) good = false;
            if (!__shfl_sync(FULL, good ? 1 : 0, 0)) break;
            if (lane == 0) mbar_expect_tx(&hd.full[s], wbytes + xbytes);
            __syncwarp();
            issue_w(c, s);
            issue_x(c, s);
            if (lane == 0) *(volatile unsigned*)&hd.issued = (unsigned)(c + 1);
        }
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            *(volatile int*)&hd.producer_done = 1;
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    // Lane l holds units pl + j*NP (j < U) over float4 columns kl, kl+KL, ...
    // of its warp's eighth of the chunk (pl = l % NP, kl = l / NP, NP = 32 /
    // KL): the 8 lanes of a quarter-warp read 8 different rows at one column.
    pdl_wait();  // the epilogue reads residuals the previous kernel wrote
    const int np = 32 / p.kl;
    const int pl = lane & (np - 1), kl = lane / np;
    constexpr int NA = SW ? 2 * MT : MT;  // values per unit
    float acc[U][NA];
#pragma unroll
    for (int j = 0; j < U; ++j)
#pragma unroll
        for (int v = 0; v < NA; ++v) acc[j][v] = 0.f;
    const int fw = p.kc / (4 * FG_CW);  // float4 columns of a chunk per warp
    // float4 offsets of each unit's gate / up row
    int wrow[U], wrow_up[U], sw7[U];
    bool act[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
        const int ul = pl + j * np;
        act[j] = ul < nu;
        wrow[j] = p.boxed ? ul * 8 : ul * (p.rs / 4);
        wrow_up[j] = p.boxed ? nwb * (p.bstride / 4) + ul * 8 : (p.br + ul) * (p.rs / 4);
        sw7[j] = ul & 7;
    }
    bool ok = true;
    for (int c = 0; c < nch; ++c) {
        const int s = c % S;
        if (!fg_wait(&hd.full[s], (uint32_t)(c / S) & 1u, a.err)) {
            ok = false;
            break;
        }
        if (c == 0 && tid == 0) stamp_max(a.ts ? a.ts + 4 : nullptr);
        if (c < 4 && tid == 0) stamp_max(a.ts ? a.ts + 8 + c : nullptr);  // chunk c landed
        const float4* w4 = reinterpret_cast<const float4*>(ring + (size_t)s * p.slot);
        const float4* xs = reinterpret_cast<const float4*>(ring + (size_t)s * p.slot + p.wfloats);
        if (act[0]) {
            for (int f = fw * warp + kl; f < fw * warp + fw; f += p.kl) {
                // weight float4 f of each row: box f/8, 16-byte chunk f%8
                // (swizzled by the row's phase), or the padded row
                float4 wg[U], wu[U];
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    const int wo = p.boxed ? (f >> 3) * (p.bstride / 4) + ((f & 7) ^ sw7[j]) : f;
                    wg[j] = act[j] ? w4[wrow[j] + wo] : make_float4(0.f, 0.f, 0.f, 0.f);
                    wu[j] = (SW && act[j]) ? w4[wrow_up[j] + wo] : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                const float4* xr = xs + (f >> 6) * (MT * FG_XBOX / 4) + (f & 63);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    const float4 x = xr[m * (FG_XBOX / 4)];
#pragma unroll
                    for (int j = 0; j < U; ++j) {
                        float t = acc[j][m];
                        t = fmaf(wg[j].x, x.x, t);
                        t = fmaf(wg[j].y, x.y, t);
                        t = fmaf(wg[j].z, x.z, t);
                        t = fmaf(wg[j].w, x.w, t);
                        acc[j][m] = t;
                        if (SW) {
                            float t2 = acc[j][SW ? MT + m : 0];
                            t2 = fmaf(wu[j].x, x.x, t2);
                            t2 = fmaf(wu[j].y, x.y, t2);
                            t2 = fmaf(wu[j].z, x.z, t2);
                            t2 = fmaf(wu[j].w, x.w, t2);
                            acc[j][SW ? MT + m : 0] = t2;
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) fg_arrive(&hd.empty[s]);
        if (c < 4 && tid == 0) stamp_max(a.ts ? a.ts + 12 + c : nullptr);  // chunk c consumed (warp 0)
    }
    // the KL lanes of a unit (lane bits above NP), then the warps (in warp order)
    for (int o = np; o < 32; o <<= 1)
#pragma unroll
        for (int j = 0; j < U; ++j)
#pragma unroll
            for (int v = 0; v < NA; ++v) acc[j][v] += __shfl_xor_sync(FULL, acc[j][v], o);
    if (!ok && lane == 0) {
        // a copy never arrived: let the producer stop, then wait (bounded) for
        // every copy it issued before this CTA's shared memory is released
        const uint64_t t0 = globaltimer_ns();
        while (!*(volatile int*)&hd.producer_done && globaltimer_ns() - t0 < FG_WAIT_NS) {
        }
        const unsigned issued = *(volatile unsigned*)&hd.issued;
        const unsigned first = issued > (unsigned)S ? issued - (unsigned)S : 0u;
        for (unsigned k = first; k < issued; ++k) fg_wait(&hd.full[k % S], (k / S) & 1u, nullptr);
    }
    if (tid == 0) stamp_max(a.ts ? a.ts + 5 : nullptr);
    if (!fg_sync_and(ok ? 1 : 0)) return;
    // partials [warp][unit][v] over the ring (every chunk is consumed)
    float* red = ring;
    if (kl == 0)
#pragma unroll
        for (int j = 0; j < U; ++j)
            if (act[j])
#pragma unroll
                for (int v = 0; v < NA; ++v) red[((size_t)warp * nu + pl + j * np) * NA + v] = acc[j][v];
    fg_sync();
    if (tid == 0) stamp_max(a.ts ? a.ts + 6 : nullptr);
    for (int t = tid; t < a.T * nu; t += 32 * FG_CW) {
        const int m = t / nu, u = t - m * nu, n = u0 + u;
        float v = 0.f, vu = 0.f;
#pragma unroll
        for (int w = 0; w < FG_CW; ++w) {
            v += red[((size_t)w * nu + u) * NA + m];
            if (SW) vu += red[((size_t)w * nu + u) * NA + (SW ? MT + m : 0)];
        }
        float* o = a.out + (size_t)m * a.ldo + n;
        if (SW) {
            *o = silu(v) * vu;
        } else {
            if (a.mode == 1) v += __ldcg(a.resid + (size_t)m * a.ldr + n);
            if (a.mode == 2) v += __ldg(a.bias + n);
            *o = v;
        }
    }
    if (tid == 0) stamp_max(a.ts ? a.ts + 3 : nullptr);
}

PFN_cuTensorMapEncodeTiled_v12000 fg_encode = nullptr;

int fg_n_sm() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

int fg_mt(int T) { return T <= 8 ? 8 : (T <= 16 ? 16 : 32); }

// The launch plan of `a`; false when the FFMA kernel does not take the shape.
bool fg_plan(const GemmArgs& a, FgPlan& p, int& grid) {
    p = FgPlan{};
    if (a.T < 1 || a.T > 32 || a.K < FG_KC_MIN || a.K % FG_KC_MIN != 0 || a.N < 1) return false;
    const bool sw = a.interleave != 0;
    if (sw ? (a.mode != 3 || a.N % 2 != 0) : a.mode == 3) return false;
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    if (!al16(a.A) || (a.lda & 3) != 0) return false;
    const int NU = sw ? a.N / 2 : a.N;
    int len[3] = {NU, 0, 0};
    if (!sw) {
        const int s1 = a.seg1 < a.N ? a.seg1 : a.N, s2 = a.seg2 < a.N ? a.seg2 : a.N;
        if (s1 > s2) return false;
        len[0] = s1;
        len[1] = s2 - s1;
        len[2] = a.N - s2;
    }
    const float* wp[3] = {a.w0, sw ? a.w1 : a.w1, a.w2};
    for (int i = 0; i < (sw ? 2 : 3); ++i)
        if ((sw || len[i] > 0) && !al16(wp[i])) return false;
    p.nseg = sw ? 1 : 3;
    const int G = NU < fg_n_sm() ? NU : fg_n_sm();
    // CTAs per segment in proportion to its rows (at least one per non-empty segment)
    int g[3] = {0, 0, 0}, sum = 0;
    for (int i = 0; i < p.nseg; ++i) {
        if (len[i] > 0) g[i] = (int)((long long)G * len[i] / NU) > 0 ? (int)((long long)G * len[i] / NU) : 1;
        sum += g[i];
    }
    while (sum < G) {  // the segment with the most rows per CTA gets another
        int best = -1;
        for (int i = 0; i < p.nseg; ++i)
            if (len[i] > 0 && (best < 0 || (long long)len[i] * g[best] > (long long)len[best] * g[i])) best = i;
        ++g[best];
        ++sum;
    }
    while (sum > G) {  // the segment with the fewest rows per CTA gives one up
        int best = -1;
        for (int i = 0; i < p.nseg; ++i)
            if (g[i] > 1 && (best < 0 || (long long)len[i] * g[best] < (long long)len[best] * g[i])) best = i;
        if (best < 0) return false;
        --g[best];
        --sum;
    }
    p.seg0[0] = 0;
    p.gseg[0] = 0;
    p.br = 0;
    for (int i = 0; i < p.nseg; ++i) {
        p.seg0[i + 1] = p.seg0[i] + len[i];
        p.gseg[i + 1] = p.gseg[i] + g[i];
        if (g[i] > 0) {
            const int per = (len[i] + g[i] - 1) / g[i];
            p.br = per > p.br ? per : p.br;
        }
    }
    if (p.br < 1 || p.br > FG_MAX_UNITS) return false;
    const int mt = fg_mt(a.T), nm = sw ? 2 : 1;
    p.u = mt <= 16 ? 2 : 1;
    int np = 1;  // lane slots of a warp holding units: the units' groups rounded up to a power of two
    while (np < (p.br + p.u - 1) / p.u) np <<= 1;
    p.kl = 32 / np;
    p.boxed = p.br > 16;  // then np >= 8: a quarter-warp reads 8 rows of one column
    p.bstride = ((p.br + 7) / 8) * 8 * 32;
    // row padding (16-byte units) so that a quarter-warp -- np rows x 8/np
    // columns -- hits 8 different 16-byte bank groups
    const int pad = np >= 8 ? 1 : 8 / np;
    for (p.kc = 4 * FG_KC_MIN; p.kc >= FG_KC_MIN; p.kc >>= 1) {
        if (a.K % p.kc != 0) continue;
        p.rs = p.kc + 4 * pad;
        const int wf = p.boxed ? nm * (p.kc / 32) * p.bstride : nm * p.br * p.rs;
        p.wfloats = (wf + 255) & ~255;
        p.slot = p.wfloats + (p.kc / FG_XBOX) * mt * FG_XBOX;
        const int sl = (int)(FG_RING / ((size_t)p.slot * 4));
        p.slots = sl > FG_MAX_SLOTS ? FG_MAX_SLOTS : sl;
        if (p.slots >= 2) break;
    }
    if (p.slots < 2) return false;
    // partials of the reduction (warps x units x values) reuse the ring
    if ((size_t)FG_CW * p.br * nm * mt * 4 > (size_t)p.slots * p.slot * 4) return false;
    grid = G;
    return true;
}

bool fg_map(CUtensorMap* m, const float* ptr, int inner, int rows, int ld, int box_inner, int box_rows, bool swz) {
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    const cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fg_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swz ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MT, bool SW>
cudaError_t fg_launch_t(const GemmArgs& a, const FgPlan& p, const FgMaps& tm, int grid, cudaStream_t s, bool pdl) {
    constexpr int U = MT <= 16 ? 2 : 1;  // fg_plan's choice
    static bool attr_done = false;
    if (!attr_done) {
        const cudaError_t e = set_smem_attrs(fgemm_kernel<MT, SW, U>, FG_SMEM);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    return launch(fgemm_kernel<MT, SW, U>, dim3(grid), dim3(FG_THREADS), FG_SMEM, s, pdl, a, p, tm);
}

bool fg_prepare() {
    static int state = 0;  // 0 unknown, 1 ready, -1 unavailable
    if (state == 0) {
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&fg_encode),
                                                      cudaEnableDefault, &q);
        state = (e == cudaSuccess && q == cudaDriverEntryPointSuccess && fg_encode != nullptr) ? 1 : -1;
        if (state < 0) cudaGetLastError();
    }
    return state > 0;
}

}  // namespace

bool fgemm_supported(const GemmArgs& a) {
    FgPlan p;
    int grid = 0;
    return fg_plan(a, p, grid);
}

cudaError_t fgemm_launch(const GemmArgs& a, cudaStream_t s, bool pdl) {
    FgPlan p;
    int grid = 0;
    if (!fg_plan(a, p, grid)) return cudaErrorInvalidValue;
    if (!fg_prepare()) return cudaErrorNotSupported;
    const bool sw = a.interleave != 0;
    const int mt = fg_mt(a.T);
    FgMaps tm;
    memset(&tm, 0, sizeof tm);
    bool ok = fg_map(&tm.x, a.A, a.K, a.T, a.lda, FG_XBOX, mt, false);
    if (p.boxed) {
        if (sw) {
            ok = ok && fg_map(&tm.w[0], a.w0, a.K, a.N / 2, a.K, 32, p.br, true);
            ok = ok && fg_map(&tm.w[1], a.w1, a.K, a.N / 2, a.K, 32, p.br, true);
        } else {
            const float* wp[3] = {a.w0, a.w1, a.w2};
            for (int i = 0; i < 3; ++i) {
                const int len = p.seg0[i + 1] - p.seg0[i];
                if (len > 0) ok = ok && fg_map(&tm.w[i], wp[i], a.K, len, a.K, 32, p.br, true);
            }
        }
    }
    if (!ok) return cudaErrorInvalidValue;
    if (mt == 8) return sw ? fg_launch_t<8, true>(a, p, tm, grid, s, pdl) : fg_launch_t<8, false>(a, p, tm, grid, s, pdl);
    if (mt == 16)
        return sw ? fg_launch_t<16, true>(a, p, tm, grid, s, pdl) : fg_launch_t<16, false>(a, p, tm, grid, s, pdl);
    return sw ? fg_launch_t<32, true>(a, p, tm, grid, s, pdl) : fg_launch_t<32, false>(a, p, tm, grid, s, pdl);
}

}  // namespace skb
