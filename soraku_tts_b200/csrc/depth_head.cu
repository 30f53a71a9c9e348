// Persistent depth head for one CFG request: the 16 depth steps of a frame
// (graph_frame.py:201-241; model.py:147-174 body + classifier, 579-595 and
// 686-708 CFG and sampling, 600-605 prefix, 105-114 frame embedding) as ONE
// cooperative launch with one CTA per SM, in place of 64 dependent kernels.
//
// The depth MLP's gate/up matrices (16.8 MB) are read by every depth step of
// every frame.  Here each CTA loads its slice of them (its SwiGLU row pairs,
// up to 112 KB) into shared memory once per frame and keeps it there for all
// 16 steps, so the UP phase streams nothing.  Per step q:
//
//   UP    a = norm_in(final_norm(x) + prefix) from registers (the final-normed
//         residual stream and the prefix live in registers: no global read),
//         act = silu(a Wg^T) * (a Wu^T) on the resident slice
//   DN    y = act Wd^T + a (K split over the warps)
//   CLS   logits = norm_out(y) table[q]^T + bias[q]
//   SMP   every CTA runs the same sampler on the same logits and uniform, so
//         every CTA knows the code; each adds table[q][code] * scale to its
//         prefix registers and starts the next UP without a barrier.
//
// DN and CLS stream their weight rows (the down matrix, re-read from L2 every
// step, and table[q] from HBM) through a ring of 16 KB slots: a producer warp
// issues 1-D bulk copies (TMA engine; source: this GPU's own memory,
// destination: this CTA, no multicast) for every step ahead of the math,
// bounded only by the ring's free slots.  Phases that read another CTA's
// output are separated by a sense-reversing grid barrier: 3 per step, 48 per
// frame.  After the last step every CTA writes its slice of the frame
// embedding (sum over q in order, * scale) as both rows' residual stream.
//
// Every wait is bounded (about 2 s): a timeout sets err[3] and the abort
// flag, every other wait gives up once it sees the flag, and each CTA drains
// its own copies in flight before it exits.
#include "depth_head.cuh"
#include "ops.cuh"
#include "rgemv.cuh"
#include "sampler.cuh"

namespace skb {

namespace {

constexpr int DH_CW = 8;                       // consumer warps
constexpr int DH_THREADS = 32 * (DH_CW + 1);   // + the producer warp
constexpr int DH_D = 1024;                     // model width
constexpr int DH_I = 2048;                     // depth MLP inner size
constexpr int DH_UPMAX = 14;                   // SwiGLU pairs per CTA held resident
constexpr int DH_DNMAX = 8;                    // down rows per CTA (K split over warps)
constexpr int DH_CLSMAX = 16;                  // classifier rows per CTA
constexpr int DH_SLOTS = 3;
constexpr int DH_SLOT = 16 * 1024;
constexpr int DH_VMAX = DEPTH_VMAX_SMALL;
constexpr size_t DH_UNION = sampler_smem_bytes<DH_VMAX>();
constexpr uint64_t DH_TIMEOUT_NS = 2000000000ull;

// dynamic shared memory layout (bytes)
constexpr size_t DH_OFF_RES = 256;                                         // resident gate | up rows
constexpr size_t DH_OFF_RING = DH_OFF_RES + (size_t)DH_UPMAX * 2 * DH_D * 4;
constexpr size_t DH_OFF_U = DH_OFF_RING + (size_t)DH_SLOTS * DH_SLOT;      // sampler | GEMV scratch
constexpr size_t DH_OFF_SMALL = DH_OFF_U + DH_UNION;
constexpr size_t DH_SMEM = DH_OFF_SMALL + 256;
static_assert(DH_SMEM <= 227 * 1024, "one CTA per SM");

struct DhHead {
    uint64_t full[DH_SLOTS];
    uint64_t empty[DH_SLOTS];
    uint64_t res_bar;   // the resident slice has landed
    unsigned issued;    // ring chunks the producer issued
    int producer_done;
    unsigned bar_old;   // thread 0: barrier word before this CTA's arrival
    int ok;
    int frame;          // the request's frame index (read at launch)
    int ph;             // thread 0: current phase (debug timeline)
};
static_assert(sizeof(DhHead) <= DH_OFF_RES, "head");

struct DhScratch {  // GEMV scratch (union with the sampler)
    float4 xs[2][256];
    float red[2][DH_CW][2];
    float epi[DH_CLSMAX];
    float kpart[DH_CW][DH_DNMAX * 2];
};
static_assert(sizeof(DhScratch) <= DH_UNION, "union");

struct DhSmall {  // survives every phase
    float ares[2][DH_DNMAX];  // a (the down residual) at this CTA's down rows
    int codes[32];
};
static_assert(sizeof(DhSmall) <= 256, "small");

__device__ __forceinline__ int dh_sync_and(int v) {
    int r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.and.pred q, 1, 256, p;\n selp.s32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"(v)
        : "memory");
    return r;
}
__device__ __forceinline__ bool dh_aborted(const DepthArgs& A) { return *(volatile const int*)A.abort != 0; }
__device__ __forceinline__ void dh_raise(const DepthArgs& A) {
    atomicExch(A.err + 3, 1);
    atomicExch(A.abort, 1);
}

// Bounded mbarrier wait that also gives up when another CTA raised the abort flag.
__device__ bool dh_mbar_wait(uint64_t* bar, uint32_t parity, const DepthArgs& A) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0;
    for (int it = 0;; ++it) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if ((it & 255) == 255) {
            if (dh_aborted(A)) return false;
            const uint64_t now = globaltimer_ns();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > DH_TIMEOUT_NS) {
                dh_raise(A);
                return false;
            }
        }
    }
}

// ------------------------------------------------------------- grid barrier
// Sense-reversing barrier on one word: CTA 0 adds 2^31 - (G - 1), every other
// CTA adds 1, so each barrier flips bit 31 and leaves the low bits as they
// were; a CTA waits until bit 31 differs from the value it saw when it arrived.
// Ends the current phase; arrives at the grid barrier when `barrier`.
// Returns the CTA-wide AND of the phase's success.
__device__ __forceinline__ bool dh_end(const DepthArgs& A, DhHead& hd, bool good, bool barrier) {
    const int ok = dh_sync_and(good ? 1 : 0);  // every consumer thread's stores are done
    if (threadIdx.x == 0) {
        if (A.ts != nullptr && blockIdx.x == 0) A.ts[2 * hd.ph + 1] = globaltimer_ns();
        ++hd.ph;
    }
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(A.abort, 1);
        return false;
    }
    if (barrier && threadIdx.x == 0) {
        const unsigned nb = blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1u) : 1u;
        __threadfence();
        hd.bar_old = atomicAdd(A.bar, nb);
    }
    return true;
}
__device__ __forceinline__ bool dh_wait(const DepthArgs& A, DhHead& hd) {
    if (threadIdx.x == 0) {
        const unsigned old = hd.bar_old;
        int good = 1;
        uint64_t t0 = 0;
        for (int it = 0;; ++it) {
            unsigned cur;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(A.bar) : "memory");
            if ((cur ^ old) & 0x80000000u) break;
            if ((it & 63) == 63) {
                if (dh_aborted(A)) {
                    good = 0;
                    break;
                }
                const uint64_t now = globaltimer_ns();
                if (t0 == 0) {
                    t0 = now;
                } else if (now - t0 > DH_TIMEOUT_NS) {
                    dh_raise(A);
                    good = 0;
                    break;
                }
            }
        }
        __threadfence();
        hd.ok = good;
        if (A.ts != nullptr && blockIdx.x == 0) A.ts[2 * hd.ph] = globaltimer_ns();
    }
    named_sync_consumers();
    return hd.ok != 0;
}

// This CTA's rows [u0, u1) of n rows.
__device__ __forceinline__ void dh_split(int n, int& u0, int& u1) {
    u0 = (int)((long long)blockIdx.x * n / gridDim.x);
    u1 = (int)((long long)(blockIdx.x + 1) * n / gridDim.x);
}
constexpr int DH_DN_UPC = DH_SLOT / (DH_I * 4);   // down rows per slot (2)
constexpr int DH_CLS_UPC = DH_SLOT / (DH_D * 4);  // classifier rows per slot (4)

// ---------------------------------------------------------------- producer
__device__ void dh_producer(const DepthArgs& A, DhHead& hd, float* ring, float* res) {
    // the resident gate / up slice (one barrier for all of it)
    int p0, p1;
    dh_split(DH_I, p0, p1);
    const int np = p1 - p0;
    mbar_expect_tx(&hd.res_bar, (uint32_t)np * 2u * DH_D * 4u);
    for (int r = 0; r < np; r += 4) {
        const int n = min(4, np - r);
        bulk_g2s(res + (size_t)r * DH_D, A.wg + (size_t)(p0 + r) * DH_D, (uint32_t)n * DH_D * 4u, &hd.res_bar);
        bulk_g2s(res + (size_t)(DH_UPMAX + r) * DH_D, A.wu + (size_t)(p0 + r) * DH_D, (uint32_t)n * DH_D * 4u,
                 &hd.res_bar);
    }
    int d0, d1, c0, c1;
    dh_split(DH_D, d0, d1);
    dh_split(A.V, c0, c1);
    uint32_t g = 0;
    auto slot_free = [&](uint32_t k) -> bool {
        if (k < DH_SLOTS) return true;
        return dh_mbar_wait(&hd.empty[k % DH_SLOTS], ((k / DH_SLOTS) - 1u) & 1u, A);
    };
    // table[0]'s slice into L2 now, table[q+1]'s at the start of step q: the
    // classifier phase then streams its rows from L2 rather than HBM
    if (c1 > c0) bulk_prefetch_l2(A.table + (size_t)c0 * DH_D, (unsigned)(c1 - c0) * DH_D * 4u);
    for (int q = 0; q < A.Q; ++q) {
        if (q + 1 < A.Q && c1 > c0)
            bulk_prefetch_l2(A.table + ((size_t)(q + 1) * A.V + c0) * DH_D, (unsigned)(c1 - c0) * DH_D * 4u);
        for (int r = d0; r < d1; r += DH_DN_UPC) {
            if (!slot_free(g)) goto done;
            const int n = min(DH_DN_UPC, d1 - r);
            const int s = (int)(g % DH_SLOTS);
            mbar_expect_tx(&hd.full[s], (uint32_t)n * DH_I * 4u);
            bulk_g2s(ring + (size_t)s * (DH_SLOT / 4), A.wd + (size_t)r * DH_I, (uint32_t)n * DH_I * 4u, &hd.full[s]);
            *(volatile unsigned*)&hd.issued = ++g;
        }
        const float* tq = A.table + (size_t)q * A.V * DH_D;
        for (int r = c0; r < c1; r += DH_CLS_UPC) {
            if (!slot_free(g)) goto done;
            const int n = min(DH_CLS_UPC, c1 - r);
            const int s = (int)(g % DH_SLOTS);
            mbar_expect_tx(&hd.full[s], (uint32_t)n * DH_D * 4u);
            bulk_g2s(ring + (size_t)s * (DH_SLOT / 4), tq + (size_t)r * DH_D, (uint32_t)n * DH_D * 4u, &hd.full[s]);
            *(volatile unsigned*)&hd.issued = ++g;
        }
    }
done:
    __threadfence_block();
    *(volatile int*)&hd.producer_done = 1;
}

// ------------------------------------------------------------ consumer parts
__device__ __forceinline__ float sq4(float4 v) { return v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w; }
__device__ __forceinline__ float4 scale4(float4 w, float4 v, float inv) {
    return make_float4(w.x * (v.x * inv), w.y * (v.y * inv), w.z * (v.z * inv), w.w * (v.w * inv));
}
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// RMSNorm of both rows held as one float4 column per thread (warp w, lane l:
// column l + 32 w); the normalised rows go to s.xs and every warp then takes
// all 8 of its lane's columns into registers.
__device__ __forceinline__ void dh_norm_to_regs(float4 (&v)[2], float4 w, float eps, DhScratch& s,
                                                float4 (&xv)[2][8]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        const float t = warp_sum(sq4(v[m]));
        if (lane == 0) s.red[0][warp][m] = t;
    }
    named_sync_consumers();
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        float tot = 0.f;
#pragma unroll
        for (int k = 0; k < DH_CW; ++k) tot += s.red[0][k][m];
        v[m] = scale4(w, v[m], rsqrtf(tot / (float)DH_D + eps));
        s.xs[m][lane + 32 * warp] = v[m];
    }
    named_sync_consumers();
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int q = 0; q < 8; ++q) xv[m][q] = s.xs[m][lane + 32 * q];
}

// Warp-per-row dot products of both rows with `rows` FP32 rows of 1024.
__device__ __forceinline__ void dh_dot2(const float* w, const float4 (&xv)[2][8], float (&acc)[2]) {
    const int lane = threadIdx.x & 31;
    const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 wv = w4[lane + 32 * q];
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            float t = acc[m];
            t = fmaf(wv.x, xv[m][q].x, t);
            t = fmaf(wv.y, xv[m][q].y, t);
            t = fmaf(wv.z, xv[m][q].z, t);
            t = fmaf(wv.w, xv[m][q].w, t);
            acc[m] = t;
        }
    }
}

__global__ void __launch_bounds__(DH_THREADS, 1) depth_head_kernel(const DepthArgs A) {
    extern __shared__ __align__(128) unsigned char smem[];
    DhHead& hd = *reinterpret_cast<DhHead*>(smem);
    float* res = reinterpret_cast<float*>(smem + DH_OFF_RES);  // [gate rows DH_UPMAX | up rows DH_UPMAX][1024]
    float* ring = reinterpret_cast<float*>(smem + DH_OFF_RING);
    unsigned char* uni = smem + DH_OFF_U;
    DhScratch& S = *reinterpret_cast<DhScratch*>(uni);
    DhSmall& sm = *reinterpret_cast<DhSmall*>(smem + DH_OFF_SMALL);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int s = 0; s < DH_SLOTS; ++s) {
            mbar_init(&hd.full[s], 1);
            mbar_init(&hd.empty[s], DH_CW);
        }
        mbar_init(&hd.res_bar, 1);
        hd.issued = 0;
        hd.producer_done = 0;
        hd.ph = 0;
        hd.frame = __ldcg(&A.st->frame);
        mbar_fence_init();
    }
    __syncthreads();
    if (warp == DH_CW) {
        if (lane == 0) dh_producer(A, hd, ring, res);
        return;
    }

    // ---------------------------------------------------------- consumers
    int p0, p1, d0, d1, c0, c1;
    dh_split(DH_I, p0, p1);
    dh_split(DH_D, d0, d1);
    dh_split(A.V, c0, c1);
    const int col = lane + 32 * warp;  // this thread's float4 column of a 1024-vector
    const float4 w_fin = __ldg(reinterpret_cast<const float4*>(A.final_norm) + col);
    const float4 w_in = __ldg(reinterpret_cast<const float4*>(A.norm_in) + col);
    const float4 w_out = __ldg(reinterpret_cast<const float4*>(A.norm_out) + col);
    const ReqState* st = A.st;
    const int frame = hd.frame;
    pdl_wait();
    if (tid == 0 && A.ts != nullptr && blockIdx.x == 0) A.ts[0] = globaltimer_ns();
    // final norm of the trunk output (kept in registers for the 16 steps)
    float4 hn[2];
#pragma unroll
    for (int m = 0; m < 2; ++m) hn[m] = ld_cg4(reinterpret_cast<const float4*>(A.x + (size_t)m * DH_D) + col);
    {
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const float t = warp_sum(sq4(hn[m]));
            if (lane == 0) S.red[1][warp][m] = t;
        }
        named_sync_consumers();
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            float tot = 0.f;
#pragma unroll
            for (int k = 0; k < DH_CW; ++k) tot += S.red[1][k][m];
            hn[m] = scale4(w_fin, hn[m], rsqrtf(tot / (float)DH_D + A.rms_eps));
            if (blockIdx.x == 0) reinterpret_cast<float4*>(A.hidden + (size_t)m * DH_D)[col] = hn[m];
        }
    }
    float4 pre = make_float4(0.f, 0.f, 0.f, 0.f);  // the request's prefix (this column)
    bool ok = dh_mbar_wait(&hd.res_bar, 0, A);
    ok = dh_sync_and(ok ? 1 : 0) != 0;
    uint32_t g = 0;  // ring chunks consumed

    for (int q = 0; q < A.Q && ok; ++q) {
        float* lg = A.logits + (size_t)q * A.logits_q_stride;
        // ----------------------------------------------------------- UP
        {
            float4 v[2] = {add4(hn[0], pre), add4(hn[1], pre)};
            float4 xv[2][8];
            dh_norm_to_regs(v, w_in, A.depth_eps, S, xv);
            // a at this CTA's down rows: the down phase's residual
            if (tid < 2 * (d1 - d0)) {
                const int m = tid / (d1 - d0), u = d0 + tid % (d1 - d0);
                sm.ares[m][u - d0] = reinterpret_cast<const float*>(&S.xs[m][0])[u];
            }
            for (int j = warp; j < p1 - p0; j += DH_CW) {
                float ag[2] = {0.f, 0.f}, au[2] = {0.f, 0.f};
                dh_dot2(res + (size_t)j * DH_D, xv, ag);
                dh_dot2(res + (size_t)(DH_UPMAX + j) * DH_D, xv, au);
                float t[4] = {ag[0], ag[1], au[0], au[1]};
                const float r = butterfly_reduce<4>(t, lane);  // lane l holds value l >> 3
                const float up = __shfl_down_sync(FULL, r, 16);
                if (lane == 0 || lane == 8) A.act[(size_t)(lane >> 3) * DH_I + p0 + j] = silu(r) * up;
            }
            if (!(ok = dh_end(A, hd, true, true))) break;
        }
        // ----------------------------------------------------------- DN
        {
            bool good = dh_wait(A, hd);
            if (!good) {
                ok = false;
                break;
            }
            // act columns: float4 columns lane + 32 (warp + 8 qi), qi < 2
            float4 xo[2][2];
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int qi = 0; qi < 2; ++qi)
                    xo[m][qi] = ld_cg4(reinterpret_cast<const float4*>(A.act + (size_t)m * DH_I) + lane + 32 * (warp + 8 * qi));
            constexpr int NVK = DH_DNMAX * 2;
            float acc[NVK];
#pragma unroll
            for (int v = 0; v < NVK; ++v) acc[v] = 0.f;
            const int nu = d1 - d0;
            for (int jb = 0; jb < nu; jb += DH_DN_UPC, ++g) {
                const int s = (int)(g % DH_SLOTS);
                if (!dh_mbar_wait(&hd.full[s], (g / DH_SLOTS) & 1u, A)) {
                    good = false;
                    ++g;
                    break;
                }
                const float* slot = ring + (size_t)s * (DH_SLOT / 4);
#pragma unroll
                for (int jj = 0; jj < DH_DNMAX; ++jj) {
                    if (jj >= jb && jj < jb + DH_DN_UPC && jj < nu) {
                        const float4* w = reinterpret_cast<const float4*>(slot + (size_t)(jj - jb) * DH_I);
#pragma unroll
                        for (int qi = 0; qi < 2; ++qi) {
                            const float4 wv = w[lane + 32 * (warp + 8 * qi)];
#pragma unroll
                            for (int m = 0; m < 2; ++m) {
                                float t = acc[jj * 2 + m];
                                t = fmaf(wv.x, xo[m][qi].x, t);
                                t = fmaf(wv.y, xo[m][qi].y, t);
                                t = fmaf(wv.z, xo[m][qi].z, t);
                                t = fmaf(wv.w, xo[m][qi].w, t);
                                acc[jj * 2 + m] = t;
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&hd.empty[s]);
            }
            const float r = butterfly_reduce<NVK>(acc, lane);  // lane l holds value l >> 1
            if ((lane & 1) == 0) S.kpart[warp][lane >> 1] = r;
            named_sync_consumers();
            if (tid < nu * 2) {
                const int j = tid >> 1, m = tid & 1;
                float v = 0.f;
#pragma unroll
                for (int k = 0; k < DH_CW; ++k) v += S.kpart[k][j * 2 + m];
                A.y[(size_t)m * DH_D + d0 + j] = v + sm.ares[m][j];
            }
            if (!(ok = dh_end(A, hd, good, true))) break;
        }
        // ---------------------------------------------------------- CLS
        {
            const int nu = c1 - c0;
            for (int t = tid; t < nu; t += 32 * DH_CW) S.epi[t] = __ldg(A.bias + (size_t)q * A.V + c0 + t);
            bool good = dh_wait(A, hd);
            if (!good) {
                ok = false;
                break;
            }
            float4 v[2];
#pragma unroll
            for (int m = 0; m < 2; ++m) v[m] = ld_cg4(reinterpret_cast<const float4*>(A.y + (size_t)m * DH_D) + col);
            float4 xv[2][8];
            dh_norm_to_regs(v, w_out, A.depth_eps, S, xv);
            for (int jb = 0; jb < nu; jb += DH_CLS_UPC, ++g) {
                const int s = (int)(g % DH_SLOTS);
                if (!dh_mbar_wait(&hd.full[s], (g / DH_SLOTS) & 1u, A)) {
                    good = false;
                    ++g;
                    break;
                }
                const float* slot = ring + (size_t)s * (DH_SLOT / 4);
                const int je = min(jb + DH_CLS_UPC, nu);
                for (int j = jb + ((warp - jb) % DH_CW + DH_CW) % DH_CW; j < je; j += DH_CW) {
                    float acc[2] = {0.f, 0.f};
                    dh_dot2(slot + (size_t)(j - jb) * DH_D, xv, acc);
                    const float r = butterfly_reduce<2>(acc, lane);  // lane l holds row l >> 4
                    if ((lane & 15) == 0) lg[(size_t)(lane >> 4) * A.V + c0 + j] = r + S.epi[j];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&hd.empty[s]);
            }
            if (!(ok = dh_end(A, hd, good, true))) break;
        }
        // ---------------------------------------------------------- SAMPLE
        {
            const bool q0 = q == 0;
            SampleJob J;
            J.cond = lg;
            J.uncond = lg + A.V;
            J.V = A.V;
            J.cfg_scale = st->cfg;
            J.temperature = q0 ? st->temp_q0 : st->temp;
            J.top_k = q0 ? st->top_k_q0 : st->top_k;
            J.top_p = q0 ? st->top_p_q0 : st->top_p;
            J.mask_eos = !q0 ? 1 : (st->eos_rule == 0 ? (*A.host_flag != 0) : (frame < st->min_new_frames));
            J.bos = A.bos;
            J.pad = A.pad;
            J.eos = A.eos;
            J.u = philox_uniform(st->seed, st->stream, (uint32_t)frame, (uint32_t)q);
            J.ts = nullptr;
            if (!dh_wait(A, hd)) {
                ok = false;
                break;
            }
            const int code = sample_one<ConsumerSync, DH_VMAX>(J, uni);
            if (tid == 0) sm.codes[q] = code;
            if (blockIdx.x == 0 && tid == 0) {
                A.cur_codes[q] = code;
                if (frame < A.max_frames) A.hist[(size_t)frame * A.Q + q] = code;
                if (q0 && code == A.eos) A.st->done = 1;
            }
            if (q < A.Q - 1) {
                const float4 t = __ldg(reinterpret_cast<const float4*>(A.table + ((size_t)q * A.V + code) * DH_D) + col);
                pre = make_float4(pre.x + t.x * A.scale, pre.y + t.y * A.scale, pre.z + t.z * A.scale,
                                  pre.w + t.w * A.scale);
            } else {
                // the frame embedding (sum over q in order, * scale) is both
                // rows' next residual stream: CTA c writes its columns of it
                named_sync_consumers();
                int i0, i1;
                dh_split(DH_D, i0, i1);
                for (int i = i0 + tid; i < i1; i += 32 * DH_CW) {
                    float v[32];
#pragma unroll
                    for (int qq = 0; qq < 32; ++qq) {
                        int c = qq < A.Q ? sm.codes[qq] : 0;
                        if (c < 0 || c >= A.V) c = 0;
                        v[qq] = qq < A.Q ? __ldg(A.table + ((size_t)qq * A.V + c) * DH_D + i) : 0.f;
                    }
                    float acc = v[0];
#pragma unroll
                    for (int qq = 1; qq < 32; ++qq)
                        if (qq < A.Q) acc = acc + v[qq];
                    acc = acc * A.scale;
                    A.x[i] = acc;
                    A.x[DH_D + i] = acc;
                }
                if (blockIdx.x == 0 && tid == 0) A.st->frame = frame + 1;
            }
            if (!(ok = dh_end(A, hd, true, false))) break;
        }
    }
    if (ok) return;
    // aborted: let the producer stop, then wait (bounded) for every copy it
    // issued before this CTA's shared memory is released
    if (tid == 0) {
        atomicExch(A.abort, 1);
        const uint64_t t0 = globaltimer_ns();
        while (!*(volatile int*)&hd.producer_done && globaltimer_ns() - t0 < DH_TIMEOUT_NS) {
        }
        mbar_wait(&hd.res_bar, 0, nullptr);
        const unsigned issued = *(volatile unsigned*)&hd.issued;
        for (unsigned k = issued > (unsigned)DH_SLOTS ? issued - DH_SLOTS : 0u; k < issued; ++k)
            mbar_wait(&hd.full[k % DH_SLOTS], (k / DH_SLOTS) & 1u, nullptr);
    }
    named_sync_consumers();
}

}  // namespace

int depth_head_phases(int Q) { return 4 * Q; }

bool depth_head_supported(int D, int I, int V, int Q, int nsm, int device) {
    if (D != DH_D || I != DH_I || V > DH_VMAX || Q < 1 || Q > 32) return false;
    if ((DH_I + nsm - 1) / nsm > DH_UPMAX || (DH_D + nsm - 1) / nsm > DH_DNMAX || (V + nsm - 1) / nsm > DH_CLSMAX)
        return false;
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device);
    if (!coop) return false;
    if (depth_head_prepare() != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, depth_head_kernel, DH_THREADS, DH_SMEM) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        return false;
    }
    return true;
}

cudaError_t depth_head_prepare() { return set_smem_attrs(depth_head_kernel, DH_SMEM); }

cudaError_t depth_head_launch(const DepthArgs& a, int grid, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(DH_THREADS);
    cfg.dynamicSmemBytes = DH_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, depth_head_kernel, a);
}

}  // namespace skb
