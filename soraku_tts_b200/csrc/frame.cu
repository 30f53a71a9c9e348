// Persistent frame kernel: a whole decode frame -- 16 depth steps with their
// sampling, the frame embedding and one 28-layer trunk step -- as ONE
// cooperative launch with one CTA per SM, for `frames` frames in a row.
//
// The frame is a fixed program of phases (GEMV or attention), the same ones
// the multi-kernel path launches as separate kernels.  Each CTA runs
//   * a producer warp (warp 8) that walks the whole program ahead of time and
//     streams every weight row this CTA will need, phase after phase, into a
//     ring of FK_SLOTS shared-memory slots with 1-D bulk copies (TMA engine;
//     source: this GPU's own memory, destination: this CTA, no multicast),
//     completing on a "full" mbarrier per slot and waiting on an "empty"
//     mbarrier before reusing a slot;
//   * 8 consumer warps that execute the phases: a GEMV phase consumes its
//     slots (same per-CTA row split, register-resident activations, butterfly
//     reduction and fused prologue/epilogues as gemv_kernel), an attention
//     phase processes (row, kv head, split) items, and the classifier phase's
//     last CTA runs the sampler.  Phases are separated by a grid barrier.
// Because weights do not depend on activations, the producer keeps HBM busy
// while the consumers wait at grid barriers or in the sampler, instead of
// every kernel boundary draining the memory pipeline.
//
// Every wait is bounded (~2 s): a timeout records an error, raises an abort
// flag that all CTAs poll, and the CTA drains its own copies in flight before
// it exits, so a fault in the program can never hang the GPU.
#include "engine_types.cuh"
#include "frame.cuh"
#include "ops.cuh"

namespace skb {

namespace {

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile_i32(const int* p) {
    int v;
    asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded mbarrier wait that also gives up when another CTA raised the abort flag.
__device__ bool fk_wait(uint64_t* bar, uint32_t parity, const FrameArgs& fa) {
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
        if ((it & 63) == 0) {
            if (ld_volatile_i32(fa.abort_flag)) return false;
            const uint64_t now = globaltimer_ns();
            if (it == 0) t0 = now;
            else if (now - t0 > 2000000000ull) {
                atomicExch(fa.err + 2, 1);
                atomicExch(fa.abort_flag, 1);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void phase_rows(const GemvArgs& g, int em, int& r0, int& r1) {
    const int unit = (em == E_SWIGLU) ? 2 : 1;
    const int NU = g.N / unit;
    r0 = (int)((long long)blockIdx.x * NU / gridDim.x) * unit;
    r1 = (int)((long long)(blockIdx.x + 1) * NU / gridDim.x) * unit;
}

// Rows per ring slot for inner size K (an even number for SwiGLU pairs).
__device__ __host__ __forceinline__ int chunk_rows(int K, int em) {
    int rows = (int)(FK_SLOT_BYTES / ((uint32_t)K * 4u));
    if (em == E_SWIGLU) rows &= ~1;
    return rows;
}

struct FkShared {
    uint64_t full[FK_SLOTS];
    uint64_t empty[FK_SLOTS];
    unsigned issued;        // chunks the producer has issued (for draining after an abort)
    int producer_done;
    int flag;
};

// ------------------------------------------------------------------ producer
// Walks the program's GEMV chunks for this CTA in execution order.
struct ChunkCursor {
    int f = 0, p = -1, rb = 0, r1 = 0, cr = 1;
    const Phase* ph = nullptr;
    __device__ bool next(const FrameArgs& fa, int& rb_out, int& re_out) {
        while (ph == nullptr || rb >= r1) {
            if (++p >= fa.n_phases) {
                p = 0;
                if (++f >= fa.frames) return false;
            }
            ph = &fa.prog[p];
            if (ph->kind != PH_GEMV) {
                ph = nullptr;
                continue;
            }
            int r0;
            phase_rows(ph->g, ph->em, r0, r1);
            rb = r0;
            cr = chunk_rows(ph->g.K, ph->em);
        }
        rb_out = rb;
        re_out = min(rb + cr, r1);
        rb = re_out;
        return true;
    }
};

// Chunks the producer prefetches into L2 ahead of copying them into the ring.
constexpr int FK_L2_AHEAD = 10;

__device__ void fk_producer(const FrameArgs& fa, FkShared& sh, unsigned char* ring) {
    if ((threadIdx.x & 31) != 0) return;
    ChunkCursor cp, pf;
    int rb, re;
    // the L2 cursor starts FK_L2_AHEAD chunks in
    for (int i = 0; i < FK_L2_AHEAD; ++i) {
        if (!pf.next(fa, rb, re)) break;
        const uint32_t row_bytes = (uint32_t)pf.ph->g.K * 4u;
        for (int r = rb; r < re; ++r) bulk_prefetch_l2(gemv_row(pf.ph->g, r), row_bytes);
    }
    uint32_t c = 0;
    while (cp.next(fa, rb, re)) {
        int prb, pre;
        if (pf.next(fa, prb, pre)) {
            const uint32_t pbytes = (uint32_t)pf.ph->g.K * 4u;
            for (int r = prb; r < pre; ++r) bulk_prefetch_l2(gemv_row(pf.ph->g, r), pbytes);
        }
        const GemvArgs& g = cp.ph->g;
        const uint32_t row_bytes = (uint32_t)g.K * 4u;
        const int slot = (int)(c % FK_SLOTS);
        const uint32_t round = c / FK_SLOTS;
        if (round > 0 && !fk_wait(&sh.empty[slot], (round - 1) & 1u, fa)) {
            *(volatile int*)&sh.producer_done = 1;
            return;
        }
        mbar_expect_tx(&sh.full[slot], (uint32_t)(re - rb) * row_bytes);
        unsigned char* dst = ring + (size_t)slot * FK_SLOT_BYTES;
        for (int r = rb; r < re; ++r) bulk_g2s(dst + (size_t)(r - rb) * row_bytes, gemv_row(g, r), row_bytes, &sh.full[slot]);
        ++c;
        *(volatile unsigned*)&sh.issued = c;
    }
    *(volatile int*)&sh.producer_done = 1;
}

// -------------------------------------------------------------- grid barrier
__device__ bool fk_grid_barrier(const FrameArgs& fa, unsigned target, FkShared& sh) {
    ConsumerSync::sync();
    if (threadIdx.x == 0) {
        int good = 1;
        // release this CTA's writes (ordered before by the CTA barrier), then arrive
        asm volatile("fence.acq_rel.gpu;\n red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(fa.bar_count) : "memory");
        uint64_t t0 = 0;
        for (int it = 0;; ++it) {
            if (ld_acquire_u32(fa.bar_count) >= target) break;
            if ((it & 63) == 0) {
                if (ld_volatile_i32(fa.abort_flag)) {
                    good = 0;
                    break;
                }
                const uint64_t now = globaltimer_ns();
                if (it == 0) t0 = now;
                else if (now - t0 > 2000000000ull) {
                    atomicExch(fa.err + 3, 1);
                    atomicExch(fa.abort_flag, 1);
                    good = 0;
                    break;
                }
            }
        }
        sh.flag = good;
    }
    ConsumerSync::sync();
    return sh.flag != 0;
}

// ------------------------------------------------------------ GEMV phase
template <int M, int KV4, int XM, int EM>
__device__ bool fk_gemv(const Phase& ph, const FrameArgs& fa, FkShared& sh, unsigned char* ring, uint32_t& c,
                        float (*red)[GEMV_WARPS][32], float* nred) {
    constexpr int RC = (int)(FK_SLOT_BYTES / (KV4 * 4096u)) >= 1 ? (int)(FK_SLOT_BYTES / (KV4 * 4096u)) : 1;
    constexpr int RCE = (EM == E_SWIGLU) ? (RC & ~1) : RC;
    constexpr int NV_RAW = RCE * M;
    constexpr int NV = NV_RAW <= 2 ? 2 : (NV_RAW <= 4 ? 4 : (NV_RAW <= 8 ? 8 : (NV_RAW <= 16 ? 16 : 32)));
    static_assert(NV_RAW <= 32, "chunk too large for the warp reduction");
    const GemvArgs& a = ph.g;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K4 = a.K >> 2;
    if (a.inc != nullptr && blockIdx.x == 0 && tid < a.n_inc) atomicAdd(a.inc + tid, 1);

    float4 xv[M][KV4];
    gemv_load_x<M, KV4, XM, ConsumerSync>(a, xv, nred);

    int r0, r1;
    phase_rows(a, EM, r0, r1);
    const int cr = chunk_rows(a.K, EM);  // == RCE for the K this variant serves
    if (cr > RCE) {  // the host only builds phases whose chunks fit this variant
        if (tid == 0) {
            atomicExch(fa.err + 2, 3);
            atomicExch(fa.abort_flag, 1);
        }
        return false;
    }
    int buf = 0;
    for (int rb = r0; rb < r1; rb += cr) {
        const int re = min(rb + cr, r1);
        const int slot = (int)(c % FK_SLOTS);
        const bool arrived = fk_wait(&sh.full[slot], (c / FK_SLOTS) & 1u, fa);
        const float* ws = reinterpret_cast<const float*>(ring + (size_t)slot * FK_SLOT_BYTES);
        float acc[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) acc[i] = 0.f;
#pragma unroll
        for (int rc = 0; rc < RCE; ++rc) {
            if (arrived && rb + rc < re) {
                const float4* wr = reinterpret_cast<const float4*>(ws + (size_t)rc * a.K);
#pragma unroll
                for (int j = 0; j < KV4; ++j) {
                    const int k4 = tid + j * GEMV_THREADS;
                    if (k4 < K4) {
                        const float4 w = wr[k4];
#pragma unroll
                        for (int m = 0; m < M; ++m) {
                            float sacc = acc[rc * M + m];
                            sacc = fmaf(w.x, xv[m][j].x, sacc);
                            sacc = fmaf(w.y, xv[m][j].y, sacc);
                            sacc = fmaf(w.z, xv[m][j].z, sacc);
                            sacc = fmaf(w.w, xv[m][j].w, sacc);
                            acc[rc * M + m] = sacc;
                        }
                    }
                }
            }
        }
        const float v = butterfly_reduce<NV>(acc, lane);
        constexpr int DUP = 32 / NV;
        if ((lane & (DUP - 1)) == 0) red[buf][warp][lane / DUP] = v;
        // every consumer is done with the slot and red[buf] is complete; the
        // vote makes a timed-out wait (in any thread) a decision of all threads
        if (!ConsumerSync::sync_and(arrived)) return false;
        if (tid == 0) mbar_arrive(&sh.empty[slot]);
        if (EM == E_SWIGLU) {
            if (tid < (RCE / 2) * M) {
                const int p = tid / M, m = tid % M;
                const int rg = rb + 2 * p;
                if (rg < re) {
                    float gs = 0.f, us = 0.f;
#pragma unroll
                    for (int w = 0; w < GEMV_WARPS; ++w) {
                        gs += red[buf][w][(2 * p) * M + m];
                        us += red[buf][w][(2 * p + 1) * M + m];
                    }
                    a.out[(size_t)m * a.ldo + (rg >> 1)] = silu(gs) * us;
                }
            }
        } else {
            if (tid < RCE * M) {
                const int rc = tid / M, m = tid % M;
                const int r = rb + rc;
                if (r < re) {
                    float sum = 0.f;
#pragma unroll
                    for (int w = 0; w < GEMV_WARPS; ++w) sum += red[buf][w][rc * M + m];
                    if (EM == E_RESID) sum += __ldcg(a.resid + (size_t)m * a.ldr + r);
                    if (EM == E_BIAS) sum += __ldg(a.bias + r);
                    a.out[(size_t)m * a.ldo + r] = sum;
                }
            }
        }
        buf ^= 1;
        ++c;
    }
    return true;
}

template <int M>
__device__ bool fk_gemv_dispatch(const Phase& ph, const FrameArgs& fa, FkShared& sh, unsigned char* ring, uint32_t& c,
                                 float (*red)[GEMV_WARPS][32], float* nred) {
#define FK_CASE(KV, X, E) \
    if (ph.kv4 == KV && ph.xm == X && ph.em == E) return fk_gemv<M, KV, X, E>(ph, fa, sh, ring, c, red, nred);
    FK_CASE(1, X_NORM_ADD_NORM, E_SWIGLU)  // depth up
    FK_CASE(2, X_PLAIN, E_RESID)           // depth down, trunk O
    FK_CASE(1, X_RMSNORM, E_BIAS)          // classifier
    FK_CASE(1, X_RMSNORM, E_STORE)         // trunk QKV
    FK_CASE(1, X_RMSNORM, E_SWIGLU)        // trunk gate/up
    FK_CASE(3, X_PLAIN, E_RESID)           // trunk down
#undef FK_CASE
    atomicExch(fa.err + 2, 2);
    atomicExch(fa.abort_flag, 1);
    return false;
}

// ------------------------------------------------------------------ kernel
template <int M>
__global__ void __launch_bounds__(FK_THREADS, 1) frame_kernel(const FrameArgs fa) {
    extern __shared__ __align__(128) unsigned char fsm[];
    FkShared& sh = *reinterpret_cast<FkShared*>(fsm);
    unsigned char* ring = fsm + FK_HEAD;
    unsigned char* samp = ring + (size_t)FK_SLOTS * FK_SLOT_BYTES;
    __shared__ float red[2][GEMV_WARPS][32];
    __shared__ float nred[GEMV_WARPS * 4];
    __shared__ AttnSmem asmem;
    __shared__ int codes_s[32];

    if (threadIdx.x == 0) {
        for (int i = 0; i < FK_SLOTS; ++i) {
            mbar_init(&sh.full[i], 1);
            mbar_init(&sh.empty[i], 1);
        }
        sh.issued = 0;
        sh.producer_done = 0;
        mbar_fence_init();
    }
    __syncthreads();  // the only barrier the producer warp joins

    if (threadIdx.x >= FK_CONSUMER_THREADS) {
        fk_producer(fa, sh, ring);
        return;
    }

    uint32_t c = 0;
    unsigned nbar = 0;
    bool ok = true;
    for (int f = 0; f < fa.frames && ok; ++f) {
        for (int p = 0; p < fa.n_phases && ok; ++p) {
            const Phase& ph = fa.prog[p];
            unsigned long long* tl = fa.timeline ? fa.timeline + 2 * ((size_t)f * fa.n_phases + p) : nullptr;
            if (tl && blockIdx.x == 0 && threadIdx.x == 0) tl[0] = globaltimer_ns();
            if (ph.kind == PH_GEMV) {
                ok = fk_gemv_dispatch<M>(ph, fa, sh, ring, c, red, nred);
                if (ok && ph.sample) {
                    // the CTA that finishes the classifier last samples every request
                    __threadfence();
                    ConsumerSync::sync();
                    if (threadIdx.x == 0) sh.flag = (atomicAdd(fa.sample_ticket, 1) == (int)gridDim.x - 1) ? 1 : 0;
                    ConsumerSync::sync();
                    if (sh.flag) {
                        __threadfence();
                        for (int r = 0; r < ph.n_req; ++r)
                            depth_sample_body<ConsumerSync, FK_VMAX>(ph.s, r, samp, codes_s);
                        if (threadIdx.x == 0) {
                            *fa.sample_ticket = 0;
                            if (tl) tl[1] = globaltimer_ns();
                        }
                    }
                }
            } else {
                const DecodeAttnArgs& at = ph.at;
                const int per_row = at.kv.KVH * at.S;
                const int items = ph.attn_rows * per_row;
                for (int it = blockIdx.x; it < items; it += gridDim.x) {
                    const int r = it / per_row, rem = it % per_row;
                    decode_attn_item<ConsumerSync>(at, rem % at.S, rem / at.S, r, asmem);
                }
            }
            if (tl && blockIdx.x == 0 && threadIdx.x == 0 && !(ph.kind == PH_GEMV && ph.sample))
                tl[1] = globaltimer_ns();
            if (fa.cta_end && threadIdx.x == 0)
                fa.cta_end[((size_t)f * fa.n_phases + p) * gridDim.x + blockIdx.x] = globaltimer_ns();
            if (ok) ok = fk_grid_barrier(fa, ++nbar * gridDim.x, sh);
        }
    }
    if (!ok && threadIdx.x == 0) {
        // abort: let the producer stop, then drain every copy still in flight
        // into this CTA's ring before the CTA exits
        const uint64_t t0 = globaltimer_ns();
        while (!*(volatile int*)&sh.producer_done && globaltimer_ns() - t0 < 2000000000ull) {
        }
        const unsigned issued = *(volatile unsigned*)&sh.issued;
        for (unsigned k = c; k < issued; ++k) mbar_wait(&sh.full[k % FK_SLOTS], (k / FK_SLOTS) & 1u, nullptr);
    }
}

}  // namespace

size_t frame_kernel_smem() { return FK_SMEM; }

cudaError_t frame_kernel_prepare(int M) {
    cudaError_t e = cudaErrorInvalidValue;
    if (M == 1) e = cudaFuncSetAttribute(frame_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FK_SMEM);
    if (M == 2) e = cudaFuncSetAttribute(frame_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FK_SMEM);
    if (M == 4) e = cudaFuncSetAttribute(frame_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FK_SMEM);
    return e;
}

int frame_kernel_occupancy(int M) {
    int n = 0;
    if (M == 1) cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, frame_kernel<1>, FK_THREADS, FK_SMEM);
    if (M == 2) cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, frame_kernel<2>, FK_THREADS, FK_SMEM);
    if (M == 4) cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, frame_kernel<4>, FK_THREADS, FK_SMEM);
    return n;
}

// Cooperative launch: the runtime refuses it unless every CTA is resident at
// once, which the grid barriers require.
cudaError_t frame_kernel_launch(int M, const FrameArgs& fa, int grid, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(FK_THREADS);
    cfg.dynamicSmemBytes = FK_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (M == 1) return cudaLaunchKernelEx(&cfg, frame_kernel<1>, fa);
    if (M == 2) return cudaLaunchKernelEx(&cfg, frame_kernel<2>, fa);
    if (M == 4) return cudaLaunchKernelEx(&cfg, frame_kernel<4>, fa);
    return cudaErrorInvalidValue;
}



}  // namespace skb
