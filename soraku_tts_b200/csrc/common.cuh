// Shared device/host helpers for the sm_100a decode kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/soraku_b200.h"

namespace skb {

constexpr unsigned FULL = 0xffffffffu;

// ---------------------------------------------------------------- PDL
// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialization attribute may start while its predecessor still runs.
// Everything before pdl_wait() may only touch data no predecessor writes
// (weights, L2 prefetches); pdl_wait() returns once every predecessor grid has
// completed and flushed its memory.  Every kernel calls pdl_wait()
// unconditionally, so completion of a kernel implies completion of all
// earlier ones.
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------- L2 prefetch
// Up to 4 byte ranges of weights a later kernel will read.  The CTAs of the
// issuing kernel split the union of the ranges evenly; thread 0 of each CTA
// issues bulk L2 prefetches for its share, which proceed in the memory
// system while the kernels in between run.
struct PrefetchList {
    const char* ptr[4];
    unsigned long long bytes[4];
    int n;
};

__device__ __forceinline__ void bulk_prefetch_l2(const void* p, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Issued by the calling thread alone.
__device__ __forceinline__ void prefetch_share_from(const PrefetchList& pf, int cta, int ncta) {
    if (pf.n <= 0) return;
    unsigned long long total = 0;
    for (int i = 0; i < pf.n; ++i) total += pf.bytes[i] & ~15ull;
    // 16-byte granules keep every prefetch aligned
    unsigned long long g_total = total >> 4;
    unsigned long long g0 = g_total * (unsigned long long)cta / (unsigned long long)ncta;
    unsigned long long g1 = g_total * (unsigned long long)(cta + 1) / (unsigned long long)ncta;
    unsigned long long lo = g0 << 4, hi = g1 << 4;
    unsigned long long base = 0;
    for (int i = 0; i < pf.n; ++i) {
        const unsigned long long seg = pf.bytes[i] & ~15ull;
        unsigned long long s0 = base, s1 = base + seg;
        base += seg;
        if ((reinterpret_cast<uintptr_t>(pf.ptr[i]) & 15u) != 0) continue;  // bulk prefetch needs 16-B alignment
        unsigned long long a = lo > s0 ? lo : s0;
        unsigned long long b = hi < s1 ? hi : s1;
        while (a < b) {
            unsigned long long chunk = b - a;
            if (chunk > 65536ull) chunk = 65536ull;
            bulk_prefetch_l2(pf.ptr[i] + (a - s0), (unsigned)chunk);
            a += chunk;
        }
    }
}

// Issued by thread 0 of the CTA.
__device__ __forceinline__ void prefetch_share(const PrefetchList& pf, int cta, int ncta) {
    if (threadIdx.x == 0) prefetch_share_from(pf, cta, ncta);
}

// ----------------------------------------------------------- vector loads
// Weights are read once per pass: read-only path, no L1 allocation.
__device__ __forceinline__ float4 ldg_stream(const float4* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}
// Data written by other CTAs of the same grid (or a predecessor): L2 only.
__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float4 ld_cg4(const float4* p) { return __ldcg(p); }

// -------------------------------------------------------- warp reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}

template <int N>
struct Log2 {
    static constexpr int value = N <= 1 ? 0 : 1 + Log2<(N > 1 ? N / 2 : 1)>::value;
};
template <>
struct Log2<1> {
    static constexpr int value = 0;
};

// Butterfly reduce-scatter of N (power of two, <= 32) values per lane: on
// return, v[0] of lane l holds the warp-wide sum of value index
// (l >> (5 - log2 N)).  N - 1 + (5 - log2 N) shuffles instead of 5 N.
template <int N>
__device__ __forceinline__ float butterfly_reduce(float (&v)[N], int lane) {
    constexpr int L = Log2<N>::value;
#pragma unroll
    for (int step = 0; step < L; ++step) {
        const int half = N >> (step + 1);
        const int off = 16 >> step;
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            float send = upper ? v[i] : v[i + half];
            float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(FULL, send, off);
        }
    }
#pragma unroll
    for (int off = 16 >> L; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(FULL, v[0], off);
    return v[0];
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// Barrier policies of the block-wide building blocks (sampler, attention
// item).  BlockSync: every thread of the CTA takes part.
struct BlockSync {
    __device__ __forceinline__ static void sync() { __syncthreads(); }
};
// The same for code run by the 256 threads of warps 0..7 of a CTA whose other
// warps have exited or run independently: named barrier 1.
struct ConsumerSync {
    __device__ __forceinline__ static void sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
};

// ------------------------------------------------------ bulk copy + mbarrier
// 1-D bulk copies (TMA engine, no tensor map) from global memory into this
// CTA's shared memory, completing on an mbarrier.  No multicast: the source is
// always this GPU's own memory and the destination this CTA.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Waits for phase `parity` of an mbarrier, giving up after `limit_ns`: then
// it records the failure in *err (if given) and returns false, so a kernel
// never hangs on a copy that does not arrive.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, int* err, uint64_t limit_ns) {
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
        if (it == 0) t0 = globaltimer_ns();
        else if ((it & 255) == 0 && globaltimer_ns() - t0 > limit_ns) {
            if (err) atomicExch(err, 1);
            return false;
        }
    }
}
// The decode kernels' wait: about 2 s.
constexpr uint64_t SKB_WAIT_LIMIT_NS = 2000000000ull;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    return mbar_wait_limit(bar, parity, err, SKB_WAIT_LIMIT_NS);
}

// --------------------------------------------------------- kernel stamps
// Debug timeline of one launch (all null unless the engine's debug mode is
// on), SKB_KTS_STRIDE slots: ts[0] earliest CTA start, ts[1] earliest and
// ts[2] latest release from the programmatic-dependent-launch wait, ts[3]
// latest CTA end, ts[4..] latest CTA to reach kernel-specific points
// (%globaltimer ns).
constexpr int SKB_KTS_STRIDE = 16;
__device__ __forceinline__ void stamp_min(unsigned long long* p) {
    if (p) atomicMin(p, (unsigned long long)globaltimer_ns());
}
__device__ __forceinline__ void stamp_max(unsigned long long* p) {
    if (p) atomicMax(p, (unsigned long long)globaltimer_ns());
}
__device__ __forceinline__ void stamp_wait(unsigned long long* ts) {
    if (ts) {
        const unsigned long long t = globaltimer_ns();
        atomicMin(ts + 1, t);
        atomicMax(ts + 2, t);
    }
}

// --------------------------------------------------------------- launching
// Dynamic shared-memory limit plus the largest shared-memory carveout.  Every
// decode kernel asks for the same carveout: an SM can only hold CTAs of
// kernels whose carveouts agree, and a programmatic dependent launch is only
// useful when the next kernel's CTAs can join the running ones.
template <typename K>
inline cudaError_t set_smem_attrs(K* kernel, size_t dyn_bytes) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn_bytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
    return e;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, bool pdl, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline int status_from(cudaError_t e) { return e == cudaSuccess ? SKB_OK : SKB_ERR_CUDA; }

}  // namespace skb
