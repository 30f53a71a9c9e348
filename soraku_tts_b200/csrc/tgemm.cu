// FP32 GEMM on the 5th-generation tensor cores with 3xTF32:
//   out[m][n] = epilogue( sum_k X[m][k] * W(n)[k] )
// for the prefill and for batched decode (more rows than the ring GEMV
// serves).  X [M][K] and W [N][K] are both K-major, as stored.
//
// 3xTF32: every operand x is split into big = x with its 13 low mantissa
// bits cleared (exactly a TF32 value) and small = x - big (exact in FP32);
// the product is big*big + big*small + small*big, accumulated in FP32 in
// tensor memory.  A kind::tf32 MMA reads only the TF32 bits of each 32-bit
// operand, so the raw FP32 tile in shared memory serves as `big` and only
// `small` is computed.  The dropped small*small term and the TF32 truncation
// of `small` leave a relative error around 2^-21 per product: FP32 parity
// within the 1e-4 tolerance.
//
// CTA tile 128 (rows of X) x 64 (rows of W), K in stages of 32, a ring of 4
// stages.  Every thread copies 6 16-byte chunks of each stage with cp.async
// (8 threads per 128-byte row segment) straight into the K-major
// 128-byte-swizzle layout the MMA reads (row r of a tile at (r/8)*1024 +
// (r%8)*128, its 16-byte chunk c at slot c ^ (r%8)); three stages are in
// flight while one is multiplied.  When a stage has landed each thread turns
// its own chunks into the `small` tile (same layout, no barrier needed
// between copy and split), then one thread issues the stage's 12
// tcgen05.mma (4 k-steps of 8 x 3 products, M=128, N=64) and commits them to
// the slot's mbarrier, which frees the slot for the stage 3 ahead.  Weight
// chunks of the first stages are requested before the wait on the previous
// kernel (they do not depend on it).
//
// Split-K: grid.z = ks CTAs share an output tile, each over a contiguous
// range of K stages, launched as one thread-block cluster (1, 1, ks).  Each
// CTA stages its 128 x 64 accumulator in its own shared memory; after a
// cluster barrier CTA z sums rows slice z of the tile over the ks CTAs in
// split order through distributed shared memory (deterministic, no global
// scratch) and applies the epilogue: store / residual / bias / SwiGLU
// (interleaved gate, up rows) with coalesced 16-byte stores.
//
// Descriptor bit layouts (shared-memory matrix descriptor, instruction
// descriptor) follow the sm_100 UMMA definitions published in CUTLASS/CuTe
// (cute/arch/mma_sm100_desc.hpp).
#include "ops.cuh"
#include "trunk.cuh"
#include "trunk_api.cuh"

namespace skb {

constexpr int TG_BM = 128, TG_BN = 64, TG_BK = 32;
constexpr int TG_THREADS = 256;
constexpr int TG_A_BYTES = TG_BM * TG_BK * 4;  // 16 KB
constexpr int TG_B_BYTES = TG_BN * TG_BK * 4;  // 8 KB
constexpr int TG_RAW = TG_A_BYTES + TG_B_BYTES;  // one stage as copied (read as `big`)
constexpr int TG_STAGE = 2 * TG_RAW;             // + its `small` parts
constexpr int TG_STAGES = 4;
constexpr int TG_MAX_SPLITS = 8;
constexpr int TG_OUT_LD = TG_BN + 4;  // staged accumulator row, floats (conflict-free 16-B stores)
constexpr size_t TG_SMEM = 1024 /* alignment slack */ + (size_t)TG_STAGES * TG_STAGE + 64;
static_assert(TG_BM * TG_OUT_LD * 4 <= TG_STAGES * TG_STAGE, "staged accumulator fits the ring");
static_assert(TG_THREADS * 4 == TG_BM * 8 && TG_THREADS * 2 == TG_BN * 8, "6 chunks per thread per stage");

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    // start address >> 4 [0,14); LBO (16 B units) [16,30) = 1; SBO [32,46) = 1024 B / 16;
    // version [46,48) = 1; layout type [61,64) = 2 (SWIZZLE_128B)
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// kind::tf32 instruction descriptor: D F32, A/B TF32, both K-major, N=64, M=128.
constexpr uint32_t TG_IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(TG_BN >> 3) << 17) |
                              ((uint32_t)(TG_BM >> 4) << 24);

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, bool accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(TG_IDESC), "r"((uint32_t)accumulate), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 16-byte global -> shared copy; `valid` false writes zeros and reads nothing.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t tg_off(int r, int c) {
    return (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u + (uint32_t)((c ^ (r & 7)) * 16);
}

__device__ __forceinline__ float4 tg_small(float4 v) {
    float4 s;
    s.x = v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
    s.y = v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
    s.z = v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
    s.w = v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
    return s;
}

__device__ __forceinline__ const float* tg_wrow(const GemmArgs& a, int n) {
    if (a.interleave) return ((n & 1) ? a.w1 : a.w0) + (size_t)(n >> 1) * a.K;
    if (n < a.seg1) return a.w0 + (size_t)n * a.K;
    if (n < a.seg2) return a.w1 + (size_t)(n - a.seg1) * a.K;
    return a.w2 + (size_t)(n - a.seg2) * a.K;
}

__device__ __forceinline__ uint32_t tg_cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t tg_cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ float4 tg_ld_peer4(uint32_t local, uint32_t rank) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(local), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(ra)
                 : "memory");
    return v;
}

__global__ void __launch_bounds__(TG_THREADS, 1) tgemm_kernel(const GemmArgs a) {
    extern __shared__ unsigned char tg_raw[];
    // 1024-byte aligned stage buffers (the swizzle pattern repeats every 1024 B)
    unsigned char* base = tg_raw + ((1024u - (smem_u32(tg_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(base);
    uint64_t* mma_bar = reinterpret_cast<uint64_t*>(base + TG_STAGES * TG_STAGE);  // [TG_STAGES]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + TG_STAGES);
    __shared__ int tg_err;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * TG_BN, m0 = blockIdx.y * TG_BM;
    const int nst = a.K / TG_BK;
    // Split-K: this CTA runs stages [sb, se) of the nst K-stages.
    const int ks = gridDim.z, z = blockIdx.z;
    const int sb = (int)((long long)z * nst / ks), se = (int)((long long)(z + 1) * nst / ks);
    const int nloc = se - sb;

    if (tid == 0) {
        for (int s = 0; s < TG_STAGES; ++s) mbar_init(&mma_bar[s], 1);
        mbar_fence_init();
        // a split grid must run as one cluster per tile (peer reads below)
        tg_err = (ks > 1 && (int)tg_cluster_size() != ks) ? 1 : 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TG_BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }

    // This thread's chunks of a stage: A rows (tid + 256 j) / 8, j < 4, and
    // W rows (tid + 256 j) / 8, j < 2; 16-byte column tid % 8.
    const int c = tid & 7;
    auto issue_w = [&](int st, int slot) {
        const uint32_t dst = sbase + slot * TG_STAGE + TG_A_BYTES;
        const int k0 = st * TG_BK + 4 * c;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int r = (tid + TG_THREADS * j) >> 3, n = n0 + r;
            const bool ok = n < a.N;
            cp_async16(dst + tg_off(r, c), ok ? tg_wrow(a, n) + k0 : a.w0, ok);
        }
    };
    auto issue_a = [&](int st, int slot) {
        const uint32_t dst = sbase + slot * TG_STAGE;
        const int k0 = st * TG_BK + 4 * c;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int r = (tid + TG_THREADS * j) >> 3, m = m0 + r;
            const bool ok = m < a.T;
            cp_async16(dst + tg_off(r, c), ok ? a.A + (size_t)m * a.lda + k0 : a.A, ok);
        }
    };
    auto split_own = [&](int slot) {
        unsigned char* raw = base + slot * TG_STAGE;
        unsigned char* sml = raw + TG_RAW;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t o = tg_off((tid + TG_THREADS * j) >> 3, c);
            *reinterpret_cast<float4*>(sml + o) = tg_small(*reinterpret_cast<const float4*>(raw + o));
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t o = TG_A_BYTES + tg_off((tid + TG_THREADS * j) >> 3, c);
            *reinterpret_cast<float4*>(sml + o) = tg_small(*reinterpret_cast<const float4*>(raw + o));
        }
    };

    // weights of the first stages do not depend on the previous kernel
    for (int i = 0; i < TG_STAGES - 1 && i < nloc; ++i) issue_w(sb + i, i);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    pdl_wait();
    // group i holds stage i's activation chunks (group 0 also the weights above)
    for (int i = 0; i < TG_STAGES - 1; ++i) {
        if (i < nloc) issue_a(sb + i, i);
        cp_async_commit();
    }
    pdl_trigger();

    int err = 0;
    for (int i = 0; i < nloc; ++i) {
        const int slot = i % TG_STAGES;
        cp_async_wait<TG_STAGES - 2>();  // this thread's chunks of stage i have landed
        split_own(slot);
        // generic-proxy shared writes -> visible to the tensor core (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t ab = sbase + slot * TG_STAGE, bb = ab + TG_A_BYTES;
            const uint32_t as_ = ab + TG_RAW, bs = bb + TG_RAW;
#pragma unroll
            for (int kk = 0; kk < TG_BK / 8; ++kk) {
                const uint32_t o = kk * 32;  // 8 TF32 = 32 bytes along K
                umma_tf32(tmem, umma_desc_sw128(ab + o), umma_desc_sw128(bb + o), i > 0 || kk > 0);
                umma_tf32(tmem, umma_desc_sw128(ab + o), umma_desc_sw128(bs + o), true);
                umma_tf32(tmem, umma_desc_sw128(as_ + o), umma_desc_sw128(bb + o), true);
            }
            umma_commit(&mma_bar[slot]);
        }
        // refill: stage i+3 goes into the slot of stage i-1, once its MMAs are done
        const int nx = i + TG_STAGES - 1;
        if (nx < nloc) {
            const int ns = nx % TG_STAGES;
            if (i >= 1 && !mbar_wait(&mma_bar[ns], (uint32_t)((i - 1) / TG_STAGES) & 1u, a.err)) err = 1;
            issue_w(sb + nx, ns);
            issue_a(sb + nx, ns);
        }
        cp_async_commit();
    }
    // all MMAs done: the last commit covers every earlier MMA of this thread
    if (nloc > 0 && !mbar_wait(&mma_bar[(nloc - 1) % TG_STAGES], (uint32_t)((nloc - 1) / TG_STAGES) & 1u, a.err))
        err = 1;
    cp_async_wait<0>();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    // accumulator -> shared tile [128][TG_OUT_LD]: warp w reads TMEM lanes
    // 32*(w%4).. (tile rows) and columns 32*(w/4)..
    const int rq = warp & 3, ch = warp >> 2;
    uint32_t r32[32];
    const uint32_t taddr = tmem + ((uint32_t)(32 * rq) << 16) + (uint32_t)(32 * ch);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r32[0]), "=r"(r32[1]), "=r"(r32[2]), "=r"(r32[3]), "=r"(r32[4]), "=r"(r32[5]), "=r"(r32[6]),
          "=r"(r32[7]), "=r"(r32[8]), "=r"(r32[9]), "=r"(r32[10]), "=r"(r32[11]), "=r"(r32[12]), "=r"(r32[13]),
          "=r"(r32[14]), "=r"(r32[15]), "=r"(r32[16]), "=r"(r32[17]), "=r"(r32[18]), "=r"(r32[19]),
          "=r"(r32[20]), "=r"(r32[21]), "=r"(r32[22]), "=r"(r32[23]), "=r"(r32[24]), "=r"(r32[25]),
          "=r"(r32[26]), "=r"(r32[27]), "=r"(r32[28]), "=r"(r32[29]), "=r"(r32[30]), "=r"(r32[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    if (nloc == 0) {
#pragma unroll
        for (int j = 0; j < 32; ++j) r32[j] = 0u;  // no K range: a zero partial
    }
    float* acc_s = reinterpret_cast<float*>(base);  // the ring is idle now
    {
        float* row = acc_s + (32 * rq + lane) * TG_OUT_LD + 32 * ch;
#pragma unroll
        for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(row + 4 * q) =
                make_float4(__uint_as_float(r32[4 * q]), __uint_as_float(r32[4 * q + 1]),
                            __uint_as_float(r32[4 * q + 2]), __uint_as_float(r32[4 * q + 3]));
    }
    if (err) atomicExch(&tg_err, 1);
    const bool split = ks > 1;
    if (split)  // every CTA's tile is in its shared memory (release / acquire)
        asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    else
        __syncthreads();
    const bool peers_ok = !split || tg_err == 0;

    // rows slice z of the tile: 16-byte groups [z*2048/ks, (z+1)*2048/ks)
    constexpr int G4 = TG_BM * TG_BN / 4;
    const int g_lo = split ? (int)(z * G4 / ks) : 0, g_hi = split ? (int)((z + 1) * G4 / ks) : G4;
    const bool vec_out = ((a.ldo & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.out) & 15) == 0);
    const bool vec_res =
        a.mode != 1 || (((a.ldr & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.resid) & 15) == 0));
    for (int g = g_lo + tid; g < g_hi; g += TG_THREADS) {
        const int r = g >> 4, c4 = g & 15;
        const int m = m0 + r, n = n0 + 4 * c4;
        const uint32_t la = smem_u32(acc_s + r * TG_OUT_LD + 4 * c4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (!split) {
            v = *reinterpret_cast<const float4*>(acc_s + r * TG_OUT_LD + 4 * c4);
        } else if (peers_ok) {
            for (int zz = 0; zz < ks; ++zz) {
                const float4 p = tg_ld_peer4(la, (uint32_t)zz);
                v.x += p.x;
                v.y += p.y;
                v.z += p.z;
                v.w += p.w;
            }
        }
        if (m >= a.T || tg_err) continue;
        float* orow = a.out + (size_t)m * a.ldo;
        if (a.mode == 3) {  // SwiGLU over (gate, up) column pairs
            if (n + 1 < a.N) orow[n >> 1] = silu(v.x) * v.y;
            if (n + 3 < a.N) orow[(n >> 1) + 1] = silu(v.z) * v.w;
            continue;
        }
        float e[4] = {v.x, v.y, v.z, v.w};
        if (n + 3 < a.N && vec_out && vec_res) {
            if (a.mode == 1) {
                const float4 q = __ldcg(reinterpret_cast<const float4*>(a.resid + (size_t)m * a.ldr + n));
                e[0] += q.x, e[1] += q.y, e[2] += q.z, e[3] += q.w;
            } else if (a.mode == 2) {
#pragma unroll
                for (int t = 0; t < 4; ++t) e[t] += __ldg(a.bias + n + t);
            }
            *reinterpret_cast<float4*>(orow + n) = make_float4(e[0], e[1], e[2], e[3]);
        } else {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                if (n + t >= a.N) break;
                float val = e[t];
                if (a.mode == 1) val += __ldcg(a.resid + (size_t)m * a.ldr + n + t);
                if (a.mode == 2) val += __ldg(a.bias + n + t);
                orow[n + t] = val;
            }
        }
    }
    if (tid == 0 && tg_err && a.err != nullptr) atomicExch(a.err, 1);
    // peers may still read this CTA's tile
    if (split) asm volatile("barrier.cluster.arrive.relaxed.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    // release the accumulator
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TG_BN) : "memory");
}

namespace {
int tg_n_sm = 148;
int tg_max_clusters[TG_MAX_SPLITS + 1];  // resident clusters of (1, 1, c) CTAs
}  // namespace

cudaError_t tgemm_prepare() {
    static bool done = false;
    if (done) return cudaSuccess;
    cudaError_t e = set_smem_attrs(tgemm_kernel, TG_SMEM);
    if (e != cudaSuccess) return e;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&tg_n_sm, cudaDevAttrMultiProcessorCount, dev);
    tg_max_clusters[1] = tg_n_sm;
    for (int c = 2; c <= TG_MAX_SPLITS; ++c) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1, 1, c);
        cfg.blockDim = dim3(TG_THREADS);
        cfg.dynamicSmemBytes = TG_SMEM;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 1;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = c;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, tgemm_kernel, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        tg_max_clusters[c] = n;
    }
    done = true;
    return cudaSuccess;
}

// Split-K factor: a.splits when given (clamped to 1..8 and the stage count),
// else the most splits (<= 8, >= 4 stages each) for which one cluster per
// tile is resident at once.
int tgemm_splits(const GemmArgs& a) {
    const int tiles = ((a.N + TG_BN - 1) / TG_BN) * ((a.T + TG_BM - 1) / TG_BM);
    const int nst = a.K / TG_BK;
    int ks;
    if (a.splits > 0) {
        ks = a.splits < TG_MAX_SPLITS ? a.splits : TG_MAX_SPLITS;
        if (ks > nst) ks = nst;
        while (ks > 1 && tg_max_clusters[ks] < 1) --ks;
        return ks < 1 ? 1 : ks;
    }
    ks = tg_n_sm / tiles;
    if (ks > nst / 4) ks = nst / 4;
    if (ks > TG_MAX_SPLITS) ks = TG_MAX_SPLITS;
    while (ks > 1 && tg_max_clusters[ks] < tiles) --ks;
    return ks < 1 ? 1 : ks;
}

// K a multiple of 32, 16-byte aligned rows.
cudaError_t tgemm_launch(const GemmArgs& a, cudaStream_t s, bool pdl) {
    const cudaError_t pe = tgemm_prepare();
    if (pe != cudaSuccess) return pe;
    if (a.K % TG_BK != 0 || a.K <= 0 || a.T <= 0 || a.N <= 0) return cudaErrorInvalidValue;
    const int ks = tgemm_splits(a);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.N + TG_BN - 1) / TG_BN, (a.T + TG_BM - 1) / TG_BM, ks);
    cfg.blockDim = dim3(TG_THREADS);
    cfg.dynamicSmemBytes = TG_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = ks;
    ++na;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, tgemm_kernel, a);
}

}  // namespace skb
