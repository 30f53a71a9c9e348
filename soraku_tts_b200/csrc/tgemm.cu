// FP32 GEMM on the 5th-generation tensor cores with 3xTF32:
//   out[m][n] = epilogue( sum_k X[m][k] * W(n)[k] )
// for the prefill and for batched decode (more rows than the ring GEMV
// serves).  X [M][K] and W [N][K] are both K-major, as stored.
//
// 3xTF32: every operand x is split into big = x with its 13 low mantissa
// bits cleared (exactly a TF32 value) and small = x - big (exact in FP32);
// the product is big*big + big*small + small*big, accumulated in FP32 in
// tensor memory.  A kind::tf32 MMA reads only the TF32 bits of each 32-bit
// operand, so raw FP32 values serve as `big` and only `small` is computed.
// The dropped small*small term and the TF32 truncation of `small` leave a
// relative error around 2^-21 per product: FP32 parity within the 1e-4
// tolerance.
//
// A TF32 MMA with M = 128 costs nearly the same time for N = 64 and 128 and
// only ~1.2x that for N = 256 (measured on B200), so the tile is 128 rows of
// X x 128 rows of W and the W operand of the main product is the stacked
// [W_big; W_small] (N = 256): per k-step of 8,
//   D[:, 0:256)  += X_big   . [W_big; W_small]^T    (N = 256)
//   D[:, 0:128)  += X_small . W_big^T               (N = 128)
// and the result is D[:, 0:128) + D[:, 128:256).  K runs in stages of 32,
// warp specialised:
//   warp 0 (one thread)  TMA: 2-D tiled loads (128-byte swizzle, the K-major
//                        layout the MMA reads) of the X and W boxes of a
//                        stage into a ring of 4 stages; rows past the end of
//                        X or W arrive as zeros;
//   warps 4-7            X to tensor memory: lane l of warp w moves row
//                        32*(w%4)+l of the stage (its TMEM lane) as big and
//                        small TF32 columns, so the MMAs read X from TMEM;
//   warps 2-3            W split: W_small of the stage, written right after
//                        W_big in the same 128-byte-swizzle layout;
//   warp 1 (one thread)  MMA: 8 tcgen05.mma per stage, committed to the
//                        stage's slot (which frees it for the stage 4 ahead).
// One lane per warp waits on and arrives at the barriers; the warp
// synchronises around it.  Weight boxes of the first stages are requested
// before the wait on the previous kernel (they do not depend on it).  For
// SwiGLU the W box is 64 gate rows then the 64 matching up rows, so result
// column j pairs with column j + 64.
//
// Split-K: grid.z = ks CTAs share an output tile, each over a contiguous
// range of K stages, launched as one thread-block cluster (1, 1, ks).  Each
// CTA stages its 128 x 128 result in its own shared memory; after a cluster
// barrier CTA z sums rows slice z of the tile over the ks CTAs in split
// order through distributed shared memory (deterministic, no global
// scratch) and applies the epilogue (store / residual / bias / SwiGLU) with
// coalesced 16-byte stores.
//
// Descriptor bit layouts (shared-memory matrix descriptor, instruction
// descriptor) follow the sm_100 UMMA definitions published in CUTLASS/CuTe
// (cute/arch/mma_sm100_desc.hpp).
#include <cudaTypedefs.h>

#include "ops.cuh"
#include "trunk.cuh"
#include "trunk_api.cuh"

namespace skb {

constexpr int TG_BM = 128, TG_BN = 128, TG_BK = 32;
constexpr int TG_THREADS = 256;
constexpr int TG_X_BYTES = TG_BM * TG_BK * 4;                 // 16 KB
constexpr int TG_W_BYTES = TG_BN * TG_BK * 4;                 // 16 KB
constexpr int TG_STAGE = TG_X_BYTES + 2 * TG_W_BYTES;         // X | W_big | W_small
constexpr int TG_STAGES = 4;
constexpr int TG_WSPLIT_THREADS = 64;                         // warps 2-3
constexpr int TG_READY_WARPS = 6;                             // warps 2-7 arrive per stage
constexpr uint32_t TG_XCOL = 2 * TG_BN;                       // TMEM: result [0, 256), X buffers after
constexpr uint32_t TG_TMEM_COLS = 512;
constexpr int TG_MAX_SPLITS = 8;
constexpr int TG_EB = 4;  // epilogue groups per thread per batch
constexpr int TG_OUT_LD = TG_BN + 4;  // staged result row, floats (conflict-free 16-B stores)
constexpr int TG_BAR_BYTES = 128;
constexpr size_t TG_SMEM = 1024 /* alignment slack */ + (size_t)TG_STAGES * TG_STAGE + TG_BAR_BYTES;
static_assert(TG_BM * TG_OUT_LD * 4 <= TG_STAGES * TG_STAGE, "staged result fits the ring");
static_assert((TG_W_BYTES / 16) % TG_WSPLIT_THREADS == 0, "split work divides evenly");
static_assert(TG_XCOL + TG_STAGES * 2 * TG_BK <= TG_TMEM_COLS, "X buffers fit the TMEM allocation");
static_assert((3 * TG_STAGES + 1) * 8 + 4 <= TG_BAR_BYTES, "barriers fit");

// Operand tensor maps: X, then W as up to three row segments (or gate, up).
struct TgMaps {
    CUtensorMap a, w[3];
};

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

// kind::tf32 instruction descriptor: D F32, A/B TF32, both K-major, M=128.
__host__ __device__ constexpr uint32_t tg_idesc(int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TG_BM >> 4) << 24);
}

// A (X) from tensor memory, B (W) from shared memory.
template <int N>
__device__ __forceinline__ void umma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, bool accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %3, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %4, {%5, %5, %5, %5}, p;\n}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"((uint32_t)accumulate), "r"(tg_idesc(N)), "r"(0u)
        : "memory");
}

// 32 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
          "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
          "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tg_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 2-D tiled TMA load of box (x = K offset, y = row) into this CTA's shared
// memory, completing on `bar`.  No multicast.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// byte offset of 16-byte chunk c of row r in a K-major 128-byte-swizzle tile
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

// PART: a batch of fewer than 128 rows (one row tile, partly filled): the
// X movers, the result staging and the split-K reduction skip the rows past
// it.  Full tiles run without those tests (they cost the full-tile K loop
// several per cent in measurement).
template <bool PART>
__global__ void __launch_bounds__(TG_THREADS, 1) tgemm_kernel(const GemmArgs a, const __grid_constant__ TgMaps tm) {
    extern __shared__ unsigned char tg_raw[];
    // 1024-byte aligned stage buffers (the swizzle pattern repeats every 1024 B)
    unsigned char* base = tg_raw + ((1024u - (smem_u32(tg_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(base);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + TG_STAGES * TG_STAGE);  // TMA landed [STAGES]
    uint64_t* ready = full + TG_STAGES;    // X in TMEM and W_small written [STAGES]
    uint64_t* empty = ready + TG_STAGES;   // MMAs done with a stage [STAGES]
    uint64_t* accfull = empty + TG_STAGES; // every MMA done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accfull + 1);
    __shared__ int tg_err;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * TG_BN, m0 = blockIdx.y * TG_BM;
    const int nst = a.K / TG_BK;
    // Split-K: this CTA runs stages [sb, se) of the nst K-stages.
    const int ks = gridDim.z, z = blockIdx.z;
    const int sb = (int)((long long)z * nst / ks), se = (int)((long long)(z + 1) * nst / ks);
    const int nloc = se - sb;

    // W box of a stage: 128 rows of one segment, or 64 gate + 64 up rows
    const CUtensorMap* wmap0;
    const CUtensorMap* wmap1 = nullptr;
    int wy;
    if (a.interleave) {
        wmap0 = &tm.w[0];
        wmap1 = &tm.w[1];
        wy = n0 >> 1;
    } else if (n0 < a.seg1) {
        wmap0 = &tm.w[0];
        wy = n0;
    } else if (n0 < a.seg2) {
        wmap0 = &tm.w[1];
        wy = n0 - a.seg1;
    } else {
        wmap0 = &tm.w[2];
        wy = n0 - a.seg2;
    }
    auto load_w = [&](int st, int slot) {
        const uint32_t dst = sbase + slot * TG_STAGE + TG_X_BYTES;
        if (wmap1) {
            tma_load_2d(dst, wmap0, st * TG_BK, wy, &full[slot]);
            tma_load_2d(dst + TG_W_BYTES / 2, wmap1, st * TG_BK, wy, &full[slot]);
        } else {
            tma_load_2d(dst, wmap0, st * TG_BK, wy, &full[slot]);
        }
    };

    if (tid == 0) {
        stamp_min(a.ts);
        for (int s = 0; s < TG_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&ready[s], TG_READY_WARPS);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accfull, 1);
        mbar_fence_init();
        // a split grid must run as one cluster per tile (peer reads below)
        tg_err = (ks > 1 && (int)tg_cluster_size() != ks) ? 1 : 0;
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(wmap0)) : "memory");
        if (wmap1) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(wmap1)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm.a)) : "memory");
        // weights of the first stages do not depend on the previous kernel
        for (int i = 0; i < TG_STAGES && i < nloc; ++i) {
            mbar_expect_tx(&full[i], TG_X_BYTES + TG_W_BYTES);
            load_w(sb + i, i);
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TG_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    pdl_wait();
    if (tid == 0) stamp_wait(a.ts);
    int err = 0;
    if (warp == 0) {
        if (lane == 0) {  // producer
            for (int i = 0; i < TG_STAGES && i < nloc; ++i)
                tma_load_2d(sbase + i * TG_STAGE, &tm.a, (sb + i) * TG_BK, m0, &full[i]);
            pdl_trigger();
            for (int i = TG_STAGES; i < nloc; ++i) {
                const int s = i % TG_STAGES;
                if (!mbar_wait(&empty[s], (uint32_t)((i - TG_STAGES) / TG_STAGES) & 1u, a.err)) err = 1;
                mbar_expect_tx(&full[s], TG_X_BYTES + TG_W_BYTES);
                load_w(sb + i, s);
                tma_load_2d(sbase + s * TG_STAGE, &tm.a, (sb + i) * TG_BK, m0, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issue
            for (int i = 0; i < nloc; ++i) {
                const int s = i % TG_STAGES;
                if (!mbar_wait(&ready[s], (uint32_t)(i / TG_STAGES) & 1u, a.err)) err = 1;
                if (i == 0 && a.ts) {
                    stamp_max(a.ts + 4);
                    stamp_min(a.ts + 8);
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t wb = sbase + s * TG_STAGE + TG_X_BYTES;  // W_big, W_small follows
                const uint32_t xb = tmem + TG_XCOL + (uint32_t)s * 2 * TG_BK, xs = xb + TG_BK;
#pragma unroll
                for (int kk = 0; kk < TG_BK / 8; ++kk) {
                    // 8 TF32 per k-step: 32 bytes along K in shared memory, 8 TMEM columns
                    const uint64_t dw = umma_desc_sw128(wb + kk * 32);
                    umma_tf32_ts<2 * TG_BN>(tmem, xb + kk * 8, dw, i > 0 || kk > 0);
                    umma_tf32_ts<TG_BN>(tmem, xs + kk * 8, dw, true);
                }
                umma_commit(&empty[s]);
            }
            if (nloc > 0) umma_commit(accfull);
        }
    } else if (warp < 4) {  // W split
        const int t = tid - 64;
        for (int i = 0; i < nloc; ++i) {
            const int s = i % TG_STAGES;
            if (lane == 0 && !mbar_wait(&full[s], (uint32_t)(i / TG_STAGES) & 1u, a.err)) err = 1;
            __syncwarp();
            const float4* wr = reinterpret_cast<const float4*>(base + s * TG_STAGE + TG_X_BYTES);
            float4* ws = reinterpret_cast<float4*>(base + s * TG_STAGE + TG_X_BYTES + TG_W_BYTES);
#pragma unroll
            for (int q = 0; q < TG_W_BYTES / 16 / TG_WSPLIT_THREADS; ++q)
                ws[t + TG_WSPLIT_THREADS * q] = tg_small(wr[t + TG_WSPLIT_THREADS * q]);
            // generic-proxy shared writes -> visible to the tensor core (async proxy)
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) tg_arrive(&ready[s]);
        }
    } else {  // X rows -> TMEM (warp w owns TMEM lanes 32*(w%4)..)
        const int r = 32 * (warp & 3) + lane;
        const uint32_t lane_addr = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        // a warp whose 32 rows all lie past the batch moves nothing (those
        // TMEM lanes only feed result rows that are never stored) but still
        // paces its arrivals by the stages
        const bool moves = !PART || 32 * (warp & 3) < a.T - m0;
        for (int i = 0; i < nloc; ++i) {
            const int s = i % TG_STAGES;
            if (lane == 0 && !mbar_wait(&full[s], (uint32_t)(i / TG_STAGES) & 1u, a.err)) err = 1;
            __syncwarp();
            if (!moves) {
                if (lane == 0) tg_arrive(&ready[s]);
                continue;
            }
            // The stage's TMEM buffer is free: its previous MMAs completed
            // before the producer refilled this slot.
            const unsigned char* raw = base + s * TG_STAGE;
            uint32_t big[32], sml[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float4 v = *reinterpret_cast<const float4*>(raw + tg_off(r, c));
                const float4 w = tg_small(v);
                big[4 * c] = __float_as_uint(v.x);
                big[4 * c + 1] = __float_as_uint(v.y);
                big[4 * c + 2] = __float_as_uint(v.z);
                big[4 * c + 3] = __float_as_uint(v.w);
                sml[4 * c] = __float_as_uint(w.x);
                sml[4 * c + 1] = __float_as_uint(w.y);
                sml[4 * c + 2] = __float_as_uint(w.z);
                sml[4 * c + 3] = __float_as_uint(w.w);
            }
            const uint32_t col = lane_addr + TG_XCOL + (uint32_t)s * 2 * TG_BK;
            tmem_st32(col, big);
            tmem_st32(col + TG_BK, sml);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) tg_arrive(&ready[s]);
        }
    }
    __syncwarp();
    // all MMAs done (so every TMA load was consumed)
    if (lane == 0 && nloc > 0 && !mbar_wait(accfull, 0u, a.err)) err = 1;
    if (tid == 0) stamp_max(a.ts ? a.ts + 5 : nullptr);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    // result -> shared tile [128][TG_OUT_LD]: warp w reads TMEM lanes
    // 32*(w%4).. (tile rows) and result columns 64*(w/4).. as D[c] + D[128+c]
    const int rq = warp & 3, hf = warp >> 2;
    float* acc_s = reinterpret_cast<float*>(base);  // the ring is idle now
    // rows of X this tile holds (a batch of 32 or 64 rows fills part of the
    // 128-row tile): staging and the split-K reduction skip the rest
    const int rows_here = PART ? (a.T - m0 < TG_BM ? a.T - m0 : TG_BM) : TG_BM;
    if (!PART || 32 * rq < rows_here) {
        const uint32_t lrow = tmem + ((uint32_t)(32 * rq) << 16);
        float* row = acc_s + (32 * rq + lane) * TG_OUT_LD;
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
            const int c0 = 64 * hf + 32 * h;
            uint32_t d1[32], d2[32];
            tmem_ld32(lrow + (uint32_t)c0, d1);
            tmem_ld32(lrow + (uint32_t)(TG_BN + c0), d2);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (nloc > 0)  // no K range: a zero partial
                    v = make_float4(__uint_as_float(d1[4 * q]) + __uint_as_float(d2[4 * q]),
                                    __uint_as_float(d1[4 * q + 1]) + __uint_as_float(d2[4 * q + 1]),
                                    __uint_as_float(d1[4 * q + 2]) + __uint_as_float(d2[4 * q + 2]),
                                    __uint_as_float(d1[4 * q + 3]) + __uint_as_float(d2[4 * q + 3]));
                *reinterpret_cast<float4*>(row + c0 + 4 * q) = v;
            }
        }
    }
    if (err) atomicExch(&tg_err, 1);
    const bool split = ks > 1;
    if (split)  // every CTA's tile is in its shared memory (release / acquire)
        asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    else
        __syncthreads();
    const bool peers_ok = !split || tg_err == 0;
    if (tid == 0) stamp_max(a.ts ? a.ts + 6 : nullptr);

    // 16-byte groups of the output: rows x 32 (rows x 16 for SwiGLU, whose
    // group c pairs gate columns 4c.. with up columns 64+4c..); CTA z of a
    // split tile owns groups [z*G/ks, (z+1)*G/ks)
    const bool glu = a.mode == 3;
    const int per_row = glu ? TG_BN / 8 : TG_BN / 4;
    const int G = rows_here * per_row;
    const int g_lo = split ? (int)((long long)z * G / ks) : 0;
    const int g_hi = split ? (int)((long long)(z + 1) * G / ks) : G;
    const bool vec_out = ((a.ldo & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.out) & 15) == 0);
    const bool vec_res =
        a.mode != 1 || (((a.ldr & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.resid) & 15) == 0));
    const int ncols = glu ? a.N >> 1 : a.N;  // output columns
    const int oc0 = glu ? n0 >> 1 : n0;
    // Groups are handled TG_EB at a time with every load of the batch (peer
    // partials, residual) issued before any is used: one memory round trip
    // per batch instead of one per load.
    for (int g0 = g_lo + tid; g0 < g_hi; g0 += TG_THREADS * TG_EB) {
        float4 v[TG_EB], u[TG_EB], q[TG_EB];
#pragma unroll
        for (int b = 0; b < TG_EB; ++b) {
            const int g = g0 + b * TG_THREADS;
            v[b] = u[b] = q[b] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (g >= g_hi) continue;
            const int r = g / per_row, c4 = g % per_row;
            const int m = m0 + r, n = oc0 + 4 * c4;
            if (a.mode == 1 && m < a.T && n + 3 < ncols && vec_res)
                q[b] = __ldcg(reinterpret_cast<const float4*>(a.resid + (size_t)m * a.ldr + n));
        }
#pragma unroll
        for (int b = 0; b < TG_EB; ++b) {
            const int g = g0 + b * TG_THREADS;
            if (g >= g_hi) continue;
            const int r = g / per_row, c4 = g % per_row;
            const float* src = acc_s + r * TG_OUT_LD + 4 * c4;
            if (!split) {
                v[b] = *reinterpret_cast<const float4*>(src);
                if (glu) u[b] = *reinterpret_cast<const float4*>(src + TG_BN / 2);
            } else if (peers_ok) {
                const uint32_t la = smem_u32(src);
                float4 p[TG_MAX_SPLITS], pu[TG_MAX_SPLITS];
#pragma unroll
                for (int zz = 0; zz < TG_MAX_SPLITS; ++zz) {
                    if (zz < ks) {
                        p[zz] = tg_ld_peer4(la, (uint32_t)zz);
                        if (glu) pu[zz] = tg_ld_peer4(la + TG_BN / 2 * 4, (uint32_t)zz);
                    }
                }
#pragma unroll
                for (int zz = 0; zz < TG_MAX_SPLITS; ++zz) {  // split order
                    if (zz < ks) {
                        v[b].x += p[zz].x, v[b].y += p[zz].y, v[b].z += p[zz].z, v[b].w += p[zz].w;
                        if (glu) u[b].x += pu[zz].x, u[b].y += pu[zz].y, u[b].z += pu[zz].z, u[b].w += pu[zz].w;
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < TG_EB; ++b) {
            const int g = g0 + b * TG_THREADS;
            if (g >= g_hi || tg_err) continue;
            const int r = g / per_row, c4 = g % per_row;
            const int m = m0 + r, n = oc0 + 4 * c4;
            if (m >= a.T) continue;
            float e[4] = {v[b].x, v[b].y, v[b].z, v[b].w};
            if (glu) {
                e[0] = silu(v[b].x) * u[b].x;
                e[1] = silu(v[b].y) * u[b].y;
                e[2] = silu(v[b].z) * u[b].z;
                e[3] = silu(v[b].w) * u[b].w;
            }
            float* orow = a.out + (size_t)m * a.ldo;
            if (n + 3 < ncols && vec_out && vec_res) {
                if (a.mode == 1) {
                    e[0] += q[b].x, e[1] += q[b].y, e[2] += q[b].z, e[3] += q[b].w;
                } else if (a.mode == 2) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) e[k] += __ldg(a.bias + n + k);
                }
                *reinterpret_cast<float4*>(orow + n) = make_float4(e[0], e[1], e[2], e[3]);
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (n + k >= ncols) break;
                    float val = e[k];
                    if (a.mode == 1) val += __ldcg(a.resid + (size_t)m * a.ldr + n + k);
                    if (a.mode == 2) val += __ldg(a.bias + n + k);
                    orow[n + k] = val;
                }
            }
        }
    }
    if (tid == 0) {
        stamp_max(a.ts ? a.ts + 7 : nullptr);
        // no copy may still be landing when the CTA exits (only reachable
        // after a timed-out wait; these phases are complete otherwise)
        for (int i = nloc > TG_STAGES ? nloc - TG_STAGES : 0; i < nloc; ++i)
            mbar_wait(&full[i % TG_STAGES], (uint32_t)(i / TG_STAGES) & 1u, a.err);
        if (tg_err && a.err != nullptr) atomicExch(a.err, 1);
    }
    // peers may still read this CTA's tile
    if (split) asm volatile("barrier.cluster.arrive.relaxed.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    // release tensor memory
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TG_TMEM_COLS)
                     : "memory");
    if (tid == 0) stamp_max(a.ts ? a.ts + 3 : nullptr);
}

namespace {
int tg_n_sm = 148;
int tg_max_clusters[TG_MAX_SPLITS + 1];  // resident clusters of (1, 1, c) CTAs
PFN_cuTensorMapEncodeTiled_v12000 tg_encode = nullptr;

// 2-D map over rows x inner FP32 values (row stride ld floats), box
// 32 x box_rows, 128-byte swizzle, zero fill outside.
bool tg_map(CUtensorMap* m, const float* p, int inner, int rows, int ld, int box_rows) {
    if (rows <= 0) return true;  // segment not present: never read
    if ((reinterpret_cast<uintptr_t>(p) & 15) != 0 || (ld & 3) != 0) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    const cuuint32_t box[2] = {(cuuint32_t)TG_BK, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return tg_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

template <typename Kern>
int tg_clusters(Kern* kern, size_t smem, int c) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, c);
    cfg.blockDim = dim3(TG_THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = c;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    return n;
}

cudaError_t tgemm_prepare() {
    static bool done = false;
    if (done) return cudaSuccess;
    cudaError_t e = set_smem_attrs(tgemm_kernel<false>, TG_SMEM);
    if (e == cudaSuccess) e = set_smem_attrs(tgemm_kernel<true>, TG_SMEM);
    if (e != cudaSuccess) return e;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&tg_encode), cudaEnableDefault,
                                &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || tg_encode == nullptr) {
        cudaGetLastError();
        return cudaErrorNotSupported;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&tg_n_sm, cudaDevAttrMultiProcessorCount, dev);
    tg_max_clusters[1] = tg_n_sm;
    for (int c = 2; c <= TG_MAX_SPLITS; ++c) {
        tg_max_clusters[c] = tg_clusters(tgemm_kernel<false>, TG_SMEM, c);
    }
    done = true;
    return cudaSuccess;
}

// Split-K factor: a.splits when given (clamped to 1..8 and the stage count),
// else the most splits (<= 8, >= 4 stages each) for which one cluster per
// tile is resident at once.
int tgemm_splits(const GemmArgs& a) {
    const int* mc = tg_max_clusters;
    const int tiles = ((a.N + TG_BN - 1) / TG_BN) * ((a.T + TG_BM - 1) / TG_BM);
    const int nst = a.K / TG_BK;
    const int min_stages = 4;
    int ks;
    if (a.splits > 0) {
        ks = a.splits < TG_MAX_SPLITS ? a.splits : TG_MAX_SPLITS;
        if (ks > nst) ks = nst;
        while (ks > 1 && mc[ks] < 1) --ks;
        return ks < 1 ? 1 : ks;
    }
    ks = tg_n_sm / tiles;
    if (ks > nst / min_stages) ks = nst / min_stages;
    if (ks > TG_MAX_SPLITS) ks = TG_MAX_SPLITS;
    while (ks > 1 && mc[ks] < tiles) --ks;
    return ks < 1 ? 1 : ks;
}

// K a multiple of 32; X, W and the row strides 16-byte aligned; SwiGLU
// (interleave) needs N a multiple of 128, row segments start at multiples of
// 128.
cudaError_t tgemm_launch(const GemmArgs& a, cudaStream_t s, bool pdl) {
    const cudaError_t pe = tgemm_prepare();
    if (pe != cudaSuccess) return pe;
    if (a.K % TG_BK != 0 || a.K <= 0 || a.T <= 0 || a.N <= 0) return cudaErrorInvalidValue;
    // the FFMA kernel up to 16 rows (measured: at 32 rows the tcgen05 tile wins)
    if (a.variant == 2 || (a.variant == 0 && a.T <= 16 && fgemm_supported(a))) return fgemm_launch(a, s, pdl);
    TgMaps tm;
    memset(&tm, 0, sizeof tm);
    bool ok = tg_map(&tm.a, a.A, a.K, a.T, a.lda, TG_BM);
    if (a.interleave) {
        ok = ok && a.N % TG_BN == 0 && a.mode == 3;
        ok = ok && tg_map(&tm.w[0], a.w0, a.K, a.N / 2, a.K, TG_BN / 2);
        ok = ok && tg_map(&tm.w[1], a.w1, a.K, a.N / 2, a.K, TG_BN / 2);
    } else {
        ok = ok && a.mode != 3;
        const int s1 = a.seg1 < a.N ? a.seg1 : a.N, s2 = a.seg2 < a.N ? a.seg2 : a.N;
        ok = ok && (s1 == a.N || s1 % TG_BN == 0) && (s2 == a.N || s2 % TG_BN == 0) && s1 <= s2;
        ok = ok && tg_map(&tm.w[0], a.w0, a.K, s1, a.K, TG_BN);
        ok = ok && tg_map(&tm.w[1], a.w1, a.K, s2 - s1, a.K, TG_BN);
        ok = ok && tg_map(&tm.w[2], a.w2, a.K, a.N - s2, a.K, TG_BN);
    }
    if (!ok) return cudaErrorInvalidValue;
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
    return a.T < TG_BM ? cudaLaunchKernelEx(&cfg, tgemm_kernel<true>, a, tm) : cudaLaunchKernelEx(&cfg, tgemm_kernel<false>, a, tm);
}

}  // namespace skb
