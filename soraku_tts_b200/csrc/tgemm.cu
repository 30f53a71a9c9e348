// FP32 GEMM on the 5th-generation tensor cores with 3xTF32:
//   out[m][n] = epilogue( sum_k X[m][k] * W(n)[k] )
// for the prefill and for batched decode (more rows than the ring GEMV
// serves).  X [M][K] and W [N][K] are both K-major, as stored.
//
// 3xTF32: every operand x is split into big = x with its 13 low mantissa
// bits cleared (exactly a TF32 value) and small = x - big (exact in FP32);
// the product is big*big + big*small + small*big, accumulated in FP32 in
// tensor memory.  The dropped small*small term and the TF32 truncation of
// `small` leave a relative error around 2^-21 per product: FP32 parity within
// the 1e-4 tolerance.
//
// CTA tile 128 (rows of X) x 64 (rows of W), K in stages of 32.  All 256
// threads load a stage with coalesced 128-bit loads (8 threads per 128-byte
// row segment), split it, and store big and small tiles into shared memory in
// the K-major 128-byte-swizzle layout the MMA reads (row r of a tile at
// (r/8)*1024 + (r%8)*128, its 16-byte chunk c at slot c ^ (r%8)).  One thread
// issues the stage's 12 tcgen05.mma (4 k-steps of 8 x 3 products, M=128,
// N=64, kind::tf32) and commits them to the stage buffer's mbarrier; two
// buffers let the next stage's loads overlap the MMAs.  The epilogue reads
// the 128 x 64 FP32 accumulator with tcgen05.ld (warp w: TMEM lanes
// 32*(w%4).., columns 32*(w/4)..) and applies store / residual / bias /
// SwiGLU (interleaved gate, up rows).
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
constexpr int TG_STAGE = 2 * TG_A_BYTES + 2 * TG_B_BYTES;  // big + small of A and B
constexpr int TG_STAGES = 2;
constexpr size_t TG_SMEM = 1024 /* alignment slack */ + (size_t)TG_STAGES * TG_STAGE + 64;

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

__device__ __forceinline__ void tg_split_store(unsigned char* tile_big, unsigned char* tile_small, int r, int c,
                                               float4 v) {
    const uint32_t off = (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u + (uint32_t)((c ^ (r & 7)) * 16);
    float4 b, s;
    b.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
    b.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
    b.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
    b.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
    s.x = v.x - b.x;
    s.y = v.y - b.y;
    s.z = v.z - b.z;
    s.w = v.w - b.w;
    *reinterpret_cast<float4*>(tile_big + off) = b;
    *reinterpret_cast<float4*>(tile_small + off) = s;
}

__device__ __forceinline__ const float* tg_wrow(const GemmArgs& a, int n) {
    if (a.interleave) return ((n & 1) ? a.w1 : a.w0) + (size_t)(n >> 1) * a.K;
    if (n < a.seg1) return a.w0 + (size_t)n * a.K;
    if (n < a.seg2) return a.w1 + (size_t)(n - a.seg1) * a.K;
    return a.w2 + (size_t)(n - a.seg2) * a.K;
}

__global__ void __launch_bounds__(TG_THREADS) tgemm_kernel(const GemmArgs a) {
    extern __shared__ unsigned char tg_raw[];
    // 1024-byte aligned stage buffers (the swizzle pattern repeats every 1024 B)
    unsigned char* base = tg_raw + ((1024u - (smem_u32(tg_raw) & 1023u)) & 1023u);
    uint64_t* mma_bar = reinterpret_cast<uint64_t*>(base + TG_STAGES * TG_STAGE);  // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + TG_STAGES);
    __shared__ int tg_err;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * TG_BN, m0 = blockIdx.y * TG_BM;
    const int nst = a.K / TG_BK;

    if (tid == 0) {
        for (int s = 0; s < TG_STAGES; ++s) mbar_init(&mma_bar[s], 1);
        mbar_fence_init();
        tg_err = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TG_BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    pdl_wait();
    pdl_trigger();

    // loader mapping: 6 chunks of 16 B per thread per stage; chunk t < 1024 is
    // X row t/8, t >= 1024 is W row (t-1024)/8; 16-byte column t%8
    for (int st = 0; st < nst; ++st) {
        const int buf = st & 1;
        unsigned char* sb = base + buf * TG_STAGE;
        unsigned char* a_big = sb;
        unsigned char* a_small = sb + TG_A_BYTES;
        unsigned char* b_big = sb + 2 * TG_A_BYTES;
        unsigned char* b_small = b_big + TG_B_BYTES;
        float4 v[6];
        const int k0 = st * TG_BK;
#pragma unroll
        for (int j = 0; j < 6; ++j) {
            const int t = tid + TG_THREADS * j;
            const int c = t & 7;
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < 1024) {
                const int r = t >> 3, m = m0 + r;
                if (m < a.T) x = ld_cg4(reinterpret_cast<const float4*>(a.A + (size_t)m * a.lda + k0) + c);
            } else {
                const int r = (t - 1024) >> 3, n = n0 + r;
                if (n < a.N) x = ldg_stream(reinterpret_cast<const float4*>(tg_wrow(a, n) + k0) + c);
            }
            v[j] = x;
        }
        // the buffer's previous MMAs (stage st - 2) must be done reading it
        if (st >= TG_STAGES && !mbar_wait(&mma_bar[buf], (uint32_t)((st - TG_STAGES) / TG_STAGES) & 1u, a.err))
            tg_err = 1;
#pragma unroll
        for (int j = 0; j < 6; ++j) {
            const int t = tid + TG_THREADS * j;
            const int c = t & 7;
            if (t < 1024)
                tg_split_store(a_big, a_small, t >> 3, c, v[j]);
            else
                tg_split_store(b_big, b_small, (t - 1024) >> 3, c, v[j]);
        }
        // generic-proxy stores -> visible to the tensor core (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t ab = smem_u32(a_big), as_ = smem_u32(a_small);
            const uint32_t bb = smem_u32(b_big), bs = smem_u32(b_small);
#pragma unroll
            for (int kk = 0; kk < TG_BK / 8; ++kk) {
                const uint32_t o = kk * 32;  // 8 TF32 = 32 bytes along K
                umma_tf32(tmem, umma_desc_sw128(ab + o), umma_desc_sw128(bb + o), st > 0 || kk > 0);
                umma_tf32(tmem, umma_desc_sw128(ab + o), umma_desc_sw128(bs + o), true);
                umma_tf32(tmem, umma_desc_sw128(as_ + o), umma_desc_sw128(bb + o), true);
            }
            umma_commit(&mma_bar[buf]);
        }
    }
    // all MMAs done: the last stage's commit covers every earlier MMA
    if (nst > 0) {
        const int last = nst - 1;
        if (!mbar_wait(&mma_bar[last & 1], (uint32_t)(last / TG_STAGES) & 1u, a.err)) tg_err = 1;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    // epilogue: warp w reads TMEM lanes 32*(w%4).. (tile rows) and columns 32*(w/4)..
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
    const int m = m0 + 32 * rq + lane;
    const int nb = n0 + 32 * ch;
    if (m < a.T && !tg_err) {
        if (a.mode == 3) {  // SwiGLU over (gate, up) column pairs
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
                const int n = nb + j;
                if (n + 1 < a.N)
                    a.out[(size_t)m * a.ldo + (n >> 1)] = silu(__uint_as_float(r32[j])) * __uint_as_float(r32[j + 1]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int n = nb + j;
                if (n < a.N) {
                    float val = __uint_as_float(r32[j]);
                    if (a.mode == 1) val += __ldcg(a.resid + (size_t)m * a.ldr + n);
                    if (a.mode == 2) val += __ldg(a.bias + n);
                    a.out[(size_t)m * a.ldo + n] = val;
                }
            }
        }
    }
    if (tg_err && tid == 0 && a.err != nullptr) atomicExch(a.err, 1);
    // release the accumulator
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TG_BN) : "memory");
}

cudaError_t tgemm_prepare() { return set_smem_attrs(tgemm_kernel, TG_SMEM); }

// K a multiple of 32, 16-byte aligned rows.
cudaError_t tgemm_launch(const GemmArgs& a, cudaStream_t s, bool pdl) {
    static bool prepared = false;
    if (!prepared) {
        const cudaError_t e = tgemm_prepare();
        if (e != cudaSuccess) return e;
        prepared = true;
    }
    if (a.K % TG_BK != 0 || a.K <= 0 || a.T <= 0 || a.N <= 0) return cudaErrorInvalidValue;
    return launch(tgemm_kernel, dim3((a.N + TG_BN - 1) / TG_BN, (a.T + TG_BM - 1) / TG_BM), dim3(TG_THREADS),
                  TG_SMEM, s, pdl, a);
}

}  // namespace skb
