// FP32 GEMV for decode: out[m, n] = epilogue(sum_k x[m, k] * W[n, k]), M <= 4
// activation rows, W row-major [N, K] (nn.Linear layout).
//
// Layout on the GPU.  CTA c owns the contiguous output rows
// [c*N/G, (c+1)*N/G) (G = grid), so its weight slice is one contiguous range
// per weight segment and the CTAs' shares differ by at most one row.  Before
// waiting on its predecessor (programmatic dependent launch) thread 0 stages
// the CTA's whole slice into shared memory with 1-D bulk copies (TMA engine),
// one mbarrier per chunk of RC rows, so every weight byte of the kernel is in
// flight at once.  Thread t owns the K-slice of float4 columns {t, t+256, ...}:
// it keeps x[m, slice] in registers and reads W[n, slice] from shared memory
// (conflict-free 128-bit loads).  The RC*M partial dot products of a chunk are
// reduced across the warp by a butterfly reduce-scatter and across the 8 warps
// through shared memory.
//
// Memory-bound: 4 bytes of weight per 2*M flops; no tensor cores (FP32
// parity with the reference's native path is required).
#pragma once

#include "common.cuh"

namespace skb {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

enum XMode : int {
    X_PLAIN = 0,          // x
    X_RMSNORM = 1,        // rmsnorm(x, nw, neps)
    X_ADD_RMSNORM = 2,    // rmsnorm(x + x2, nw, neps)
    X_NORM_ADD_NORM = 3,  // rmsnorm(rmsnorm(x, nw2, neps2) + x2, nw, neps)
};
enum EMode : int {
    E_STORE = 0,   // out = acc
    E_RESID = 1,   // out = acc + resid   (in place allowed: out == resid)
    E_BIAS = 2,    // out = acc + bias[n]
    E_SWIGLU = 3,  // logical rows interleave (gate_i, up_i): out[m, i] = silu(g) * u
};

struct GemvArgs {
    // weights: logical rows [0, N).  interleave: row 2i -> w0 row i, 2i+1 -> w1 row i.
    // otherwise rows [0, seg1) from w0, [seg1, seg2) from w1, [seg2, N) from w2.
    const float* w0;
    const float* w1;
    const float* w2;
    int seg1, seg2;
    int interleave;
    int N, K;
    // activations [M, K] with row strides
    const float* x;
    int ldx;
    const float* x2;   // addend for X_ADD_RMSNORM / X_NORM_ADD_NORM
    int ldx2;
    int x2_div;        // x2 row = m / x2_div (prefix shared by the rows of a request)
    const float* nw;   // norm weight [K]
    float neps;
    const float* nw2;  // inner norm weight [K] (X_NORM_ADD_NORM)
    float neps2;
    float* xout;       // optional: CTA 0 stores the normed x [M, K] (ld = K)
    float* hout;       // optional: CTA 0 stores the inner-normed x (X_NORM_ADD_NORM)
    // epilogue
    float* out;
    int ldo;
    const float* resid;
    int ldr;
    const float* bias;
    int* inc;   // optional: CTA 0 adds 1 to inc[0 .. n_inc) after the wait (position counters)
    int n_inc;
    int* err;   // optional: set to 1 if a weight copy did not arrive
    PrefetchList pf;
    unsigned long long* ts;  // optional debug timeline [4] (see stamp_wait)
};

__device__ __forceinline__ const float* gemv_row(const GemvArgs& a, int r) {
    if (a.interleave) return ((r & 1) ? a.w1 : a.w0) + (size_t)(r >> 1) * a.K;
    if (r < a.seg1) return a.w0 + (size_t)r * a.K;
    if (r < a.seg2) return a.w1 + (size_t)(r - a.seg1) * a.K;
    return a.w2 + (size_t)(r - a.seg2) * a.K;
}

template <int M, int KV4>
struct GemvShape {
    static constexpr int RC0 = (KV4 == 1 ? 8 : (KV4 == 2 ? 4 : 2));
    static constexpr int RC = (RC0 * M > 32) ? (32 / M) : RC0;  // rows per chunk
    static constexpr int NV_RAW = RC * M;
    static constexpr int NV = NV_RAW <= 2 ? 2 : (NV_RAW <= 4 ? 4 : (NV_RAW <= 8 ? 8 : (NV_RAW <= 16 ? 16 : 32)));
};

// Block-wide sum of M values (one per row); every thread gets the results.
template <int M, class Sync = BlockSync>
__device__ __forceinline__ void block_sum_rows(float (&v)[M], float* red /* [GEMV_WARPS * M] */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int m = 0; m < M; ++m) v[m] = warp_sum(v[m]);
    Sync::sync();
    if (lane == 0) {
#pragma unroll
        for (int m = 0; m < M; ++m) red[warp * M + m] = v[m];
    }
    Sync::sync();
#pragma unroll
    for (int m = 0; m < M; ++m) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < GEMV_WARPS; ++w) s += red[w * M + m];
        v[m] = s;
    }
}

// Loads this thread's K-slice of the M activation rows, applying the norm
// prologue.  Columns beyond K read as zero.
template <int M, int KV4, int XM, class Sync = BlockSync>
__device__ __forceinline__ void gemv_load_x(const GemvArgs& a, float4 (&xv)[M][KV4], float* red) {
    const int tid = threadIdx.x;
    const int K4 = a.K >> 2;
#pragma unroll
    for (int m = 0; m < M; ++m) {
#pragma unroll
        for (int j = 0; j < KV4; ++j) {
            const int k4 = tid + j * GEMV_THREADS;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k4 < K4) v = ld_cg4(reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx) + k4);
            xv[m][j] = v;
        }
    }
    if (XM == X_PLAIN) return;
    if (XM == X_NORM_ADD_NORM) {
        // inner norm: h = rmsnorm(x, nw2, neps2)
        float ss[M];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < KV4; ++j)
                s += xv[m][j].x * xv[m][j].x + xv[m][j].y * xv[m][j].y + xv[m][j].z * xv[m][j].z +
                     xv[m][j].w * xv[m][j].w;
            ss[m] = s;
        }
        block_sum_rows<M, Sync>(ss, red);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float inv = rsqrtf(ss[m] / (float)a.K + a.neps2);
#pragma unroll
            for (int j = 0; j < KV4; ++j) {
                const int k4 = tid + j * GEMV_THREADS;
                if (k4 < K4) {
                    const float4 w = __ldg(reinterpret_cast<const float4*>(a.nw2) + k4);
                    float4 v = xv[m][j];
                    v.x = w.x * (v.x * inv);
                    v.y = w.y * (v.y * inv);
                    v.z = w.z * (v.z * inv);
                    v.w = w.w * (v.w * inv);
                    xv[m][j] = v;
                    if (a.hout != nullptr && blockIdx.x == 0)
                        reinterpret_cast<float4*>(a.hout + (size_t)m * a.K)[k4] = v;
                }
            }
        }
    }
    if (XM == X_ADD_RMSNORM || XM == X_NORM_ADD_NORM) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float* x2 = a.x2 + (size_t)(m / a.x2_div) * a.ldx2;
#pragma unroll
            for (int j = 0; j < KV4; ++j) {
                const int k4 = tid + j * GEMV_THREADS;
                if (k4 < K4) {
                    const float4 p = ld_cg4(reinterpret_cast<const float4*>(x2) + k4);
                    xv[m][j].x += p.x;
                    xv[m][j].y += p.y;
                    xv[m][j].z += p.z;
                    xv[m][j].w += p.w;
                }
            }
        }
    }
    float ss[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < KV4; ++j)
            s += xv[m][j].x * xv[m][j].x + xv[m][j].y * xv[m][j].y + xv[m][j].z * xv[m][j].z +
                 xv[m][j].w * xv[m][j].w;
        ss[m] = s;
    }
    block_sum_rows<M, Sync>(ss, red);
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const float inv = rsqrtf(ss[m] / (float)a.K + a.neps);
#pragma unroll
        for (int j = 0; j < KV4; ++j) {
            const int k4 = tid + j * GEMV_THREADS;
            if (k4 < K4) {
                const float4 w = __ldg(reinterpret_cast<const float4*>(a.nw) + k4);
                float4 v = xv[m][j];
                v.x = w.x * (v.x * inv);
                v.y = w.y * (v.y * inv);
                v.z = w.z * (v.z * inv);
                v.w = w.w * (v.w * inv);
                xv[m][j] = v;
                if (a.xout != nullptr && blockIdx.x == 0)
                    reinterpret_cast<float4*>(a.xout + (size_t)m * a.K)[k4] = v;
            }
        }
    }
}

// Dynamic shared memory: [GEMV_MAX_CHUNKS mbarriers | pad to 256 B | weight rows].
constexpr int GEMV_MAX_CHUNKS = 30;
constexpr int GEMV_SMEM_HEAD = 256;
constexpr size_t GEMV_SMEM_MAX = 220 * 1024;  // + ~2 KB static stays under the 227 KB opt-in limit

template <int M, int KV4, int XM, int EM>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(const GemvArgs a) {
    using S = GemvShape<M, KV4>;
    constexpr int RC = S::RC;
    constexpr int NV = S::NV;
    extern __shared__ __align__(128) unsigned char gsm[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(gsm);
    float* wsm = reinterpret_cast<float*>(gsm + GEMV_SMEM_HEAD);
    __shared__ float red[2][GEMV_WARPS][NV];
    __shared__ float nred[GEMV_WARPS * M];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x;
    // SwiGLU rows come in (gate, up) pairs: split pairs, not rows.
    const int unit = (EM == E_SWIGLU) ? 2 : 1;
    const int NU = a.N / unit;
    const int r0 = (int)((long long)blockIdx.x * NU / G) * unit;
    const int r1 = (int)((long long)(blockIdx.x + 1) * NU / G) * unit;
    const int K4 = a.K >> 2;
    const int nrows = r1 - r0;
    const int nch = (nrows + RC - 1) / RC;
    const uint32_t row_bytes = (uint32_t)a.K * 4u;
    if (nch > GEMV_MAX_CHUNKS) {  // the host sizes the grid so this never happens
        if (tid == 0 && a.err) atomicExch(a.err, 2);
        pdl_wait();
        pdl_trigger();
        return;
    }

    // Everything up to the PDL wait touches only weights: stage this CTA's whole
    // (contiguous) weight slice into shared memory with bulk copies, one
    // mbarrier per chunk of RC rows, and prefetch the next kernel's share into L2.
    if (tid == 0) {
        for (int c = 0; c < nch; ++c) mbar_init(&bars[c], 1);
        mbar_fence_init();
        for (int c = 0; c < nch; ++c) {
            const int rb = r0 + c * RC;
            const int re = min(rb + RC, r1);
            mbar_expect_tx(&bars[c], (uint32_t)(re - rb) * row_bytes);
            for (int r = rb; r < re; ++r)
                bulk_g2s(wsm + (size_t)(r - r0) * a.K, gemv_row(a, r), row_bytes, &bars[c]);
        }
        prefetch_share(a.pf, blockIdx.x, G);
    }
    __syncthreads();

    pdl_wait();
    pdl_trigger();
    if (a.inc != nullptr && blockIdx.x == 0 && tid < a.n_inc) atomicAdd(a.inc + tid, 1);

    float4 xv[M][KV4];
    gemv_load_x<M, KV4, XM>(a, xv, nred);

    bool ok = true;
    int buf = 0;
    for (int c = 0; c < nch; ++c) {
        const int base = r0 + c * RC;
        if (ok) ok = mbar_wait(&bars[c], 0, a.err);
        float acc[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) acc[i] = 0.f;
        if (ok) {
#pragma unroll
            for (int rc = 0; rc < RC; ++rc) {
                if (base + rc < r1) {
                    const float4* wr = reinterpret_cast<const float4*>(wsm + (size_t)(base + rc - r0) * a.K);
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
        }
        const float v = butterfly_reduce<NV>(acc, lane);
        constexpr int DUP = 32 / NV;  // lanes holding each value
        if ((lane & (DUP - 1)) == 0) red[buf][warp][lane / DUP] = v;
        __syncthreads();
        if (EM == E_SWIGLU) {
            if (tid < (RC / 2) * M) {
                const int p = tid / M, m = tid % M;
                const int rg = base + 2 * p;
                if (rg < r1) {
                    float g = 0.f, u = 0.f;
#pragma unroll
                    for (int w = 0; w < GEMV_WARPS; ++w) {
                        g += red[buf][w][(2 * p) * M + m];
                        u += red[buf][w][(2 * p + 1) * M + m];
                    }
                    a.out[(size_t)m * a.ldo + (rg >> 1)] = silu(g) * u;
                }
            }
        } else {
            if (tid < RC * M) {
                const int rc = tid / M, m = tid % M;
                const int r = base + rc;
                if (r < r1) {
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
    }
    if (!ok) {
        // a copy never arrived: wait (bounded) for every copy still in flight
        // into this CTA's shared memory before the CTA exits
        for (int c = 0; c < nch; ++c) mbar_wait(&bars[c], 0, nullptr);
    }
}

// Rows per CTA for N logical rows on G CTAs (pairs for SwiGLU).
inline int gemv_rows_per_cta(int N, int EM, int G) {
    const int unit = (EM == E_SWIGLU) ? 2 : 1;
    const int NU = N / unit;
    return ((NU + G - 1) / G) * unit;
}
inline size_t gemv_smem_bytes(int N, int K, int EM, int G) {
    return GEMV_SMEM_HEAD + (size_t)gemv_rows_per_cta(N, EM, G) * K * 4;
}
// Smallest grid >= want whose per-CTA slice fits in shared memory and whose
// chunk count fits the barrier array.
inline int gemv_grid(int N, int K, int EM, int want, int rc) {
    int G = want < 1 ? 1 : want;
    for (;;) {
        const int rows = gemv_rows_per_cta(N, EM, G);
        if (gemv_smem_bytes(N, K, EM, G) <= GEMV_SMEM_MAX && (rows + rc - 1) / rc <= GEMV_MAX_CHUNKS) return G;
        ++G;
    }
}

// Host-side dispatch over (M, KV4, XM, EM).  `grid` is the wanted CTA count;
// it grows if a CTA's slice would not fit in shared memory.  Returns a cudaError_t.
cudaError_t gemv_launch(const GemvArgs& a, int M, int XM, int EM, int grid, cudaStream_t stream,
                        bool pdl);
// Sets the dynamic shared-memory limit of every instantiation (call before
// stream capture).
cudaError_t gemv_prepare_all();

}  // namespace skb
