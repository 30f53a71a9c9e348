// Op surface of the reference's TileLang module, as sm_100a kernels behind the
// C ABI of include/soraku_b200.h, plus the standalone fused sampler and the
// test hooks.  Argument meaning and order follow
// soraku_inference/acceleration/tilelang_kernels.py line for line.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"
#include "gemv.cuh"
#include "ops.cuh"
#include "sampler.cuh"
#include "trunk_api.cuh"

namespace skb {

static thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SKB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return SKB_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------------ rmsnorm
// out[b] = rmsnorm(x[b] (+ x2[b])) * w, one CTA per row.  Also used by prefill.
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float* __restrict__ x,
                                                           const float* __restrict__ x2,
                                                           const float* __restrict__ w,
                                                           float* __restrict__ out, int D,
                                                           float eps) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[8];
    const int b = blockIdx.x, tid = threadIdx.x;
    const float* xr = x + (size_t)b * D;
    const float* x2r = x2 ? x2 + (size_t)b * D : nullptr;
    float ss = 0.f;
    for (int i = tid; i < D; i += 256) {
        float v = xr[i];
        if (x2r) v += x2r[i];
        ss += v * v;
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float inv = rsqrtf(tot / (float)D + eps);
    float* o = out + (size_t)b * D;
    for (int i = tid; i < D; i += 256) {
        float v = xr[i];
        if (x2r) v += x2r[i];
        o[i] = w[i] * (v * inv);
    }
}

// Row norms of the batched decode path (more rows than the ring GEMV serves),
// one CTA per row, D <= 3072:
//   mode 1: xn = rmsnorm(x; nw, eps)
//   mode 3: h = rmsnorm(x; nw2, eps2) -> hout;  xn = rmsnorm(h + x2[row / x2_div]; nw, eps) -> xout
// (the same arithmetic as the ring GEMV's X_RMSNORM / X_NORM_ADD_NORM prologues).
__global__ void __launch_bounds__(256) norm_rows_kernel(const NormRowsArgs a) {
    if (threadIdx.x == 0) stamp_min(a.ts);
    pdl_wait();
    if (threadIdx.x == 0) stamp_wait(a.ts);
    pdl_trigger();
    __shared__ float red[8];
    constexpr int PT = 12;  // D / 256
    const int r = blockIdx.x, tid = threadIdx.x;
    float v[PT];
    const float* xr = a.x + (size_t)r * a.ldx;
#pragma unroll
    for (int j = 0; j < PT; ++j) {
        const int i = tid + 256 * j;
        v[j] = i < a.D ? __ldcg(xr + i) : 0.f;
    }
    auto inv_rms = [&](float eps) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < PT; ++j) ss += v[j] * v[j];
        ss = warp_sum(ss);
        __syncthreads();
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) t += red[w];
        return rsqrtf(t / (float)a.D + eps);
    };
    if (a.mode == 3) {
        const float inv = inv_rms(a.eps2);
        const float* x2 = a.x2 + (size_t)(r / a.x2_div) * a.ldx2;
#pragma unroll
        for (int j = 0; j < PT; ++j) {
            const int i = tid + 256 * j;
            if (i < a.D) {
                const float h = a.nw2[i] * (v[j] * inv);
                if (a.hout) a.hout[(size_t)r * a.D + i] = h;
                v[j] = h + __ldcg(x2 + i);
            }
        }
    }
    const float inv = inv_rms(a.eps);
#pragma unroll
    for (int j = 0; j < PT; ++j) {
        const int i = tid + 256 * j;
        if (i < a.D) {
            const float o = a.nw[i] * (v[j] * inv);
            a.xn[(size_t)r * a.D + i] = o;
            if (a.xout) a.xout[(size_t)r * a.D + i] = o;
        }
    }
    if (a.ts) {
        __syncthreads();
        if (tid == 0) stamp_max(a.ts + 3);
    }
}

int norm_rows(const NormRowsArgs& a, int rows, cudaStream_t s, bool pdl) {
    if (a.D > 3072 || rows < 1) return fail(SKB_ERR_ARG, "norm_rows: D %d rows %d", a.D, rows);
    cudaError_t e = launch(norm_rows_kernel, dim3(rows), dim3(256), 0, s, pdl, a);
    return e == cudaSuccess ? SKB_OK : fail(SKB_ERR_CUDA, "norm_rows: %s", cudaGetErrorString(e));
}

// Adds 1 to cnt[0 .. n).
__global__ void advance_kernel(int* cnt, int n) {
    pdl_wait();
    pdl_trigger();
    if ((int)threadIdx.x < n) cnt[threadIdx.x] += 1;
}

cudaError_t advance_launch(int* cnt, int n, cudaStream_t s, bool pdl) {
    return launch(advance_kernel, dim3(1), dim3(n < 32 ? 32 : ((n + 31) / 32) * 32), 0, s, pdl, cnt, n);
}

int rmsnorm_rows(const float* x, const float* x2, const float* w, float* out, int B, int D,
                 float eps, cudaStream_t s, bool pdl) {
    if (B <= 0) return SKB_OK;
    cudaError_t e = launch(rmsnorm_rows_kernel, dim3(B), dim3(256), 0, s, pdl, x, x2, w, out, D, eps);
    return e == cudaSuccess ? SKB_OK : fail(SKB_ERR_CUDA, "rmsnorm: %s", cudaGetErrorString(e));
}

// ------------------------------------------------------------- frame embed
// out[r, :] = scale * sum_{q in order} table[q, codes[r, q], :]
__global__ void __launch_bounds__(256) frame_embed_kernel(const int64_t* __restrict__ codes,
                                                          const float* __restrict__ table,
                                                          float* __restrict__ out, int Q, int V,
                                                          int D, float scale, int* err) {
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.y;
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i >= D) return;
    float acc = 0.f;
    for (int q = 0; q < Q; ++q) {
        long long c = codes[(size_t)r * Q + q];
        if (c < 0 || c >= V) {
            if (err) atomicExch(err, 1);
            c = 0;
        }
        const float v = table[((size_t)q * V + (size_t)c) * D + i];
        acc = (q == 0) ? v : acc + v;
    }
    out[(size_t)r * D + i] = acc * scale;
}

// -------------------------------------------------------------- prefix add
__global__ void __launch_bounds__(256) prefix_add_kernel(const float* __restrict__ prefix,
                                                         const float* __restrict__ table_q,
                                                         const int64_t* __restrict__ code,
                                                         float* __restrict__ out, int V, int D,
                                                         float scale) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i >= D) return;
    long long c = code[0];
    if (c < 0 || c >= V) c = 0;  // host validated; never index out of bounds
    out[(size_t)b * D + i] = prefix[(size_t)b * D + i] + table_q[(size_t)c * D + i] * scale;
}

// ----------------------------------------------------------- sampling prep
// tilelang_kernels.py:219-254: division (not reciprocal multiply), -1e30 masks.
__global__ void __launch_bounds__(256) sampling_prep_kernel(const float* __restrict__ logits,
                                                            const float* __restrict__ temperature,
                                                            const int32_t* __restrict__ mask_eos,
                                                            float* __restrict__ out, int V, int bos,
                                                            int pad, int eos) {
    pdl_wait();
    pdl_trigger();
    const int v = blockIdx.x * 256 + threadIdx.x;
    if (v >= V) return;
    float value = __fdiv_rn(logits[v], temperature[0]);
    if (v == bos) value = -1e30f;
    if (v == pad) value = -1e30f;
    if (mask_eos[0] > 0 && v == eos) value = -1e30f;
    out[v] = value;
}

// ----------------------------------------------------------- fused sampler
__global__ void __launch_bounds__(SAMPLER_THREADS) cfg_sample_kernel(
    const float* __restrict__ logits, int rows_per_req, int V, const skb_sample_params* params,
    int bos, int pad, int eos, int64_t* codes_out, float* uniform_out) {
    extern __shared__ __align__(16) unsigned char smem[];
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x;
    const skb_sample_params p = params[r];
    SampleJob J;
    J.cond = logits + (size_t)r * rows_per_req * V;
    J.uncond = rows_per_req > 1 ? J.cond + V : nullptr;
    J.V = V;
    J.cfg_scale = p.cfg_scale;
    J.temperature = p.temperature;
    J.top_p = p.top_p;
    J.top_k = p.top_k;
    J.mask_eos = p.mask_eos;
    J.bos = bos;
    J.pad = pad;
    J.eos = eos;
    J.u = philox_uniform(p.seed, p.request, p.frame, p.q);
    J.ts = nullptr;
    const int code = sample_one(J, smem);
    if (threadIdx.x == 0) {
        codes_out[r] = code;
        if (uniform_out) uniform_out[r] = J.u;
    }
}

__global__ void test_exp_kernel(const float* x, float* y, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = skb_exp(x[i]);
}

__global__ void test_philox_kernel(const uint32_t* ck, uint32_t* out, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t c[4] = {ck[6 * i], ck[6 * i + 1], ck[6 * i + 2], ck[6 * i + 3]};
    philox4x32_10(c, ck[6 * i + 4], ck[6 * i + 5]);
    for (int j = 0; j < 4; ++j) out[4 * i + j] = c[j];
}

int cfg_sample(const float* logits, int rows_per_req, int n_req, int V,
               const skb_sample_params* params, int bos, int pad, int eos, int64_t* codes,
               float* uniforms, cudaStream_t s, bool pdl) {
    static bool attr_set = false;
    if (!attr_set) {
        set_smem_attrs(cfg_sample_kernel, SAMPLER_SMEM);
        attr_set = true;
    }
    cudaError_t e = launch(cfg_sample_kernel, dim3(n_req), dim3(SAMPLER_THREADS), SAMPLER_SMEM, s,
                           pdl, logits, rows_per_req, V, params, bos, pad, eos, codes, uniforms);
    return e == cudaSuccess ? SKB_OK : fail(SKB_ERR_CUDA, "cfg_sample: %s", cudaGetErrorString(e));
}

// -------------------------------------------------------------- GEMV ops
// B rows are processed in blocks of at most 4 (the register-resident
// activation tile of gemv_kernel).
static int gemv_rows(GemvArgs a, int B, int XM, int EM, cudaStream_t s, const char* what) {
    // more than 4 rows: one pass of the 3xTF32 tensor-core GEMM over all of
    // them (the weights are read once), where its tiling accepts the shape
    if (B > 4 && XM == X_PLAIN && a.K % 32 == 0) {
        GemmArgs g = {};
        g.A = a.x;
        g.lda = a.ldx;
        g.w0 = a.w0;
        g.w1 = a.w1;
        g.w2 = a.w2;
        g.seg1 = a.seg1;
        g.seg2 = a.seg2;
        g.interleave = a.interleave;
        g.N = a.N;
        g.K = a.K;
        g.T = B;
        g.out = a.out;
        g.ldo = a.ldo;
        g.resid = a.resid;
        g.ldr = a.ldr;
        g.bias = a.bias;
        g.mode = EM == E_RESID ? 1 : (EM == E_BIAS ? 2 : (EM == E_SWIGLU ? 3 : 0));
        const cudaError_t e = tgemm_launch(g, s, false);
        if (e == cudaSuccess) return SKB_OK;
        if (e != cudaErrorInvalidValue) return fail(SKB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
        cudaGetLastError();  // a shape the tiling does not take: the ring GEMV below
    }
    int grid = a.N / (EM == E_SWIGLU ? 2 : 1);
    if (grid > 148) grid = 148;
    if (grid < 1) grid = 1;
    const float* x = a.x;
    float* out = a.out;
    const float* resid = a.resid;
    for (int b0 = 0; b0 < B;) {
        const int m = (B - b0) >= 4 ? 4 : ((B - b0) >= 2 ? 2 : 1);
        GemvArgs c = a;
        c.x = x + (size_t)b0 * a.ldx;
        c.out = out + (size_t)b0 * a.ldo;
        if (resid) c.resid = resid + (size_t)b0 * a.ldr;
        cudaError_t e = gemv_launch(c, m, XM, EM, grid, s, false);
        if (e != cudaSuccess) return fail(SKB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
        b0 += m;
    }
    return SKB_OK;
}

GemvArgs gemv_args_plain(const float* x, int ldx, int N, int K) {
    GemvArgs a = {};
    a.x = x;
    a.ldx = ldx;
    a.N = N;
    a.K = K;
    a.seg1 = a.seg2 = 1 << 30;
    a.x2_div = 1;
    return a;
}

// Failure-path hook: one thread waits, with a short limit, on an mbarrier
// phase that nothing completes (no copy is in flight), through the same
// bounded wait the decode kernels use; the wait gives up, sets *err and the
// kernel returns, leaving the context usable.
__global__ void test_wait_timeout_kernel(int* err, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
        mbar_wait_limit(&bar, 0u, err, limit_ns);
    }
}

}  // namespace skb

using namespace skb;

extern "C" {

const char* skb_last_error(void) { return g_err; }
int skb_abi_version(void) { return 5; }

int skb_add_rmsnorm(const float* hidden, const float* prefix, const float* weight, float* out,
                    int B, int D, float eps, cudaStream_t stream) {
    if (B < 0 || D <= 0 || !hidden || !prefix || !weight || !out)
        return fail(SKB_ERR_ARG, "add_rmsnorm: bad arguments (B=%d D=%d)", B, D);
    return rmsnorm_rows(hidden, prefix, weight, out, B, D, eps, stream, false);
}

int skb_rmsnorm(const float* x, const float* weight, float* out, int B, int D, float eps,
                cudaStream_t stream) {
    if (B < 0 || D <= 0 || !x || !weight || !out)
        return fail(SKB_ERR_ARG, "rmsnorm: bad arguments (B=%d D=%d)", B, D);
    return rmsnorm_rows(x, nullptr, weight, out, B, D, eps, stream, false);
}

static int check_gemv_shapes(const char* what, int B, int N, int K, const void* p0, const void* p1,
                             const void* p2, const void* p3) {
    if (B < 0 || N <= 0 || K <= 0) return fail(SKB_ERR_ARG, "%s: bad sizes B=%d N=%d K=%d", what, B, N, K);
    if (K % 4 != 0 || K > 3072)
        return fail(SKB_ERR_ARG, "%s: inner size %d must be a multiple of 4 and <= 3072", what, K);
    const void* ps[4] = {p0, p1, p2, p3};
    for (int i = 0; i < 4; ++i)
        if (ps[i] && !aligned16(ps[i])) return fail(SKB_ERR_ARG, "%s: pointer %d not 16-byte aligned", what, i);
    return SKB_OK;
}

int skb_swiglu_gemv(const float* x, const float* wg, const float* wu, float* out, int B, int I,
                    int D, cudaStream_t stream) {
    int st = check_gemv_shapes("swiglu_gemv", B, I, D, x, wg, wu, nullptr);
    if (st) return st;
    if (!out) return fail(SKB_ERR_ARG, "swiglu_gemv: null output");
    GemvArgs a = gemv_args_plain(x, D, 2 * I, D);
    a.w0 = wg;
    a.w1 = wu;
    a.interleave = 1;
    a.out = out;
    a.ldo = I;
    return gemv_rows(a, B, X_PLAIN, E_SWIGLU, stream, "swiglu_gemv");
}

int skb_down_residual_gemv(const float* act, const float* wd, const float* residual, float* out,
                           int B, int D, int I, cudaStream_t stream) {
    int st = check_gemv_shapes("down_residual_gemv", B, D, I, act, wd, nullptr, nullptr);
    if (st) return st;
    if (!out || !residual) return fail(SKB_ERR_ARG, "down_residual_gemv: null pointer");
    GemvArgs a = gemv_args_plain(act, I, D, I);
    a.w0 = wd;
    a.out = out;
    a.ldo = D;
    a.resid = residual;
    a.ldr = D;
    return gemv_rows(a, B, X_PLAIN, E_RESID, stream, "down_residual_gemv");
}

int skb_classifier_gemv(const float* body, const float* wq, const float* bias, float* out, int B,
                        int V, int D, cudaStream_t stream) {
    int st = check_gemv_shapes("classifier_gemv", B, V, D, body, wq, nullptr, nullptr);
    if (st) return st;
    if (!out || !bias) return fail(SKB_ERR_ARG, "classifier_gemv: null pointer");
    GemvArgs a = gemv_args_plain(body, D, V, D);
    a.w0 = wq;
    a.out = out;
    a.ldo = V;
    a.bias = bias;
    return gemv_rows(a, B, X_PLAIN, E_BIAS, stream, "classifier_gemv");
}

int skb_frame_embed(const int64_t* codes, const float* table, float* out, int R, int Q, int V,
                    int D, float scale, cudaStream_t stream) {
    if (R < 0 || Q <= 0 || V <= 0 || D <= 0 || !codes || !table || !out)
        return fail(SKB_ERR_ARG, "frame_embed: bad arguments");
    if (R == 0) return SKB_OK;
    cudaError_t e = launch(frame_embed_kernel, dim3((D + 255) / 256, R), dim3(256), 0, stream, false,
                           codes, table, out, Q, V, D, scale, (int*)nullptr);
    return e == cudaSuccess ? SKB_OK : fail(SKB_ERR_CUDA, "frame_embed: %s", cudaGetErrorString(e));
}

int skb_prefix_add(const float* prefix, const float* table_q, const int64_t* code, float* out,
                   int B, int V, int D, float scale, cudaStream_t stream) {
    if (B < 0 || V <= 0 || D <= 0 || !prefix || !table_q || !code || !out)
        return fail(SKB_ERR_ARG, "prefix_add: bad arguments");
    if (B == 0) return SKB_OK;
    cudaError_t e = launch(prefix_add_kernel, dim3((D + 255) / 256, B), dim3(256), 0, stream, false,
                           prefix, table_q, code, out, V, D, scale);
    return e == cudaSuccess ? SKB_OK : fail(SKB_ERR_CUDA, "prefix_add: %s", cudaGetErrorString(e));
}

int skb_sampling_prep(const float* logits, const float* temperature, const int32_t* mask_eos,
                      float* out, int V, int bos_id, int pad_id, int eos_id, cudaStream_t stream) {
    if (V <= 0 || !logits || !temperature || !mask_eos || !out)
        return fail(SKB_ERR_ARG, "sampling_prep: bad arguments");
    cudaError_t e = launch(sampling_prep_kernel, dim3((V + 255) / 256), dim3(256), 0, stream, false,
                           logits, temperature, mask_eos, out, V, bos_id, pad_id, eos_id);
    return e == cudaSuccess ? SKB_OK : fail(SKB_ERR_CUDA, "sampling_prep: %s", cudaGetErrorString(e));
}

int skb_cfg_sample(const float* logits, int rows_per_req, int n_req, int V,
                   const skb_sample_params* params, int bos_id, int pad_id, int eos_id,
                   int64_t* codes_out, float* uniform_out, cudaStream_t stream) {
    if (!logits || !params || !codes_out || n_req < 0 || V <= 0 || V > SAMPLER_VMAX ||
        (rows_per_req != 1 && rows_per_req != 2))
        return fail(SKB_ERR_ARG, "cfg_sample: bad arguments (V=%d rows_per_req=%d, V <= %d)", V,
                    rows_per_req, SAMPLER_VMAX);
    if (n_req == 0) return SKB_OK;
    return cfg_sample(logits, rows_per_req, n_req, V, params, bos_id, pad_id, eos_id, codes_out,
                      uniform_out, stream, false);
}

int skb_test_exp(const float* x, float* y, int n, cudaStream_t stream) {
    if (n < 0 || (n > 0 && (!x || !y))) return fail(SKB_ERR_ARG, "test_exp: bad arguments");
    if (n == 0) return SKB_OK;
    test_exp_kernel<<<(n + 255) / 256, 256, 0, stream>>>(x, y, n);
    return check_launch("test_exp");
}

int skb_test_wait_timeout(int* err, int limit_us, cudaStream_t stream) {
    if (!err || limit_us < 1 || limit_us > 1000000) return fail(SKB_ERR_ARG, "test_wait_timeout: bad arguments");
    test_wait_timeout_kernel<<<1, 32, 0, stream>>>(err, (unsigned long long)limit_us * 1000ull);
    int st = check_launch("test_wait_timeout");
    if (st != SKB_OK) return st;
    cudaError_t e = cudaStreamSynchronize(stream);
    int flag = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&flag, err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail(SKB_ERR_CUDA, "test_wait_timeout: %s", cudaGetErrorString(e));
    if (flag != 0) return fail(SKB_ERR_CUDA, "a device wait gave up after %d us and raised its error flag", limit_us);
    return SKB_OK;
}

int skb_test_philox(const uint32_t* ctr_key, uint32_t* out, int n, cudaStream_t stream) {
    if (n < 0 || (n > 0 && (!ctr_key || !out))) return fail(SKB_ERR_ARG, "test_philox: bad arguments");
    if (n == 0) return SKB_OK;
    test_philox_kernel<<<(n + 255) / 256, 256, 0, stream>>>(ctr_key, out, n);
    return check_launch("test_philox");
}

}  // extern "C"
