// Decode GEMV interface: out[m, n] = epilogue(sum_k x[m, k] * W[n, k]) for
// M <= 4 activation rows, W row-major [N, K] (nn.Linear layout), with the
// fused norm prologues and epilogues the frame needs.  The kernel is the
// ring-streamed GEMV of rgemv.cuh.
//
// Memory-bound: 4 bytes of weight per 2*M flops; no tensor cores (FP32
// parity with the reference's native path is required).
#pragma once

#include "common.cuh"

namespace skb {

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
    unsigned long long* ts;  // optional debug timeline [SKB_KTS_STRIDE] (see stamp_wait)
};

// Host-side dispatch over (M, inner size, XM, EM) of the ring GEMV
// (rgemv.cuh).  `grid` is the wanted CTA count (at most one CTA per unit).
// Returns a cudaError_t.
cudaError_t gemv_launch(const GemvArgs& a, int M, int XM, int EM, int grid, cudaStream_t stream,
                        bool pdl);
// Sets the dynamic shared-memory limit of every instantiation (call before
// stream capture).
cudaError_t gemv_prepare_all();

}  // namespace skb
